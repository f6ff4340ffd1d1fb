// fdb_internal.h -- internal declarations shared by the engine's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <functional>
#include <mutex>
#include <stdexcept>
#include <string>

#include "fastdec_b200.h"

namespace fdb {

// ---------------------------------------------------------------- errors
struct Error : public std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define FDB_CUDA(call)                                                                         \
    do {                                                                                       \
        cudaError_t fdb_e_ = (call);                                                           \
        if (fdb_e_ != cudaSuccess)                                                             \
            throw ::fdb::Error(fdb_e_ == cudaErrorMemoryAllocation ? FDB200_ENOMEM : FDB200_ECUDA, \
                               std::string(#call) + " failed: " + cudaGetErrorString(fdb_e_) + \
                                   " (" __FILE__ ":" + std::to_string(__LINE__) + ")");       \
    } while (0)

extern thread_local long long g_launches;   // kernels launched by this thread (for FdB200Stats)
#define FDB_LAUNCHED()                                                                         \
    do {                                                                                       \
        ++::fdb::g_launches;                                                                   \
        FDB_CUDA(cudaGetLastError());                                                          \
    } while (0)

#define FDB_REQUIRE(cond, msg)                                                                 \
    do {                                                                                       \
        if (!(cond)) throw ::fdb::Error(FDB200_EINVAL, (msg));                                 \
    } while (0)

// ---------------------------------------------------------------- constants
constexpr int kBlock = 128;              // points per triangle block (rows and columns of a tile)
constexpr uint64_t kEmptyKey = ~0ull;    // an empty list slot; greater than every real entry

// ---------------------------------------------------------------- device workspace
// Grow-only device allocation, kept across calls on one device.
struct DevBuf {
    void* ptr = nullptr;
    size_t bytes = 0;
    void* ensure(size_t need);
    void release();
    template <typename T> T* as(size_t count) { return static_cast<T*>(ensure(count * sizeof(T))); }
};

struct Workspace {
    int device = 0;
    std::mutex mu;
    cudaStream_t own_stream = nullptr;
    int* pinned = nullptr;                 // small pinned host scratch for flags / counters
    DevBuf data, norms, lists, thr, fthr, cand, cnt, flags;
    DevBuf dist, idx, den, parent, cores, scan, mean_tmp, dc_tmp, dc_sel, labels_tmp, misc, ops, misc2, spill;
    void release_all();
};

Workspace& workspace(int device);

// Runs fn with the workspace of opts->device locked and the device current; converts exceptions
// into status codes and records the message.
int guarded(const FdB200Opts* opts, FdB200Opts* resolved, Workspace** ws_out,
            const std::function<void(Workspace&, const FdB200Opts&, cudaStream_t)>& fn);
void set_last_error(const std::string& msg);
extern thread_local int last_call_launches;   // kernels launched by the last guarded call

// Event-based stage timer on one stream.
struct StageTimer {
    cudaStream_t s;
    cudaEvent_t ev[32];
    int n = 0;
    explicit StageTimer(cudaStream_t st);
    ~StageTimer();
    int mark();                        // records an event, returns its slot
    double ms(int a, int b);           // elapsed between two marks (synchronises on b)
};

// ---------------------------------------------------------------- kNN
struct KnnConfig {
    int n = 0, d = 0, k = 0;
    int ldx = 0;                 // leading dimension (elements) of the dim-major dataset
    int precision = FDB200_FP32;
    int engine = FDB200_ENGINE_AUTO;
    int shard_rank = 0, shard_count = 1;
    int block_lo = -1, block_hi = -1;   // explicit row-block range of the shard (-1: from rank / count)
    int cand_capacity = 0;
    fdb200_round_hook round_hook = nullptr;   // symmetric shards: thresholds combined between rounds
    void* round_hook_ctx = nullptr;
};

struct KnnResult {
    uint64_t* lists = nullptr;   // n * k packed (d2 bits << 32 | index), point-major, ascending
    long long pairs = 0, candidates = 0;
    int rounds = 0, overflow_reruns = 0, engine_used = FDB200_ENGINE_SIMT;
    double tile_ms = 0.0;
};

// x: dim-major dataset on the device. Fills ws.lists.
KnnResult knn_lists(Workspace& ws, const float* x, const KnnConfig& cfg, cudaStream_t s);

// rank-major sqrt'd distances + indices from packed lists
void lists_to_rank_major(const uint64_t* lists, int n, int k, float* dist, int* idx, cudaStream_t s);

// dst (n*k) <- k-smallest of dst and nsrc blocks of n*k lists in srcs
void merge_list_blocks(Workspace& ws, uint64_t* dst, const uint64_t* srcs, int nsrc, int n, int k,
                       cudaStream_t s);

void compute_norms(const float* x, int ldx, int n, int d, float* norms, cudaStream_t s);

// true when the tcgen05 tile engine can run this shape on the current device
bool tc_engine_supported(int d);
// where the list merge writes each point's folded filter bound for the tcgen05 engine: the A
// operand image (w parts of every row) and the TF32 norms the fold needs
struct TcFold {
    unsigned char* aimg = nullptr;
    const float* ntf = nullptr;
    int sym = 0;   // 1: symmetric schedule (unfolded rows, strict bounds in U)
};
// builds the tcgen05 operand images (pre-swizzled augmented rows) and the exact point-major copy;
// sym selects the symmetric schedule's unfolded row image
TcFold tc_prepare(Workspace& ws, const float* x, int ldx, int n, int d, const float* norms, const float* U,
                  const uint64_t* thr, int sym, cudaStream_t s);

// filter audit (diagnostics): raw tcgen05 accumulators of every ordered pair with the thresholds thr_d2
// folded in, the folded bounds V, and the operand images row by row (n x kp each)
void tc_filter_audit(Workspace& ws, const float* x, int n, int d, const float* thr_d2, int precision, float* acc,
                     float* V, float* arows, float* brows, cudaStream_t s);

// ---------------------------------------------------------------- density / detection
// Sequential-order double mean of the first k ranks (rank stride n) -- bit-identical to the
// host loop fastdecbase.cpp:257-274. Result left in *mean_dev.
void exact_mean(Workspace& ws, const float* dist_rm, int n, int k, double* mean_dev, cudaStream_t s);
// The same mean with its working memory supplied by the caller (no workspace, no allocation).
// mean_scratch_bytes(n) is the space it needs: two doubles per 32-point chunk plus the binade-map
// tree (32 bytes per map, one level per factor of 32).
constexpr size_t mean_scratch_bytes(long long n)
{
    const long long nchunks = (n + 31) / 32;
    long long maps = nchunks, c = nchunks;
    while (c > 1) {
        c = (c + 31) / 32;
        maps += c;
    }
    return (size_t)(16 * nchunks + 16 + 32 * maps + 256);
}
void exact_mean_in(void* scratch, size_t scratch_bytes, const float* dist_rm, int n, int k, double* mean_dev,
                   cudaStream_t s);
void density_from_mean(const float* dist_rm, int n, int k, int gaussian, const double* mean_dev,
                       float* den, cudaStream_t s);
// loads the kernels of the two calls above on the current device (CUDA loads kernels lazily, at their
// first launch, otherwise)
void preload_mean_density_kernels();
// parent + ordered core list; returns the core count (synchronises on s)
int dc_detection(Workspace& ws, const int* idx_rm, const float* den, int n, int k, int* parent,
                 int* cores, cudaStream_t s);

// ---------------------------------------------------------------- DC reduction / labels
// Outputs core_parent (device, core_nb), centers (device, num_centers).
void dc_reduction(Workspace& ws, const float* x, int ldx, int n, int d, const float* norms,
                  const float* den, const int* cores, int core_nb, int num_centers,
                  int* core_parent, int* centers, cudaStream_t s);
void scatter_core_parents(const int* cores, const int* core_parent, int core_nb, int* parent,
                          cudaStream_t s);
// The same reduction split by point ranges (for sharding it across GPUs): stage 0 writes best[c] = the
// lexicographic minimum (d2 bits << 32 | index) over the strictly denser points of [p_lo, p_hi)
// (UINT64_MAX if none); stage 1 writes rank[c] = the points of [p_lo, p_hi) closer to core c than the
// parent in best[c]. Keys of several ranges combine by minimum, ranks by sum; dc_select then finishes
// (parents, delta, fills, center selection) from the combined arrays.
void dc_stage_range(Workspace& ws, int stage, const float* x, int ldx, int n, int d, const float* norms,
                    const float* den, const int* cores, int core_nb, int p_lo, int p_hi, uint64_t* best, int* rank,
                    cudaStream_t s);
void dc_select(Workspace& ws, const float* den, const int* cores, int core_nb, const uint64_t* best, const int* rank,
               int num_centers, int* core_parent, int* centers, cudaStream_t s);
// labels on the device; throws Error(FDB200_ECYCLE) if the parent graph has a cycle
void final_cluster(Workspace& ws, const int* parent, int n, const int* centers, int c, int* labels,
                   cudaStream_t s);

}  // namespace fdb
