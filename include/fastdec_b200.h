/*
 * fastdec_b200.h -- C ABI of the B200 FastDEC engine (libfastdec_b200.so).
 *
 * Plain pointers and sizes only; no exceptions cross this boundary. Every call returns
 * FDB200_OK (0) or a negative FDB200_E* code; fdb200_last_error() gives the message for the
 * calling thread's last failure. Each entry point names the reference interface it replaces
 * (paths inside cyberbull66/symwarp-fastdec).
 *
 * Data layout is the reference's: the dataset is DIM-MAJOR, element (dim t, point i) at
 * data[t * n + i] (test.cpp:110-115, dataset.h:8-39). kNN outputs are RANK-MAJOR, element
 * (point i, rank q) at [q * n + i] (symtriknncuda.h:11-12, helper.cpp:295-317).
 *
 * Pointers are host pointers unless FdB200Opts.inputs_on_device / outputs_on_device say they
 * are device pointers on FdB200Opts.device.
 */
#ifndef FASTDEC_B200_H
#define FASTDEC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FDB200_ABI_VERSION 3

enum {
    FDB200_OK = 0,
    FDB200_EINVAL = -1,      /* bad argument (the reference returns false / throws) */
    FDB200_ECUDA = -2,       /* a CUDA runtime call failed */
    FDB200_ENOMEM = -3,      /* device allocation failed */
    FDB200_ECORES = -4,      /* "Fit: not enough core points" (fastdecbase.cpp:188-191) */
    FDB200_ECYCLE = -5,      /* label propagation did not converge (symwarpfastdeccuda.cu:338-339) */
    FDB200_EINTERNAL = -6    /* an internal consistency check failed */
};

/*
 * Environment variables the library reads:
 *   FDB200_TRACE=1                            per-round tile statistics on stderr (diagnostics).
 *   FDB200_FAULT_INJECT=withhold_row_copy     TEST-ONLY failure injection. Read once per process: the
 *       first tcgen05 tile launch of the process withholds one shared-memory copy in every CTA, its
 *       bounded waits run out after about a second, and that call returns FDB200_EINTERNAL; every
 *       later call runs normally. Never set it in production.
 */

enum { FDB200_FP32 = 0, FDB200_TF32 = 1 };              /* distance precision */
enum { FDB200_LAPLACIAN = 0, FDB200_GAUSSIAN = 1 };    /* density kernel (USE_GAUSSIAN_KERNEL) */
enum { FDB200_ENGINE_AUTO = 0, FDB200_ENGINE_SIMT = 1, FDB200_ENGINE_TCGEN05 = 2 };

/*
 * Round hook of a symmetric sharded kNN (fdb200_knn_partial with round_hook set). Between the rounds
 * of the triangle the library asks the caller to combine two small device arrays over all shards,
 * on `stream`, and returns without waiting: the caller enqueues the combination (an NCCL all-reduce,
 * say) on that stream and returns. kind FDB200_HOOK_FLAGS: `count` int32 flags (the round's overflow
 * tag and error code) to combine by MAX, before the round's list merge, so that every shard discards
 * and re-plans an overflowed round alike. kind FDB200_HOOK_THRESHOLDS: `count` packed uint64 per-point
 * thresholds (see fdb200_knn_partial) to combine by unsigned MIN after the merge: the k-th key of any
 * shard's partial list bounds the k-th key of the union, so every shard filters with the tightest.
 * Every shard makes the same calls in the same order. No counterpart in the reference (single-GPU).
 */
enum { FDB200_HOOK_FLAGS = 0, FDB200_HOOK_THRESHOLDS = 1 };
typedef void (*fdb200_round_hook)(void* ctx, int kind, void* dev_ptr, long long count, void* stream);

typedef struct FdB200Opts {
    int struct_size;          /* sizeof(FdB200Opts); set by fdb200_opts_init */
    int device;               /* CUDA device ordinal (Dataset::cuda_device_id, dataset.h:30) */
    int precision;            /* FDB200_FP32: distances bit-identical to the reference FDS build
                                 (fmaf chain); FDB200_TF32: tensor-core TF32 distances */
    int density_kernel;       /* FDB200_LAPLACIAN (default) or FDB200_GAUSSIAN */
    int engine;               /* which distance-tile engine runs the self-kNN: AUTO = tcgen05 where
                                 supported (sm_100 and d <= 178), with the first (dense) rounds on
                                 the exact SIMT tiles; TCGEN05 = tcgen05 for every round; SIMT =
                                 SIMT for every round (any d; FP32 only) */
    int inputs_on_device;     /* nonzero: data / density / index inputs are device pointers */
    int outputs_on_device;    /* nonzero: outputs are device pointers */
    int shard_rank;           /* kNN triangle sharding: this shard's index ... */
    int shard_count;          /* ... out of shard_count (1 = whole triangle) */
    int cand_capacity;        /* per-point candidate slots per round (0 = automatic) */
    void* stream;             /* cudaStream_t to run on; NULL = the library's own stream (pass
                                 cudaStreamLegacy to run on the legacy default stream) */
    int shard_block_lo;       /* explicit shard: the 128-point row blocks [shard_block_lo, shard_block_hi) */
    int shard_block_hi;       /* (-1, -1 = the even split given by shard_rank / shard_count) */
    fdb200_round_hook round_hook;   /* fdb200_knn_partial only (other calls ignore it): NULL =
                                       ordered shards (each shard's rows
                                       against every column, its own lists final, no exchange);
                                       set = symmetric shards (each unordered block pair once over all
                                       shards, partial lists of every point, thresholds combined
                                       through the hook between rounds) */
    void* round_hook_ctx;     /* passed to round_hook */
} FdB200Opts;

typedef struct FdB200Stats {
    double total_ms;          /* device time of the whole call (CUDA events) */
    double upload_ms;         /* host->device copy of the dataset */
    double knn_ms;            /* self-kNN (tiles + merges + final ordering) */
    double density_ms;        /* density + DC detection, including k-halving retries */
    double dc_ms;             /* DC reduction + center selection */
    double labels_ms;         /* label propagation + device->host copies */
    double knn_tile_ms;       /* part of knn_ms spent in the distance-tile kernels */
    long long pairs;          /* unordered pairs evaluated by this shard */
    long long candidates;     /* candidates appended to the per-point lists */
    int rounds;               /* tile rounds run (including overflow re-runs) */
    int overflow_reruns;      /* rounds re-run because a candidate buffer overflowed */
    int num_cores;            /* density cores after the k-halving loop */
    int final_k;              /* k after the k-halving loop */
    int engine_used;          /* FDB200_ENGINE_SIMT or FDB200_ENGINE_TCGEN05 */
    int launches;             /* kernels this call launched */
    int reserved[6];
} FdB200Stats;

/* Fills opts with defaults (device 0, FP32, Laplacian, auto engine, host pointers, 1 shard). */
int fdb200_opts_init(FdB200Opts* opts);

/* Message of the calling thread's last failure ("" if none). */
const char* fdb200_last_error(void);

int fdb200_abi_version(void);

/*
 * Exact self-kNN: for every point the k nearest other points, ordered by (d2, index), with
 * Euclidean distances. Replaces symtri_knn_cuda (symtriknncuda.h:15-18) as called through the
 * kNN plug-in FastDECBase::compute_knn (fastdecbase.h:43-46, symwarpfastdec.cpp:4-10).
 * out_dist / out_idx: k * n each, rank-major. n <= 1 or k <= 0 is a no-op success; k >= n is
 * FDB200_EINVAL (symtriknncuda.cu:319-324).
 */
int fdb200_knn(const float* data, int n, int d, int k, const FdB200Opts* opts,
               float* out_dist, int* out_idx, FdB200Stats* stats);

/*
 * The whole FastDEC fit: self-kNN -> density -> DC detection (with the k-halving retry) ->
 * DC reduction + center selection -> labels. Replaces FastDECBase::Fit (fastdecbase.h:38,
 * fastdecbase.cpp:159-228) with get_center_indices() / get_labels() (fastdecbase.h:35-37), and
 * SymWarpFullGpuFastDEC::Fit (full_gpu/symwarpfullgpufastdec.h:39).
 * centers_out: c entries; labels_out: n entries; densities_out (optional, may be NULL): n.
 */
int fdb200_fit(const float* data, int n, int d, int k, int c, const FdB200Opts* opts,
               int* centers_out, int* labels_out, float* densities_out, FdB200Stats* stats);

/*
 * DC reduction + center selection for given cores. Replaces warp_parallel_dc_reduction_cuda
 * (dcreductioncuda.h:45-51): core_parent_out[i] = nearest strictly denser point of core i
 * (-1 if none); centers_out: num_centers global indices (-1 padded).
 */
int fdb200_dc_reduction(const float* data, int n, int d, const float* densities,
                        const int* core_indices, int core_nb, int num_centers,
                        const FdB200Opts* opts, int* core_parent_out, int* centers_out);

/*
 * Density of every point from the first k ranks of a rank-major kNN distance list whose rank
 * stride is n. Replaces FastDECBase::density_estimation_{laplacian,gaussian}
 * (fastdecbase.cpp:276-301; mean as the sequential double sum of fastdecbase.cpp:257-274) and
 * gpu_density_estimation_* (full_gpu/symwarpfastdeccuda.h:54-58). mean_out may be NULL.
 */
int fdb200_density(const float* knn_dist, int n, int k, const FdB200Opts* opts,
                   float* densities_out, double* mean_out);

/*
 * DC detection: parent_out[i] = first neighbour (rank order, first k ranks) with a strictly
 * greater density, else -1; cores_out = points with parent -1 in ascending order (capacity n).
 * Replaces FastDECBase::dc_detection (fastdecbase.cpp:303-333) / gpu_dc_detection
 * (full_gpu/symwarpfastdeccuda.h:60-61).
 */
int fdb200_dc_detection(const int* knn_idx, const float* densities, int n, int k,
                        const FdB200Opts* opts, int* parent_out, int* cores_out, int* num_cores_out);

/*
 * Labels: centers get 0..c-1; every other point takes the label of the first center on its
 * parent chain, or 0 when the chain ends at a parent of -1. Replaces FastDECBase::final_cluster
 * (fastdecbase.cpp:358-385) / gpu_final_cluster (full_gpu/symwarpfastdeccuda.h:70-72).
 */
int fdb200_final_cluster(const int* parent, int n, const int* centers, int c,
                         const FdB200Opts* opts, int* labels_out);

/*
 * Multi-GPU building blocks (device pointers only). A shard computes the triangle tiles of its
 * shard_rank / shard_count share into packed per-point partial lists; lists from all shards
 * are then exchanged to their owners (by the caller's NCCL / torch.distributed) and merged.
 * A packed entry is ((uint64)float_bits(d2) << 32) | index; lists are point-major, n * k,
 * ascending, padded with UINT64_MAX. No counterpart in the reference (it is single-GPU); the
 * merged result equals fdb200_knn's.
 * With the tcgen05 engine and no round_hook a shard tests its own row blocks against every column
 * (ordered pairs): the lists of its own points are then final and need no exchange. With a
 * round_hook (see fdb200_round_hook) a shard multiplies only the block pairs whose first block is
 * its own, once, tests both endpoints and keeps partial lists of every point, which the caller
 * exchanges to their owners and merges (fdb200_merge_lists); the dense first rounds then run on
 * symmetric SIMT tiles.
 */
int fdb200_knn_partial(const float* data_dev, int n, int d, int k, const FdB200Opts* opts,
                       uint64_t* lists_dev, FdB200Stats* stats);

/* lists_dev (n_points * k) <- k-smallest of itself and `nsrc` other list blocks of the same
   points, stored one after another in srcs_dev (nsrc * n_points * k). */
int fdb200_merge_lists(uint64_t* lists_dev, const uint64_t* srcs_dev, int nsrc, int n_points,
                       int k, const FdB200Opts* opts);

/* rank-major Euclidean distances / indices from packed point-major lists (device pointers). */
int fdb200_lists_to_knn(const uint64_t* lists_dev, int n, int k, const FdB200Opts* opts,
                        float* dist_dev, int* idx_dev);

/*
 * Fit from a finished kNN graph (rank-major dist / idx, rank stride n; the first k ranks are used,
 * so a graph of more ranks serves any smaller k): the stages after build_knn_graph
 * (fastdecbase.cpp:173-227). data, knn_dist and knn_idx are device pointers when
 * opts->inputs_on_device, host pointers otherwise.
 */
int fdb200_fit_from_knn(const float* data, const float* knn_dist, const int* knn_idx,
                        int n, int d, int k, int c, const FdB200Opts* opts, int* centers_out,
                        int* labels_out, float* densities_out, FdB200Stats* stats);

/*
 * The fit's stages after the kNN, split so that a multi-GPU caller can shard the DC reduction (the
 * reference's dc_reduction_cuda, dcreductioncuda.cu:189-545, is a cores x N contraction; here every GPU
 * reduces its own range of points and the partial results combine). No counterpart in the reference,
 * which is single-GPU; run on one GPU over [0, n) they give fdb200_fit_from_knn's results.
 *
 * fdb200_density_detection: density and DC detection with the k-halving retry while cores < c
 *   (fastdecbase.cpp:173-199) from a rank-major graph (rank stride n): densities_out n floats,
 *   parent_out n ints, cores_out (capacity n) the cores in ascending order, *num_cores_out their count,
 *   *final_k_out the k after halving. FDB200_ECORES when even k = 1 gives fewer than c cores.
 * fdb200_dc_stage (device pointers): stage 0 writes best_dev[i] = the lexicographic minimum packed key
 *   ((uint64)float_bits(d2) << 32 | index) over the points of [p_lo, p_hi) strictly denser than core i
 *   (UINT64_MAX when none); keys of several ranges combine by minimum. Stage 1 reads the combined keys
 *   and writes rank_dev[i] = the points of [p_lo, p_hi) closer to core i than that parent; ranks of
 *   several ranges combine by sum (dcreductioncuda.cu:63-170).
 * fdb200_dc_select (device pointers): from the combined keys and ranks, core_parent_dev (-1 when no
 *   denser point) and centers_dev (num_centers global indices, -1 padded), as
 *   warp_parallel_dc_reduction_cuda returns them (dcreductioncuda.cu:113-187, 548-619).
 */
int fdb200_density_detection(const float* knn_dist, const int* knn_idx, int n, int k, int c, const FdB200Opts* opts,
                             float* densities_out, int* parent_out, int* cores_out, int* num_cores_out,
                             int* final_k_out);
int fdb200_dc_stage(int stage, const float* data_dev, int n, int d, const float* densities_dev,
                    const int* cores_dev, int core_nb, int p_lo, int p_hi, const FdB200Opts* opts,
                    uint64_t* best_dev, int* rank_dev);
int fdb200_dc_select(const float* densities_dev, const int* cores_dev, int core_nb, const uint64_t* best_dev,
                     const int* rank_dev, int num_centers, const FdB200Opts* opts, int* core_parent_dev,
                     int* centers_dev);

/*
 * DIAGNOSTICS: audit of the tcgen05 filter's margin on a small problem (n <= 16384; device pointers). For
 * every point i the threshold thr_d2_dev[i] (a squared distance, e.g. the point's exact k-th neighbour)
 * is folded into the row operand exactly as the list merge folds a list's threshold; then one
 * tcgen05.mma per 128 x 256 tile computes acc_dev[i * n + j] = the FP32 accumulation of
 * |x~_i - x~_j|^2 - V_i, which the filter keeps a pair for iff it is negative. bound_dev[i] = V_i;
 * arows_dev / brows_dev: the TF32 operand rows (n x K each, K = *kp_out) the MMA consumed, so a test can
 * form the exact sum and measure the accumulation error against the error model the margin assumes.
 * No counterpart in the reference (its TF32 path has no rigorous filter).
 */
int fdb200_debug_tc_filter(const float* data_dev, int n, int d, const float* thr_d2_dev, const FdB200Opts* opts,
                           float* acc_dev, float* bound_dev, float* arows_dev, float* brows_dev, int* kp_out);

/* Frees the library's cached device workspace on opts->device. The workspace grows to what the
 * largest call needed: for the kNN about 6 KB a point at d = 50, k = 45 (8.5 GB at 1,291,147 points). */
int fdb200_release(const FdB200Opts* opts);

/*
 * The reference CLI's dataset file: one point per line, comma-separated numbers. Replaces
 * get_rows_coloumns + read_data (helper.cpp:9-63) and the host transpose (test.cpp:110-115), in
 * parallel: fdb200_csv_shape gives the point count n (non-blank lines) and dimension d (values on the
 * first line); fdb200_read_csv fills out_dim_major[t * n + i] (d * n floats, caller-allocated) with
 * threads host threads (0 = all cores). Values parse as strtof does (correctly rounded); a line
 * without exactly d numbers is FDB200_EINVAL. No GPU is involved.
 */
int fdb200_csv_shape(const char* path, int* n_out, int* d_out);
int fdb200_read_csv(const char* path, int n, int d, float* out_dim_major, int threads);

/*
 * Writes a dim-major dataset (data_dim_major[t * n + i]) in the reference CLI's CSV format: one point per
 * line, comma-separated, each value as the shortest text that reads back (strtof) as the same float, so
 * the reference's read_data (helper.cpp:30-63) and fdb200_read_csv recover the exact float32 values. No
 * counterpart in the reference (it only reads). Host-only; threads as in fdb200_read_csv.
 */
int fdb200_write_csv(const char* path, const float* data_dim_major, int n, int d, int threads);

/*
 * The dataset as a binary file (.fbin): int32 n, int32 d, then n * d float32, row-major (one point per
 * row), little endian. No counterpart in the reference, which reads CSV text only (helper.cpp:9-63):
 * the same dim-major output as fdb200_read_csv (out_dim_major[t * n + i]) without a text parse.
 * fdb200_write_fbin writes a dim-major array in that format (e.g. to convert a CSV once).
 * Host-only; a size that disagrees with the header is FDB200_EINVAL.
 */
int fdb200_fbin_shape(const char* path, int* n_out, int* d_out);
int fdb200_read_fbin(const char* path, int n, int d, float* out_dim_major, int threads);
int fdb200_write_fbin(const char* path, const float* data_dim_major, int n, int d);

/*
 * kNN-graph persistence. No counterpart in the reference, which recomputes the graph on every Fit
 * (build_knn_graph, fastdecbase.cpp:231-255). fdb200_knn_graph_save writes the rank-major graph that
 * fdb200_knn returns (host pointers; k ranks of n points) with a 32-byte header (magic "FDBKNNG1",
 * version, n, k, the caller's flags word, a hash of the payload); fdb200_knn_graph_shape reads n, k and
 * flags back; fdb200_knn_graph_load fills caller buffers of k * n entries, checks the hash and the
 * index range, and returns FDB200_EINVAL on a mismatch or a damaged file. A graph of k ranks serves
 * fdb200_fit_from_knn for any k' <= k, so sweeps over k and the cluster count need one kNN.
 * Host-only.
 */
int fdb200_knn_graph_save(const char* path, const float* knn_dist, const int* knn_idx, int n, int k,
                          int flags);
int fdb200_knn_graph_shape(const char* path, int* n_out, int* k_out, int* flags_out);
int fdb200_knn_graph_load(const char* path, int n, int k, float* knn_dist, int* knn_idx);

/*
 * fdb200_density without any allocation. No counterpart in the reference (every reference call,
 * and every other entry point here, obtains device memory as it goes). It is for callers that must
 * not allocate while they run: a serving loop that reserved all device memory up front, a process
 * whose memory belongs to another framework's caching allocator, or code that cannot afford the
 * device-wide synchronisation and the out-of-memory failure point that cudaMalloc / cudaFree bring.
 *
 * Same densities and mean as fdb200_density (Laplacian or Gaussian per opts->density_kernel), from
 * DEVICE pointers on opts->device: knn_dist_dev rank-major (rank stride n, k ranks),
 * densities_dev n floats, mean_dev one double. The working memory is a fixed array inside the
 * library image, sized for at most FDB200_NOALLOC_MAX_POINTS points; a larger n returns
 * FDB200_EINVAL without launching anything. Nothing in that array needs to start at zero: each call
 * writes every word it later reads.
 *
 * Asynchronous on opts->stream (NULL = the legacy default stream); results are ready when the
 * stream reaches them. The array is shared by all calls on a device, so calls whose executions
 * overlap (two streams, or two host threads with no ordering between them) race and corrupt each
 * other's mean: order them on one stream or with events. The first call on each device does a
 * one-time set-up: it looks up the array's address (cudaGetSymbolAddress) and loads the kernels
 * this entry point launches (CUDA otherwise loads each kernel lazily, obtaining device memory for
 * its code, at its first launch); make that first call before any stream capture begins. Later
 * calls on that device obtain no memory at all.
 */
#define FDB200_NOALLOC_MAX_POINTS 4194304
int fdb200_density_noalloc(const float* knn_dist_dev, int n, int k, const FdB200Opts* opts,
                           float* densities_dev, double* mean_dev);

#ifdef __cplusplus
}
#endif

#endif /* FASTDEC_B200_H */
