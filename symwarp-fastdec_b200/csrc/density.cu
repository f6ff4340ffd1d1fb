// density.cu -- kNN density with the reference's exact mean, and DC detection.
//
// The reference's host density (fastdecbase.cpp:257-301) divides by a mean formed as a
// SEQUENTIAL double sum of every kNN distance in point-major order; its GPU variant
// (full_gpu/symwarpfastdeccuda.cu:62-83) uses a tree sum whose last bits can differ. Densities are
// bit-sensitive to the mean, so this file reproduces the sequential sum exactly, in parallel:
//
//   While the running sum S stays inside one binade [2^e, 2^(e+1)), S is an integer multiple s of
//   u = 2^(e-52), and fl(S + v) for v >= 0 is S + inc * u where inc = floor(v/u) plus a rounding
//   step that depends only on the fraction of v/u and, for an exact half, on the parity of s
//   (round half to even). So a run of additions inside one binade is a map
//   parity -> (total increment, new parity), and such maps compose associatively.
//   Chunks of 32 points compute their map for the binade suggested by an approximate prefix sum;
//   maps of the same binade are composed in a tree; one thread then walks the tree, applying a
//   map only when the exact running sum starts inside its binade and the result stays below
//   2^(e+1) (so every intermediate sum was inside it), and otherwise descends, down to plain
//   sequential addition of one chunk. The approximate prefix only steers the walk; the result is
//   the sequential sum bit for bit.
#include "fdb_internal.h"

#include <algorithm>
#include <vector>

namespace fdb {

namespace {

constexpr int kLevels = 8;

struct BinadeMap {
    long long tot[2];   // increment in units of 2^(e-52), for start parity 0 / 1
    int par[2];         // parity after the run, for start parity 0 / 1
    int e;              // binade exponent
    int kind;           // 0 = unusable, 1 = valid for binade e, 2 = identity (all values zero)
};

__device__ __forceinline__ BinadeMap compose(const BinadeMap& a, const BinadeMap& b)
{
    // a first, then b
    BinadeMap r;
    if (a.kind == 2) return b;
    if (b.kind == 2) return a;
    if (a.kind == 0 || b.kind == 0 || a.e != b.e) {
        r.kind = 0;
        r.e = a.e;
        r.tot[0] = r.tot[1] = 0;
        r.par[0] = 0;
        r.par[1] = 1;
        return r;
    }
    r.kind = 1;
    r.e = a.e;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        r.tot[p] = a.tot[p] + b.tot[a.par[p]];
        r.par[p] = b.par[a.par[p]];
    }
    return r;
}

__device__ __forceinline__ BinadeMap shfl_down_map(const BinadeMap& m, int off)
{
    BinadeMap r;
    r.tot[0] = __shfl_down_sync(0xffffffffu, m.tot[0], off);
    r.tot[1] = __shfl_down_sync(0xffffffffu, m.tot[1], off);
    r.par[0] = __shfl_down_sync(0xffffffffu, m.par[0], off);
    r.par[1] = __shfl_down_sync(0xffffffffu, m.par[1], off);
    r.e = __shfl_down_sync(0xffffffffu, m.e, off);
    r.kind = __shfl_down_sync(0xffffffffu, m.kind, off);
    return r;
}

// ordered composition of the 32 lane maps (lane 0 first); result valid in lane 0
__device__ __forceinline__ BinadeMap warp_compose(BinadeMap m, int lane)
{
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        BinadeMap o = shfl_down_map(m, off);
        if ((lane & (2 * off - 1)) == 0 && lane + off < 32) m = compose(m, o);
    }
    return m;
}

// K1: approximate double sum of each chunk of 32 points (any order)
__global__ void chunk_sums_kernel(const float* __restrict__ dist, int n, int k, double* __restrict__ csum,
                                  int nchunks)
{
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= nchunks) return;
    const int p = warp * 32 + lane;
    double s = 0.0;
    if (p < n)
        for (int q = 0; q < k; ++q) s += (double)dist[(size_t)q * n + p];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_down_sync(0xffffffffu, s, off);
    if (lane == 0) csum[warp] = s;
}

// K2: exclusive prefix of the chunk sums (approximate; one block)
__global__ void prefix_kernel(const double* __restrict__ csum, int nchunks, double* __restrict__ pre)
{
    __shared__ double part[1024];
    const int t = threadIdx.x, per = (nchunks + 1023) / 1024;
    const int lo = min(nchunks, t * per), hi = min(nchunks, lo + per);
    double s = 0.0;
    for (int c = lo; c < hi; ++c) s += csum[c];
    part[t] = s;
    __syncthreads();
    if (t == 0) {
        double run = 0.0;
        for (int i = 0; i < 1024; ++i) {
            const double v = part[i];
            part[i] = run;
            run += v;
        }
    }
    __syncthreads();
    double run = part[t];
    for (int c = lo; c < hi; ++c) {
        pre[c] = run;
        run += csum[c];
    }
}

// K3: the binade map of every chunk, for the binade of its approximate start
__global__ void chunk_maps_kernel(const float* __restrict__ dist, int n, int k,
                                  const double* __restrict__ pre, const double* __restrict__ csum,
                                  BinadeMap* __restrict__ maps, int nchunks)
{
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= nchunks) return;
    BinadeMap m;
    m.tot[0] = m.tot[1] = 0;
    m.par[0] = 0;
    m.par[1] = 1;
    const double start = pre[warp];
    const int p = warp * 32 + lane;
    bool all_zero = true, bad = false;
    if (p < n)
        for (int q = 0; q < k; ++q) {
            const float v = dist[(size_t)q * n + p];
            all_zero &= (v == 0.0f);
            bad |= !(v >= 0.0f);            // negative or NaN: only plain sequential addition is exact
        }
    all_zero = __all_sync(0xffffffffu, all_zero);
    bad = __any_sync(0xffffffffu, bad);
    if (bad || (!all_zero && !(start > 0.0))) {
        m.kind = 0;
        m.e = 0;
    } else if (all_zero) {
        m.kind = 2;   // adding +0 never changes a non-negative sum
        m.e = 0;
    } else {
        const int e = ilogb(start);
        m.e = e;
        m.kind = 1;
        if (p < n) {
            for (int q = 0; q < k; ++q) {
                const double t = ldexp((double)dist[(size_t)q * n + p], 52 - e);  // v / u, exact
                if (!(t < 9007199254740992.0)) {   // v >= 2^(e+1): the run must leave the binade
                    m.kind = 0;
                    break;
                }
                const double fm = floor(t);
                const double frac = t - fm;        // exact
                const long long mi = (long long)fm;
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                    long long inc = mi;
                    if (frac > 0.5) inc += 1;
                    else if (frac == 0.5) inc += (m.par[s] + mi) & 1;   // half: round to even
                    m.tot[s] += inc;
                    m.par[s] = (int)((m.par[s] + inc) & 1);
                }
            }
        }
        if (__any_sync(0xffffffffu, m.kind == 0)) m.kind = 0;
    }
    m = warp_compose(m, lane);
    if (lane == 0) maps[warp] = m;
}

// K3b: compose runs of 32 maps of one level into the next level
__global__ void compose_level_kernel(const BinadeMap* __restrict__ in, int nin, BinadeMap* __restrict__ out,
                                     int nout)
{
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= nout) return;
    const int i = warp * 32 + lane;
    BinadeMap m;
    if (i < nin) {
        m = in[i];
    } else {
        m.kind = 2;
        m.e = 0;
        m.tot[0] = m.tot[1] = 0;
        m.par[0] = 0;
        m.par[1] = 1;
    }
    m = warp_compose(m, lane);
    if (lane == 0) out[warp] = m;
}

struct MeanLevels {
    const BinadeMap* lvl[kLevels];
    int count[kLevels];
    int nlev;
};

__device__ bool try_apply(const BinadeMap& m, double& S)
{
    if (m.kind == 2) return true;
    if (m.kind != 1) return false;
    const double lo = ldexp(1.0, m.e), hi = ldexp(1.0, m.e + 1);
    if (!(S >= lo && S < hi)) return false;
    const long long s = (long long)ldexp(S, 52 - m.e);   // exact integer in [2^52, 2^53)
    const long long ns = s + m.tot[s & 1];
    if (ns >= (1ll << 53)) return false;                   // would have left the binade
    S = ldexp((double)ns, m.e - 52);
    return true;
}

// K4: one thread walks the map tree from the top, descending where a map cannot be applied
__global__ void resolve_mean_kernel(MeanLevels L, const float* __restrict__ dist, int n, int k,
                                    double* __restrict__ mean_out)
{
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    double S = 0.0;
    int stack_lvl[kLevels * 2 + 4], stack_idx[kLevels * 2 + 4], stack_end[kLevels * 2 + 4];
    int sp = 0;
    const int top = L.nlev - 1;
    stack_lvl[0] = top;
    stack_idx[0] = 0;
    stack_end[0] = L.count[top];
    sp = 1;
    while (sp > 0) {
        const int lv = stack_lvl[sp - 1];
        const int i = stack_idx[sp - 1];
        if (i >= stack_end[sp - 1]) {
            --sp;
            continue;
        }
        stack_idx[sp - 1] = i + 1;
        if (try_apply(L.lvl[lv][i], S)) continue;
        if (lv == 0) {
            // plain sequential addition of this chunk (fastdecbase.cpp:264-271)
            const int p0 = i * 32, p1 = min(n, p0 + 32);
            for (int p = p0; p < p1; ++p)
                for (int q = 0; q < k; ++q) S += (double)dist[(size_t)q * n + p];
            continue;
        }
        stack_lvl[sp] = lv - 1;
        stack_idx[sp] = i * 32;
        stack_end[sp] = min(L.count[lv - 1], i * 32 + 32);
        ++sp;
    }
    *mean_out = S / ((double)n * k);
}

// fastdecbase.cpp:57-94 / full_gpu/symwarpfastdeccuda.cu:85-117: per-point double exp-sum
__global__ void density_kernel(const float* __restrict__ dist, int n, int k, int gaussian,
                               const double* __restrict__ mean_p, float* __restrict__ den)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const double mean = *mean_p;
    const double two_mean_sq = 2.0 * mean * mean;
    double s = 0.0;
    for (int q = 0; q < k; ++q) {
        const float v = dist[(size_t)q * n + i];
        if (gaussian) {
            const double dd = (double)v;
            s += exp(__ddiv_rn(-dd * dd, two_mean_sq));
        } else {
            const float half = __fmul_rn(-v, 0.5f);   // -row[c] / 2 in float: exact halving
            s += exp(__ddiv_rn((double)half, mean));
        }
    }
    den[i] = __double2float_rn(s);
}

}  // namespace

void exact_mean(Workspace& ws, const float* dist, int n, int k, double* mean_dev, cudaStream_t s)
{
    const int nchunks = (n + 31) / 32;
    // level sizes
    int counts[kLevels];
    int nlev = 0;
    int c = nchunks;
    counts[nlev++] = c;
    while (c > 1 && nlev < kLevels) {
        c = (c + 31) / 32;
        counts[nlev++] = c;
    }
    FDB_REQUIRE(counts[nlev - 1] <= 32 * 32, "too many points for the mean tree");
    size_t total_maps = 0;
    for (int l = 0; l < nlev; ++l) total_maps += counts[l];
    char* base = (char*)ws.mean_tmp.ensure(sizeof(double) * 2 * (size_t)nchunks + sizeof(BinadeMap) * total_maps + 256);
    double* csum = (double*)base;
    double* pre = csum + nchunks;
    BinadeMap* maps = (BinadeMap*)(((uintptr_t)(pre + nchunks) + 15) & ~uintptr_t(15));
    MeanLevels L;
    L.nlev = nlev;
    BinadeMap* cur = maps;
    for (int l = 0; l < nlev; ++l) {
        L.lvl[l] = cur;
        L.count[l] = counts[l];
        cur += counts[l];
    }
    const int wpb = 8;
    chunk_sums_kernel<<<(nchunks + wpb - 1) / wpb, wpb * 32, 0, s>>>(dist, n, k, csum, nchunks);
    FDB_LAUNCHED();
    prefix_kernel<<<1, 1024, 0, s>>>(csum, nchunks, pre);
    FDB_LAUNCHED();
    chunk_maps_kernel<<<(nchunks + wpb - 1) / wpb, wpb * 32, 0, s>>>(dist, n, k, pre, csum,
                                                                     (BinadeMap*)L.lvl[0], nchunks);
    FDB_LAUNCHED();
    for (int l = 1; l < nlev; ++l) {
        compose_level_kernel<<<(counts[l] + wpb - 1) / wpb, wpb * 32, 0, s>>>(
            L.lvl[l - 1], counts[l - 1], (BinadeMap*)L.lvl[l], counts[l]);
        FDB_LAUNCHED();
    }
    resolve_mean_kernel<<<1, 32, 0, s>>>(L, dist, n, k, mean_dev);
    FDB_LAUNCHED();
}

static_assert(sizeof(BinadeMap) == 32, "mean_scratch_bytes assumes 32-byte maps");

// exact_mean with caller-supplied scratch laid out as mean_scratch_bytes describes; every word the
// kernels read is written earlier in the same call, so the scratch needs no initial contents
void exact_mean_in(void* scratch, size_t scratch_bytes, const float* dist, int n, int k, double* mean_dev,
                   cudaStream_t s)
{
    FDB_REQUIRE(scratch_bytes >= mean_scratch_bytes(n), "mean scratch too small for " + std::to_string(n) +
                                                            " points");
    const int nchunks = (n + 31) / 32;
    int counts[kLevels];
    int nlev = 0;
    int c = nchunks;
    counts[nlev++] = c;
    while (c > 1 && nlev < kLevels) {
        c = (c + 31) / 32;
        counts[nlev++] = c;
    }
    FDB_REQUIRE(counts[nlev - 1] <= 32 * 32, "too many points for the mean tree");
    double* csum = (double*)scratch;
    double* pre = csum + nchunks;
    BinadeMap* maps = (BinadeMap*)(((uintptr_t)(pre + nchunks) + 15) & ~uintptr_t(15));
    MeanLevels L;
    L.nlev = nlev;
    BinadeMap* cur = maps;
    for (int l = 0; l < nlev; ++l) {
        L.lvl[l] = cur;
        L.count[l] = counts[l];
        cur += counts[l];
    }
    const int wpb = 8;
    chunk_sums_kernel<<<(nchunks + wpb - 1) / wpb, wpb * 32, 0, s>>>(dist, n, k, csum, nchunks);
    FDB_LAUNCHED();
    prefix_kernel<<<1, 1024, 0, s>>>(csum, nchunks, pre);
    FDB_LAUNCHED();
    chunk_maps_kernel<<<(nchunks + wpb - 1) / wpb, wpb * 32, 0, s>>>(dist, n, k, pre, csum,
                                                                     (BinadeMap*)L.lvl[0], nchunks);
    FDB_LAUNCHED();
    for (int l = 1; l < nlev; ++l) {
        compose_level_kernel<<<(counts[l] + wpb - 1) / wpb, wpb * 32, 0, s>>>(
            L.lvl[l - 1], counts[l - 1], (BinadeMap*)L.lvl[l], counts[l]);
        FDB_LAUNCHED();
    }
    resolve_mean_kernel<<<1, 32, 0, s>>>(L, dist, n, k, mean_dev);
    FDB_LAUNCHED();
}

void density_from_mean(const float* dist, int n, int k, int gaussian, const double* mean_dev, float* den,
                       cudaStream_t s)
{
    if (n <= 0) return;
    density_kernel<<<(n + 255) / 256, 256, 0, s>>>(dist, n, k, gaussian, mean_dev, den);
    FDB_LAUNCHED();
}

// Loads the kernels of exact_mean_in and density_from_mean on the current device now. With CUDA's
// lazy loading a kernel's code is loaded (and device memory obtained for it) at its first launch;
// the allocation-free entry point calls this once per device so that no later call loads anything.
void preload_mean_density_kernels()
{
    cudaFuncAttributes fa;
    FDB_CUDA(cudaFuncGetAttributes(&fa, chunk_sums_kernel));
    FDB_CUDA(cudaFuncGetAttributes(&fa, prefix_kernel));
    FDB_CUDA(cudaFuncGetAttributes(&fa, chunk_maps_kernel));
    FDB_CUDA(cudaFuncGetAttributes(&fa, compose_level_kernel));
    FDB_CUDA(cudaFuncGetAttributes(&fa, resolve_mean_kernel));
    FDB_CUDA(cudaFuncGetAttributes(&fa, density_kernel));
}

// ------------------------------------------------------------------ DC detection
namespace {

// fastdecbase.cpp:303-333 / full_gpu/symwarpfastdeccuda.cu:160-205
__global__ void detection_kernel(const int* __restrict__ idx, const float* __restrict__ den, int n, int k,
                                 int* __restrict__ parent)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float di = den[i];
    int p = -1;
    for (int q = 0; q < k; ++q) {
        const int j = idx[(size_t)q * n + i];
        if (j < 0 || j >= n) continue;   // padding / foreign input: never a denser neighbour
        if (di < den[j]) {
            p = j;
            break;
        }
    }
    parent[i] = p;
}

constexpr int kScanBlock = 1024;

__global__ void core_counts_kernel(const int* __restrict__ parent, int n, int* __restrict__ bcount)
{
    __shared__ int warp_tot[32];
    const int i = blockIdx.x * kScanBlock + threadIdx.x;
    const int f = (i < n && parent[i] == -1) ? 1 : 0;
    const int w = __popc(__ballot_sync(0xffffffffu, f));
    if ((threadIdx.x & 31) == 0) warp_tot[threadIdx.x >> 5] = w;
    __syncthreads();
    if (threadIdx.x == 0) {
        int s = 0;
        for (int t = 0; t < kScanBlock / 32; ++t) s += warp_tot[t];
        bcount[blockIdx.x] = s;
    }
}

__global__ void block_offsets_kernel(int* __restrict__ bcount, int nblocks, int* __restrict__ total)
{
    __shared__ int part[1024];
    const int t = threadIdx.x, per = (nblocks + 1023) / 1024;
    const int lo = min(nblocks, t * per), hi = min(nblocks, lo + per);
    int s = 0;
    for (int b = lo; b < hi; ++b) s += bcount[b];
    part[t] = s;
    __syncthreads();
    if (t == 0) {
        int run = 0;
        for (int i = 0; i < 1024; ++i) {
            const int v = part[i];
            part[i] = run;
            run += v;
        }
        *total = run;
    }
    __syncthreads();
    int run = part[t];
    for (int b = lo; b < hi; ++b) {
        const int v = bcount[b];
        bcount[b] = run;
        run += v;
    }
}

// ordered compaction: cores in ascending index order (thrust::copy_if semantics)
__global__ void core_scatter_kernel(const int* __restrict__ parent, int n, const int* __restrict__ boff,
                                    int* __restrict__ cores)
{
    __shared__ int warp_off[32];
    const int i = blockIdx.x * kScanBlock + threadIdx.x;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int f = (i < n && parent[i] == -1) ? 1 : 0;
    const unsigned bal = __ballot_sync(0xffffffffu, f);
    if (lane == 0) warp_off[w] = __popc(bal);
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int t = 0; t < kScanBlock / 32; ++t) {
            const int v = warp_off[t];
            warp_off[t] = run;
            run += v;
        }
    }
    __syncthreads();
    if (f) cores[boff[blockIdx.x] + warp_off[w] + __popc(bal & ((1u << lane) - 1))] = i;
}

}  // namespace

int dc_detection(Workspace& ws, const int* idx, const float* den, int n, int k, int* parent, int* cores,
                 cudaStream_t s)
{
    detection_kernel<<<(n + 255) / 256, 256, 0, s>>>(idx, den, n, k, parent);
    FDB_LAUNCHED();
    const int nblocks = (n + kScanBlock - 1) / kScanBlock;
    int* bcount = ws.scan.as<int>((size_t)nblocks + 16);
    int* total = bcount + nblocks;
    core_counts_kernel<<<nblocks, kScanBlock, 0, s>>>(parent, n, bcount);
    FDB_LAUNCHED();
    block_offsets_kernel<<<1, 1024, 0, s>>>(bcount, nblocks, total);
    FDB_LAUNCHED();
    core_scatter_kernel<<<nblocks, kScanBlock, 0, s>>>(parent, n, bcount, cores);
    FDB_LAUNCHED();
    FDB_CUDA(cudaMemcpyAsync(ws.pinned + 8, total, sizeof(int), cudaMemcpyDeviceToHost, s));
    FDB_CUDA(cudaStreamSynchronize(s));
    return ws.pinned[8];
}

}  // namespace fdb
