// knn.cu -- symmetric triangular exact self-kNN: round scheduler, SIMT distance tiles, per-point
// list merge and the final rank-major ordering.
//
// Reference behaviour (cyberbull66/symwarp-fastdec): symtri_knn_cuda (symtriknncuda.cu:310-633)
// walks the upper triangle of 9216^2 tiles one at a time, materialises each -2 X_r X_q^T tile in
// HBM (cuBLAS SGEMM or the FDS FFMA tile, symtriknnfds.h:33-166) and feeds it to warp heaps with a
// serial lane-0 insert (symtriknncuda.cu:104-210, symtriknnreverse.h:14-185). Its observable result
// is, for every point, the lexicographic (d2, index) k-smallest of
//     d2(i, j) = max((n_i + n_j) + (-2 * dot(x_i, x_j)), 0),   dot = fmaf chain over d = 0..D-1,
// sorted ascending and sqrt'd (symtriknnsort.h:13-25, symtriknncuda.cu:225-234).
//
// B200 design (no tile in HBM, no serial heap):
//   * The triangle is cut into 128-point blocks. Block pairs are visited by cyclic offset
//     delta = (R - B) mod T, so every round touches every block the same number of times.
//   * Each point keeps a sorted list of packed keys ((d2 bits << 32) | index) in HBM. A tile
//     compares every pair against the row point's and the column point's list thresholds
//     (snapshotted at round start) and appends survivors to per-point candidate buffers with one
//     atomicAdd per (point, thread). A merge kernel then folds the candidates into the lists.
//   * Rounds grow geometrically (each round adds about as many candidates per point as the list
//     has seen before, scaled so that at most half the candidate buffer fills on average), so the
//     stale-threshold cost stays O(k log N) candidates per point. A round whose buffers overflow is
//     discarded and re-run in two halves, which always terminates (one offset never exceeds 256
//     candidates per point and the buffer holds at least 256).
//   * Because every pair is evaluated once and the lists keep the exact lexicographic k-smallest,
//     the result equals the reference's FDS build bit for bit, ties included, whatever the order in
//     which tiles run.
#include "knn_common.cuh"

#include <algorithm>
#include <cfloat>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace fdb {

// ------------------------------------------------------------------ norms (symtriknncuda.cu:56-72)
__global__ void norms_kernel(const float* __restrict__ x, int ldx, int n, int d, float* __restrict__ out)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float s = 0.0f;
    for (int t = 0; t < d; ++t) {
        const float v = x[(size_t)t * ldx + i];
        s = __fmaf_rn(v, v, s);
    }
    out[i] = s;
}

void compute_norms(const float* x, int ldx, int n, int d, float* norms, cudaStream_t s)
{
    if (n <= 0) return;
    norms_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, ldx, n, d, norms);
    FDB_LAUNCHED();
}

constexpr int kSimtThreads = 256;
constexpr int kSimtRoundMaxOffsets = 16;   // rounds of at most this many offsets run on the SIMT tiles
constexpr int kDChunk = 32;

// Exact FP32 tile: 128 x 128 pairs per CTA, 8 x 8 per thread, every dot product the sequential
// fmaf chain over d = 0..D-1 (the FDS accumulation order, symtriknnfds.h:100-121).
__global__ void __launch_bounds__(kSimtThreads, 2) knn_tile_simt(TileRound r)
{
    __shared__ __align__(16) float As[kDChunk][kBlock];
    __shared__ __align__(16) float Bs[kDChunk][kBlock];
    // rounds are queued without a host check in between: once an earlier round overflowed (or this
    // one did, in another CTA), the round is discarded and the CTA does nothing (one read, made
    // uniform across the CTA)
    if (__syncthreads_or(threadIdx.x == 0 && (*(volatile const int*)r.ovf | *((volatile const int*)r.ovf + 1))))
        return;
    int B, R;
    if (!decode_unit(r, blockIdx.x, B, R)) return;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int q0 = B * kBlock, r0 = R * kBlock;

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    for (int d0 = 0; d0 < r.d; d0 += kDChunk) {
        const int steps = min(kDChunk, r.d - d0);
        for (int e = tid; e < kDChunk * kBlock; e += kSimtThreads) {
            const int dd = e / kBlock, p = e % kBlock;
            float va = 0.0f, vb = 0.0f;
            if (dd < steps) {
                const float* col = r.x + (size_t)(d0 + dd) * r.ldx;
                if (q0 + p < r.n) va = col[q0 + p];
                if (r0 + p < r.n) vb = col[r0 + p];
            }
            As[dd][p] = va;
            Bs[dd][p] = vb;
        }
        __syncthreads();
#pragma unroll 2
        for (int dd = 0; dd < steps; ++dd) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[dd][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[dd][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[dd][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[dd][64 + tx * 4]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }

    // epilogue: exact d2, lexicographic admission against the snapshotted list thresholds
    int gi[8], gj[8];
    float nq[8], nr[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        gi[t] = q0 + ((t < 4) ? ty * 4 + t : 64 + ty * 4 + (t - 4));
        gj[t] = r0 + ((t < 4) ? tx * 4 + t : 64 + tx * 4 + (t - 4));
        nq[t] = (gi[t] < r.n) ? r.norms[gi[t]] : 0.0f;
        nr[t] = (gj[t] < r.n) ? r.norms[gj[t]] : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (gi[i] >= r.n) continue;
        const uint64_t bound = r.thr[gi[i]];
        unsigned mask = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const bool ok = gj[j] < r.n && gj[j] != gi[i] &&
                            pack_key(exact_d2(nq[i], nr[j], acc[i][j]), gj[j]) < bound;
            mask |= (ok ? 1u : 0u) << j;
        }
        if (mask) {
            int slot = atomicAdd(&r.cnt[gi[i]], __popc(mask));
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (mask & (1u << j)) append_at(r, gi[i], slot++, pack_key(exact_d2(nq[i], nr[j], acc[i][j]), gj[j]));
        }
    }
    if (r.diag || r.rows_only) return;   // diagonal and rows-only units update their row block only
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        if (gj[j] >= r.n) continue;
        const uint64_t bound = r.thr[gj[j]];
        unsigned mask = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const bool ok = gi[i] < r.n && pack_key(exact_d2(nq[i], nr[j], acc[i][j]), gi[i]) < bound;
            mask |= (ok ? 1u : 0u) << i;
        }
        if (mask) {
            int slot = atomicAdd(&r.cnt[gj[j]], __popc(mask));
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (mask & (1u << i)) append_at(r, gj[j], slot++, pack_key(exact_d2(nq[i], nr[j], acc[i][j]), gi[i]));
        }
    }
}

// ------------------------------------------------------------------ merging
__device__ __forceinline__ void warp_bitonic_sort(uint64_t* buf, int m, int lane)
{
    for (int size = 2; size <= m; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = lane; t < (m >> 1); t += 32) {
                const int i = 2 * stride * (t / stride) + (t % stride);
                const int j = i + stride;
                const bool up = (i & size) == 0;
                const uint64_t a = buf[i], b = buf[j];
                if ((a > b) == up) {
                    buf[i] = b;
                    buf[j] = a;
                }
            }
            __syncwarp();
        }
    }
}

__host__ __device__ inline int next_pow2(int v)
{
    int m = 1;
    while (m < v) m <<= 1;
    return m;
}

// The tcgen05 filter bound of point p after a merge left its list threshold at key t: with the
// symmetric schedule (symb) the strict unfolded bound, else with a row image the folded bound and
// the row's w parts; the SIMT engine alone needs neither.
__device__ __forceinline__ void update_bound(uint64_t t, int p, float* U, const float* norms, int d, int kp,
                                             int exact, unsigned char* aimg, const float* ntf, int symb)
{
    const float T = (t == kEmptyKey) ? __int_as_float(0x7f800000) : __uint_as_float((uint32_t)(t >> 32));
    if (symb) {
        U[p] = strict_bound(filter_bound(T, norms[p], d, kp, exact));
    } else if (aimg) {
        float V, w;
        fold_bound(filter_bound(T, norms[p], d, kp, exact), ntf[p], kp, exact, V, w);
        U[p] = V;
        store_fold(aimg, p, d, kp, w);
    }
}

// one warp per point: list <- k-smallest of (list, new candidates); threshold <- list[k-1];
// with the tcgen05 engine also the filter bound (update_bound)
__global__ void knn_merge_kernel(uint64_t* __restrict__ lists, uint64_t* __restrict__ thr,
                                 float* __restrict__ U, const float* __restrict__ norms,
                                 const uint64_t* __restrict__ cand, int* __restrict__ cnt, int p0, int n,
                                 int k, int cap, int pw, int d, int kp, int exact,
                                 unsigned long long* __restrict__ admitted, unsigned char* __restrict__ aimg,
                                 const float* __restrict__ ntf, int symb, const int* __restrict__ stop)
{
    extern __shared__ uint64_t msm[];
    if (stop[0] | stop[1]) return;   // the round overflowed or an earlier one stopped: lists stay as they are
    const int warps = blockDim.x >> 5, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int p = p0 + blockIdx.x * warps + w;   // points [p0, n)
    if (p >= n) return;
    int c = cnt[p];
    if (c == 0) return;
    c = min(c, cap);
    uint64_t* buf = msm + (size_t)w * pw;
    const int tot = k + c, m = next_pow2(tot);
    const uint64_t* lp = lists + (size_t)p * k;
    const uint64_t* cp = cand + (size_t)p * cap;
    for (int t = lane; t < m; t += 32)
        buf[t] = (t < k) ? lp[t] : (t < tot ? cp[t - k] : kEmptyKey);
    __syncwarp();
    warp_bitonic_sort(buf, m, lane);
    uint64_t* lo = lists + (size_t)p * k;
    for (int t = lane; t < k; t += 32) lo[t] = buf[t];
    if (lane == 0) {
        const uint64_t t = buf[k - 1];
        thr[p] = t;
        cnt[p] = 0;
        update_bound(t, p, U, norms, d, kp, exact, aimg, ntf, symb);
        atomicAdd(admitted, (unsigned long long)c);
    }
}

// ---- the same merge without sorting the list: the candidates are sorted in registers (a bitonic
// network over 32*E keys, blocked layout: key e of lane l sits at position l*E + e; in-lane steps swap
// registers, cross-lane steps exchange with shfl_xor), then each output rank r < k is placed by a
// merge-path search over (list, sorted candidates) in shared memory. Shared memory is touched only
// to stage the two sorted runs, so the shared-memory traffic that bounds the sorting version goes.
template <int E>
__device__ __forceinline__ void warp_sort_regs(uint64_t (&v)[E], int lane)
{
    constexpr int m = 32 * E;
#pragma unroll
    for (int size = 2; size <= m; size <<= 1) {
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
            if (j < E) {
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const int e2 = e ^ j;
                    if (e2 > e) {
                        const bool asc = ((lane * E + e) & size) == 0;
                        const uint64_t a = v[e], b = v[e2];
                        if ((a > b) == asc) {
                            v[e] = b;
                            v[e2] = a;
                        }
                    }
                }
            } else {
                const int lx = j / E;
                const bool lower = (lane & lx) == 0;
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const uint64_t o = __shfl_xor_sync(0xffffffffu, v[e], lx);
                    const bool asc = ((lane * E + e) & size) == 0;
                    // keep the own key when it is the one this lane wants (the smaller one when
                    // taking the minimum): one 64-bit compare and one select per key
                    const bool keep = (v[e] < o) == (lower == asc);
                    v[e] = keep ? v[e] : o;
                }
            }
        }
    }
}

// number of list keys among the first r outputs of merge(list, cand), list first on ties
__device__ __forceinline__ int merge_split(const uint64_t* L, int nl, const uint64_t* C, int nc, int r)
{
    int lo = max(0, r - nc), hi = min(r, nl);
    while (lo < hi) {
        const int i = (lo + hi + 1) >> 1;   // try taking i list keys: needs L[i-1] <= C[r-i]
        if (L[i - 1] <= C[r - i]) lo = i;
        else hi = i - 1;
    }
    return lo;
}

template <int E>
__device__ __forceinline__ void merge_point_sorted(uint64_t* __restrict__ lists, const uint64_t* __restrict__ cp,
                                                   int c, int k, int p, uint64_t* sl, uint64_t* sc, int lane)
{
    uint64_t v[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int t = lane * E + e;
        v[e] = t < c ? cp[t] : kEmptyKey;
    }
    uint64_t* lp = lists + (size_t)p * k;
    for (int t = lane; t < k; t += 32) sl[t] = lp[t];
    warp_sort_regs<E>(v, lane);
#pragma unroll
    for (int e = 0; e < E; ++e) sc[lane * E + e] = v[e];
    __syncwarp();
    for (int r = lane; r < k; r += 32) {
        const int i = merge_split(sl, k, sc, c, r);
        const int j = r - i;
        lp[r] = (i < k && (j >= c || sl[i] <= sc[j])) ? sl[i] : sc[j];
    }
}

// one warp per point; k <= kSortedMergeMaxK and at most 512 candidates per point
constexpr int kSortedMergeMaxK = 256;
constexpr int kSortedMergeWarps = 8;

__global__ void __launch_bounds__(kSortedMergeWarps * 32, 4)
    knn_merge_sorted_kernel(uint64_t* __restrict__ lists, uint64_t* __restrict__ thr, float* __restrict__ U,
                            const float* __restrict__ norms, const uint64_t* __restrict__ cand,
                            int* __restrict__ cnt, int p0, int n, int k, int cap, int d, int kp, int exact,
                            unsigned long long* __restrict__ admitted, unsigned char* __restrict__ aimg,
                            const float* __restrict__ ntf, int symb, const int* __restrict__ stop)
{
    __shared__ uint64_t sl_all[kSortedMergeWarps][kSortedMergeMaxK];
    __shared__ uint64_t sc_all[kSortedMergeWarps][512];
    if (stop[0] | stop[1]) return;   // the round overflowed or an earlier one stopped: lists stay as they are
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int p = p0 + blockIdx.x * kSortedMergeWarps + w;   // points [p0, n)
    if (p >= n) return;
    int c = cnt[p];
    if (c == 0) return;
    c = min(c, cap);
    const uint64_t* cp = cand + (size_t)p * cap;
    uint64_t* sl = sl_all[w];
    uint64_t* sc = sc_all[w];
    if (c <= 32) merge_point_sorted<1>(lists, cp, c, k, p, sl, sc, lane);
    else if (c <= 64) merge_point_sorted<2>(lists, cp, c, k, p, sl, sc, lane);
    else if (c <= 128) merge_point_sorted<4>(lists, cp, c, k, p, sl, sc, lane);
    else if (c <= 256) merge_point_sorted<8>(lists, cp, c, k, p, sl, sc, lane);
    else merge_point_sorted<16>(lists, cp, c, k, p, sl, sc, lane);
    __syncwarp();
    if (lane == 0) {
        const uint64_t t = lists[(size_t)p * k + k - 1];
        thr[p] = t;
        cnt[p] = 0;
        update_bound(t, p, U, norms, d, kp, exact, aimg, ntf, symb);
        atomicAdd(admitted, (unsigned long long)c);
    }
}

// symmetric shards: the filter bounds from the thresholds just combined over the shards
__global__ void refresh_bounds_kernel(const uint64_t* __restrict__ thr, const float* __restrict__ norms,
                                      float* __restrict__ U, int n, int d, int kp, int exact)
{
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= n) return;
    const uint64_t t = thr[p];
    const float T = (t == kEmptyKey) ? __int_as_float(0x7f800000) : __uint_as_float((uint32_t)(t >> 32));
    U[p] = strict_bound(filter_bound(T, norms[p], d, kp, exact));
}

// per-point state before the first round: empty lists admit everything, padding nothing
__global__ void init_point_state_kernel(int n, int rows, float* __restrict__ norms, uint64_t* __restrict__ thr,
                                        float* __restrict__ U)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows) return;
    if (i < n) {
        thr[i] = kEmptyKey;
        U[i] = __int_as_float(0x7f800000);
    } else {
        norms[i] = 0.0f;
        thr[i] = 0;
        U[i] = __int_as_float(0xff800000);
    }
}

// dst <- k-smallest of dst and nsrc other lists of the same points
__global__ void merge_blocks_kernel(uint64_t* __restrict__ dst, const uint64_t* __restrict__ srcs,
                                   int nsrc, int n, int k, int pw)
{
    extern __shared__ uint64_t msm[];
    const int warps = blockDim.x >> 5, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int p = blockIdx.x * warps + w;
    if (p >= n) return;
    uint64_t* buf = msm + (size_t)w * pw;
    const int tot = k * (nsrc + 1), m = next_pow2(tot);
    for (int t = lane; t < m; t += 32) {
        uint64_t v = kEmptyKey;
        if (t < k) v = dst[(size_t)p * k + t];
        else if (t < tot) {
            const int b = t / k - 1, q = t % k;
            v = srcs[((size_t)b * n + p) * k + q];
        }
        buf[t] = v;
    }
    __syncwarp();
    warp_bitonic_sort(buf, m, lane);
    for (int t = lane; t < k; t += 32) dst[(size_t)p * k + t] = buf[t];
}

static void merge_launch_shape(int pw, int* warps, size_t* smem)
{
    // keep at most 48 KB of dynamic shared memory per CTA unless one warp needs more
    int w = (int)std::max<size_t>(1, std::min<size_t>(8, (48 * 1024) / ((size_t)pw * 8)));
    *warps = w;
    *smem = (size_t)w * pw * 8;
}

static void ensure_smem(const void* fn, size_t smem)
{
    if (smem > 48 * 1024)
        FDB_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
}

void merge_list_blocks(Workspace&, uint64_t* dst, const uint64_t* srcs, int nsrc, int n, int k,
                       cudaStream_t s)
{
    if (n <= 0 || k <= 0 || nsrc <= 0) return;
    const int pw = next_pow2(k * (nsrc + 1));
    FDB_REQUIRE((size_t)pw * 8 <= 200 * 1024, "merge of this many lists exceeds shared memory");
    int warps;
    size_t smem;
    merge_launch_shape(pw, &warps, &smem);
    ensure_smem((const void*)merge_blocks_kernel, smem);
    merge_blocks_kernel<<<(n + warps - 1) / warps, warps * 32, smem, s>>>(dst, srcs, nsrc, n, k, pw);
    FDB_LAUNCHED();
}

// ------------------------------------------------------------------ final ordering
// symtriknncuda.cu:225-251: sqrtf(max(d2, 0)) and the rank-major transpose
__global__ void lists_to_rank_major_kernel(const uint64_t* __restrict__ lists, int n, int k,
                                           float* __restrict__ dist, int* __restrict__ idx)
{
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= n) return;
    const uint64_t* lp = lists + (size_t)p * k;
    for (int q = 0; q < k; ++q) {
        const uint64_t key = lp[q];
        dist[(size_t)q * n + p] = sqrtf(fmaxf(__uint_as_float((uint32_t)(key >> 32)), 0.0f));
        idx[(size_t)q * n + p] = (int)(uint32_t)key;
    }
}

void lists_to_rank_major(const uint64_t* lists, int n, int k, float* dist, int* idx, cudaStream_t s)
{
    if (n <= 0 || k <= 0) return;
    lists_to_rank_major_kernel<<<(n + 127) / 128, 128, 0, s>>>(lists, n, k, dist, idx);
    FDB_LAUNCHED();
}

// ------------------------------------------------------------------ host scheduler
static long long shard_pairs(int n, int T, int b_lo, int b_hi)
{
    auto bsz = [&](int b) -> long long { return std::min(kBlock, n - b * kBlock); };
    const int dmax = T / 2;
    long long tot = 0;
    for (int b = b_lo; b < b_hi; ++b) {
        const long long mb = bsz(b);
        tot += mb * (mb - 1) / 2;
        // valid offsets for this row block
        int valid = dmax;
        if ((T & 1) == 0 && dmax >= 1 && b >= T / 2) valid -= 1;
        if (valid <= 0) continue;
        if (b == T - 1) {
            tot += mb * (long long)kBlock * valid;   // every partner of the last block is full
            continue;
        }
        tot += mb * (long long)kBlock * valid;
        // the one offset whose partner is the (possibly partial) last block
        const int d0 = T - 1 - b;
        const bool skipped = (T & 1) == 0 && d0 == T / 2 && b >= T / 2;
        if (d0 >= 1 && d0 <= dmax && !skipped) tot += mb * (bsz(T - 1) - kBlock);
    }
    return tot;
}

// timing events, created on first use and destroyed with the pool (also when a round throws)
struct EventPool {
    std::vector<cudaEvent_t> ev;
    cudaEvent_t get(int i)
    {
        while ((int)ev.size() <= i) {
            cudaEvent_t e;
            FDB_CUDA(cudaEventCreate(&e));
            ev.push_back(e);
        }
        return ev[i];
    }
    ~EventPool()
    {
        for (cudaEvent_t e : ev) cudaEventDestroy(e);
    }
};

static void launch_tile_round(const TileRound& r, int units, int engine, int precision, cudaStream_t s)
{
    if (engine == FDB200_ENGINE_TCGEN05) launch_tile_round_tc(r, units, precision, s);
    else launch_tile_round_simt(r, units, s);
}

KnnResult knn_lists(Workspace& ws, const float* x, const KnnConfig& cfg, cudaStream_t s)
{
    const int n = cfg.n, d = cfg.d, k = cfg.k;
    FDB_REQUIRE(n >= 2 && d >= 1 && k >= 1 && k < n, "kNN needs n >= 2, d >= 1 and 1 <= k < n");
    FDB_REQUIRE(cfg.shard_count >= 1 && cfg.shard_rank >= 0 && cfg.shard_rank < cfg.shard_count,
                "bad shard_rank / shard_count");
    KnnResult res;
    const int T = (n + kBlock - 1) / kBlock;
    int b_lo = (int)((long long)T * cfg.shard_rank / cfg.shard_count);
    int b_hi = (int)((long long)T * (cfg.shard_rank + 1) / cfg.shard_count);
    if (cfg.block_lo >= 0 || cfg.block_hi >= 0) {
        FDB_REQUIRE(0 <= cfg.block_lo && cfg.block_lo <= cfg.block_hi && cfg.block_hi <= T,
                    "shard_block_lo / shard_block_hi must satisfy 0 <= lo <= hi <= ceil(n / 128)");
        b_lo = cfg.block_lo;
        b_hi = cfg.block_hi;
    }
    const int nb = b_hi - b_lo;
    // admissions per round have a fat right tail (the list's k-th key is itself a random order
    // statistic), so rounds are sized for about a quarter of the buffer
    int cap = std::max(512, ((4 * k + 31) / 32) * 32);
    if (cfg.cand_capacity > 0) cap = std::max(256, cfg.cand_capacity);
    const int pw = next_pow2(k + cap);
    FDB_REQUIRE((size_t)pw * 8 <= 200 * 1024, "k too large for the list merge (k + capacity > 25600)");

    // per-point arrays cover the padded last block and one poison block (tcgen05 tiles read them)
    const int rows = T * kBlock + kBlock;
    float* norms = ws.norms.as<float>(rows);
    uint64_t* lists = ws.lists.as<uint64_t>((size_t)n * k);
    uint64_t* thr = ws.thr.as<uint64_t>(rows);
    float* U = ws.fthr.as<float>(rows);
    uint64_t* cand = ws.cand.as<uint64_t>((size_t)n * cap);
    int* cnt = ws.cnt.as<int>(n);
    int* ovf = ws.flags.as<int>(16);   // [0] overflow, [1] tcgen05 error, [2..3] admitted, [4] tcgen05 drain
                                       // timeout, [8..13] trace counters
    unsigned long long* admitted = reinterpret_cast<unsigned long long*>(ovf + 2);
    compute_norms(x, cfg.ldx, n, d, norms, s);
    init_point_state_kernel<<<(rows + 255) / 256, 256, 0, s>>>(n, rows, norms, thr, U);
    FDB_LAUNCHED();
    FDB_CUDA(cudaMemsetAsync(lists, 0xFF, sizeof(uint64_t) * (size_t)n * k, s));
    FDB_CUDA(cudaMemsetAsync(cnt, 0, sizeof(int) * (size_t)n, s));
    FDB_CUDA(cudaMemsetAsync(ovf, 0, sizeof(int) * 16, s));
    res.lists = lists;
    res.pairs = shard_pairs(n, T, b_lo, b_hi);

    int engine = cfg.engine;
    if (engine == FDB200_ENGINE_AUTO) engine = tc_engine_supported(d) ? FDB200_ENGINE_TCGEN05 : FDB200_ENGINE_SIMT;
    if (engine == FDB200_ENGINE_TCGEN05)
        FDB_REQUIRE(tc_engine_supported(d), "the tcgen05 engine does not support this dimension/device");
    FDB_REQUIRE(cfg.precision == FDB200_FP32 || engine == FDB200_ENGINE_TCGEN05,
                "TF32 distances need the tcgen05 engine");
    res.engine_used = engine;
    const int kp = tc_kp(d);
    const int exact = cfg.precision == FDB200_FP32 ? 1 : 0;
    // An unsharded tcgen05 call evaluates each unordered block pair once and tests both endpoints
    // (the symmetric schedule). A shard with a round hook does the same over the block pairs whose
    // first block is its own, keeps partial lists of every point and has its thresholds combined
    // with the other shards' through the hook after every round; a shard without one keeps ordered
    // pairs over its own rows, so that its lists are final without an exchange.
    const bool hooked = cfg.round_hook != nullptr;
    const int tc_sym = (engine == FDB200_ENGINE_TCGEN05 && (nb == T || hooked)) ? 1 : 0;
    TcFold fold;
    if (engine == FDB200_ENGINE_TCGEN05) fold = tc_prepare(ws, x, cfg.ldx, n, d, norms, U, thr, tc_sym, s);

    int mwarps;
    size_t msmem;
    merge_launch_shape(pw, &mwarps, &msmem);
    ensure_smem((const void*)knn_merge_kernel, msmem);

    TileRound r{};
    r.x = x; r.ldx = cfg.ldx; r.n = n; r.d = d; r.norms = norms; r.thr = thr; r.U = U; r.cand = cand;
    r.cnt = cnt; r.cap = cap; r.ovf = ovf; r.T = T; r.b_lo = b_lo; r.nb = nb; r.sym = tc_sym;

    // Rounds are queued back to back with no host check in between: the schedule below depends only on
    // host state, each tile kernel tags an overflow with its round, and every later kernel of the batch
    // sees the flag and does nothing. One settle per batch (normally one per fit) reads the flags; an
    // overflowed round is re-planned in halves from where it started, which is exact because lists only
    // change in the merges of rounds that completed. Host stalls between launches therefore do not
    // leave the device idle.
    struct Planned {
        int diag, delta0, ndelta, units, engine, rows_only;
        double seen;   // the `seen` estimate before the round
    };
    std::vector<Planned> plan;
    EventPool ev;
    const int dmax = T / 2;
    const char* trace_env = getenv("FDB200_TRACE");
    const bool trace = trace_env && trace_env[0] == '1';
    unsigned long long adm_before = 0, adm = 0;
    unsigned long long* counters = ws.misc2.as<unsigned long long>(16);   // trace counters
    r.counters = trace ? counters : nullptr;
    if (trace) FDB_CUDA(cudaMemsetAsync(counters, 0, 16 * sizeof(unsigned long long), s));
    bool diag_done = false;
    int next_delta = 1;
    double seen = kBlock - 1;   // candidates each point has been offered so far (approximate)
    int pending = 0;            // block offsets of a round being re-planned, 0 = none
    cudaEvent_t m0 = ev.get(0), m1 = ev.get(1);   // trace: merge timing
    for (;;) {
        // with a round hook every shard plans the same rounds, even an empty one (its launches do no
        // work), so that every shard makes the same hook calls
        const bool more = (nb > 0 || hooked) && (!diag_done || next_delta <= dmax);
        if (more) {
            Planned pl{};
            pl.seen = seen;
            if (!diag_done) {
                pl.diag = 1;
                pl.units = nb;
            } else {
                if (pending > 0) {
                    pl.ndelta = pending;
                } else {
                    // expected admissions per point ~ new * k / seen; keep them near cap / 4
                    const double want = (double)cap * seen / (8.0 * kBlock * k);
                    pl.ndelta = (int)std::max(1.0, std::min(want, (double)(dmax - next_delta + 1)));
                }
                pl.delta0 = next_delta;
                pl.units = nb * pl.ndelta;
            }
            // With the automatic engine, the first rounds run on the exact SIMT tiles: they offer every
            // point few, mostly admissible candidates (its thresholds are still loose), so nearly every
            // pair would be refined after the TF32 filter anyway (measured at the headline size: the
            // diagonal and the first three offset rounds take 28 ms instead of 67 ms). A sharded run
            // gives them rows-only SIMT tiles (each ordered block pair once, its own rows updated), so
            // a shard's lists are final without an exchange, as with its tcgen05 rounds. An explicit
            // tcgen05 request keeps tcgen05 for every round.
            pl.engine = (cfg.engine == FDB200_ENGINE_AUTO && engine == FDB200_ENGINE_TCGEN05 &&
                         (pl.diag || pl.ndelta <= kSimtRoundMaxOffsets))
                            ? FDB200_ENGINE_SIMT
                            : engine;
            pl.rows_only =
                (pl.engine == FDB200_ENGINE_SIMT && engine == FDB200_ENGINE_TCGEN05 && nb < T && !hooked) ? 1 : 0;
            if (pl.rows_only && !pl.diag) pl.units = 2 * nb * pl.ndelta;
            plan.push_back(pl);
            const int slot = (int)plan.size();
            r.diag = pl.diag;
            r.rows_only = pl.rows_only;
            r.delta0 = pl.delta0;
            r.ndelta = pl.ndelta;
            r.tag = slot;
            FDB_CUDA(cudaEventRecord(ev.get(2 * slot), s));
            launch_tile_round(r, pl.units, pl.engine, cfg.precision, s);
            FDB_CUDA(cudaEventRecord(ev.get(2 * slot + 1), s));
            // symmetric shards: the round's overflow tag and error code are combined (MAX) before the
            // merge, so every shard discards an overflowed round and re-plans it alike
            if (hooked) cfg.round_hook(cfg.round_hook_ctx, FDB200_HOOK_FLAGS, ovf, 2, (void*)s);
            if (trace) FDB_CUDA(cudaEventRecord(m0, s));
            // an ordered tcgen05 round (a shard without a hook) or a rows-only round appends only to this
            // shard's rows; a symmetric round (SIMT or tcgen05) to any point
            const bool own_rows = (pl.engine == FDB200_ENGINE_TCGEN05 && !tc_sym) || pl.rows_only;
            const int plo = own_rows ? b_lo * kBlock : 0;
            const int phi = own_rows ? std::min(n, b_hi * kBlock) : n;
            if (k <= kSortedMergeMaxK && cap <= 512)
                knn_merge_sorted_kernel<<<(phi - plo + kSortedMergeWarps - 1) / kSortedMergeWarps, kSortedMergeWarps * 32, 0, s>>>(
                    lists, thr, U, norms, cand, cnt, plo, phi, k, cap, d, kp, exact, admitted, fold.aimg, fold.ntf, fold.sym, ovf);
            else
                knn_merge_kernel<<<(phi - plo + mwarps - 1) / mwarps, mwarps * 32, msmem, s>>>(
                    lists, thr, U, norms, cand, cnt, plo, phi, k, cap, pw, d, kp, exact, admitted, fold.aimg, fold.ntf, fold.sym, ovf);
            FDB_LAUNCHED();
            if (hooked) {
                // every shard's k-th key bounds the union's: filter with the smallest (unsigned MIN)
                cfg.round_hook(cfg.round_hook_ctx, FDB200_HOOK_THRESHOLDS, thr, n, (void*)s);
                if (fold.sym) {
                    refresh_bounds_kernel<<<(n + 255) / 256, 256, 0, s>>>(thr, norms, U, n, d, kp, exact);
                    FDB_LAUNCHED();
                }
            }
            if (trace) FDB_CUDA(cudaEventRecord(m1, s));
            if (!diag_done) {
                diag_done = true;
            } else {
                next_delta += pl.ndelta;
                seen += 2.0 * kBlock * pl.ndelta;
                pending = 0;
            }
            if (!trace) continue;   // keep queueing; a trace settles (and prints) every round
        }
        if (plan.empty()) break;

        // settle the batch: flags and the admitted counter in one copy
        FDB_CUDA(cudaMemcpyAsync(ws.pinned, ovf, 8 * sizeof(int), cudaMemcpyDeviceToHost, s));
        unsigned long long cn[16] = {0};
        if (trace) FDB_CUDA(cudaMemcpyAsync(cn, counters, sizeof(cn), cudaMemcpyDeviceToHost, s));
        if (trace) FDB_CUDA(cudaMemsetAsync(counters, 0, sizeof(cn), s));
        FDB_CUDA(cudaStreamSynchronize(s));
        const int tag = ws.pinned[0], err = ws.pinned[1], drain_err = ws.pinned[4];
        std::memcpy(&adm, ws.pinned + 2, sizeof(adm));
        const int ran = tag > 0 ? tag : (int)plan.size();   // rounds after an overflowed one did nothing
        for (int i = 1; i <= (int)plan.size(); ++i) {
            float ms = 0.0f;
            FDB_CUDA(cudaEventElapsedTime(&ms, ev.get(2 * i), ev.get(2 * i + 1)));
            res.tile_ms += ms;
        }
        res.rounds += ran;
        if (err)
            throw Error(FDB200_EINTERNAL,
                        "tcgen05 tile kernel stopped on a bounded wait (code " + std::to_string(err) + ")" +
                            (drain_err ? std::string("; its drain of the ") + (drain_err == 1 ? "copies" : "MMAs") +
                                             " in flight also ran out, so the device may be unsafe to use"
                                       : std::string()));
        if (trace) {
            const Planned& pl = plan.back();
            float ms = 0.0f, merge_ms = 0.0f;
            FDB_CUDA(cudaEventElapsedTime(&ms, ev.get(2), ev.get(3)));
            FDB_CUDA(cudaEventElapsedTime(&merge_ms, m0, m1));
            const double chunks = (double)pl.units * 32.0;   // 8 warps x 4 chunks per 128 x 256 tile
            fprintf(stderr, "[fdb200] round %d %s delta0=%d ndelta=%d units=%d tile_ms=%.3f merge_ms=%.3f admitted=%llu"
                            " (%.1f/point) refined=%llu (%.2f/chunk) hit_chunks=%.1f%% drain_steps/hit_chunk=%.2f%s\n",
                    res.rounds, pl.diag ? "diag" : "offs", pl.delta0, pl.ndelta, pl.units, ms, merge_ms,
                    adm - adm_before, (double)(adm - adm_before) / n, cn[0], cn[0] / chunks,
                    100.0 * cn[1] / chunks, cn[1] ? (double)cn[2] / cn[1] : 0.0, tag ? " (overflow)" : "");
            adm_before = adm;
            if (pl.engine == FDB200_ENGINE_TCGEN05 && !pl.diag) {
                // per tcgen05 tile (counted by the MMA issuers), cycles per CTA role instance
                const double tiles = cn[3] > 0 ? (double)cn[3] : 1.0;
                const double per_f = tiles * 8.0;   // filter warp-tiles (each tile has one refine warp)
                fprintf(stderr, "[fdb200]   cycles/tile: producer wait cols %.0f rows %.0f | filter wait %.0f work %.0f |"
                                " refine wait %.0f work %.0f | entries/tile %.1f inline %llu | mma loop %.0f"
                                " (waits: row stage %.0f, accumulator %.0f)\n",
                        cn[4] / tiles, cn[5] / tiles, cn[9] / per_f, cn[10] / per_f, cn[11] / tiles, cn[12] / tiles,
                        cn[0] / tiles, cn[1], cn[15] / tiles, cn[6] / tiles, cn[7] / tiles);
            }
        }
        if (tag > 0) {
            // re-plan the overflowed round in halves; its partial appends are dropped
            const Planned pl = plan[tag - 1];
            res.overflow_reruns++;
            FDB_CUDA(cudaMemsetAsync(cnt, 0, sizeof(int) * (size_t)n, s));
            FDB_CUDA(cudaMemsetAsync(ovf, 0, sizeof(int), s));
            if (pl.diag || pl.ndelta <= 1)
                throw Error(FDB200_EINTERNAL, "candidate buffer overflow on a single-offset round");
            diag_done = true;
            next_delta = pl.delta0;
            seen = pl.seen;
            pending = pl.ndelta / 2;
        }
        plan.clear();
    }
    res.candidates = (long long)adm;
    return res;
}

// SIMT engine launcher; the tcgen05 engine lives in knn_tc.cu
void launch_tile_round_simt(const TileRound& r, int units, cudaStream_t s)
{
    if (units <= 0) return;
    knn_tile_simt<<<units, kSimtThreads, 0, s>>>(r);
    FDB_LAUNCHED();
}

}  // namespace fdb
