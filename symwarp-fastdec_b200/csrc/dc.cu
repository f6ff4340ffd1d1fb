// dc.cu -- DC reduction, center selection and label propagation.
//
// Reference: dc_reduction_cuda (dcreductioncuda.cu:189-545) materialises cores x N dot products
// with cuBLAS SGEMM in HBM and reduces them twice (stage A: nearest strictly denser point, stage
// B: rank = number of points closer than that parent); dc_select_centers_kernel
// (dcreductioncuda.cu:548-619) then runs on ONE thread. Here the dot products stay in registers
// (the same exact fmaf-chain tile as the kNN), both stages reduce on chip with one atomic per
// (core, CTA), and center selection is a block-parallel argmax with the reference's float
// expressions and tie order.
#include "fdb_internal.h"

#include <algorithm>
#include <cfloat>

namespace fdb {

namespace {

__device__ __forceinline__ uint64_t pack_key(float d2, int idx)
{
    return ((uint64_t)__float_as_uint(d2) << 32) | (uint32_t)idx;
}

__device__ __forceinline__ float exact_d2(float na, float nb, float dot)
{
    return fmaxf(__fadd_rn(__fadd_rn(na, nb), __fmul_rn(-2.0f, dot)), 0.0f);
}

constexpr int kT = 256;
constexpr int kDC = 32;

// 128 cores x 128 points of exact fmaf-chain dot products (d = 0..D-1), 8 x 8 per thread.
__device__ __forceinline__ void core_point_dots(const float* __restrict__ xc, int ldc, int ncores,
                                                const float* __restrict__ x, int ldx, int n, int d,
                                                int c0, int p0, float (&As)[kDC][kBlock],
                                                float (&Bs)[kDC][kBlock], float (&acc)[8][8])
{
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    for (int d0 = 0; d0 < d; d0 += kDC) {
        const int steps = min(kDC, d - d0);
        for (int e = tid; e < kDC * kBlock; e += kT) {
            const int dd = e / kBlock, p = e % kBlock;
            float va = 0.0f, vb = 0.0f;
            if (dd < steps) {
                if (c0 + p < ncores) va = xc[(size_t)(d0 + dd) * ldc + c0 + p];
                if (p0 + p < n) vb = x[(size_t)(d0 + dd) * ldx + p0 + p];
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
}

__device__ __forceinline__ int tile_row(int t, int ty) { return (t < 4) ? ty * 4 + t : 64 + ty * 4 + (t - 4); }

struct DcArgs {
    const float* xc;        // gathered core coordinates, dim-major (d x ldc)
    int ldc, ncores;
    const float* x;
    int ldx, n, d;
    int p_lo, p_hi;         // the points this call reduces over: [p_lo, p_hi)
    const float* norms;     // all points
    const float* den;       // all points
    const int* cores;       // global index of each core
    uint64_t* best;         // stage A result per core
    int* rank;              // stage B counter per core
};

// stage A (dcreductioncuda.cu:63-111): lexicographic min (d2, index) over strictly denser points
__global__ void __launch_bounds__(kT) dc_stage_a_kernel(DcArgs a)
{
    __shared__ __align__(16) float As[kDC][kBlock];
    __shared__ __align__(16) float Bs[kDC][kBlock];
    const int c0 = blockIdx.x * kBlock, p0 = a.p_lo + blockIdx.y * kBlock;
    float acc[8][8];
    core_point_dots(a.xc, a.ldc, a.ncores, a.x, a.ldx, a.p_hi, a.d, c0, p0, As, Bs, acc);
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float np[8], dp[8];
    int gp[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        gp[j] = p0 + tile_row(j, tx);
        np[j] = gp[j] < a.p_hi ? a.norms[gp[j]] : 0.0f;
        dp[j] = gp[j] < a.p_hi ? a.den[gp[j]] : -FLT_MAX;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int c = c0 + tile_row(i, ty);
        uint64_t best = kEmptyKey;
        if (c < a.ncores) {
            const int gc = a.cores[c];
            const float cden = a.den[gc], cn = a.norms[gc];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (gp[j] < a.p_hi && cden < dp[j]) {
                    const uint64_t key = pack_key(exact_d2(cn, np[j], acc[i][j]), gp[j]);
                    best = key < best ? key : best;
                }
            }
        }
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) {
            const uint64_t o = __shfl_xor_sync(0xffffffffu, best, off);
            best = o < best ? o : best;
        }
        if (tx == 0 && best != kEmptyKey) atomicMin((unsigned long long*)&a.best[c], (unsigned long long)best);
    }
}

// stage B (dcreductioncuda.cu:131-170): rank = number of ALL points with d2 < d2(parent)
__global__ void __launch_bounds__(kT) dc_stage_b_kernel(DcArgs a)
{
    __shared__ __align__(16) float As[kDC][kBlock];
    __shared__ __align__(16) float Bs[kDC][kBlock];
    const int c0 = blockIdx.x * kBlock, p0 = a.p_lo + blockIdx.y * kBlock;
    float acc[8][8];
    core_point_dots(a.xc, a.ldc, a.ncores, a.x, a.ldx, a.p_hi, a.d, c0, p0, As, Bs, acc);
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float np[8];
    int gp[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        gp[j] = p0 + tile_row(j, tx);
        np[j] = gp[j] < a.p_hi ? a.norms[gp[j]] : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int c = c0 + tile_row(i, ty);
        int cnt = 0;
        if (c < a.ncores) {
            const uint64_t b = a.best[c];
            if (b != kEmptyKey) {
                const float d2p = __uint_as_float((uint32_t)(b >> 32));
                const float cn = a.norms[a.cores[c]];
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (gp[j] < a.p_hi && exact_d2(cn, np[j], acc[i][j]) < d2p) ++cnt;
            }
        }
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
        if (tx == 0 && cnt > 0) atomicAdd(&a.rank[c], cnt);
    }
}

__global__ void gather_cores_kernel(const float* __restrict__ x, int ldx, int d, const int* __restrict__ cores,
                                    int ncores, int ldc, float* __restrict__ xc, const float* __restrict__ den,
                                    float* __restrict__ core_den)
{
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (size_t)ncores * d) return;
    const int dd = (int)(t / ncores), c = (int)(t % ncores);
    xc[(size_t)dd * ldc + c] = x[(size_t)dd * ldx + cores[c]];
    if (dd == 0) core_den[c] = den[cores[c]];
}

__global__ void core_den_kernel(const float* __restrict__ den, const int* __restrict__ cores, int ncores,
                                float* __restrict__ core_den)
{
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < ncores) core_den[c] = den[cores[c]];
}

// dc_cb_split_packed + dc_cb_finalize (dcreductioncuda.cu:113-129, 172-187)
__global__ void dc_finalize_kernel(const uint64_t* __restrict__ best, int* __restrict__ rank, int ncores,
                                   int* __restrict__ parent, float* __restrict__ delta)
{
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= ncores) return;
    const uint64_t b = best[c];
    if (b == kEmptyKey) {
        parent[c] = -1;
        delta[c] = -1.0f;
        rank[c] = -1;
    } else {
        parent[c] = (int)(uint32_t)b;
        delta[c] = sqrtf(__uint_as_float((uint32_t)(b >> 32)));
        if (rank[c] == 0) rank[c] = -1;
    }
}

// dcreductioncuda.cu:548-619 with a block-parallel argmax. Same float expressions, same
// tie order (highest score, then lowest core position).
__global__ void __launch_bounds__(1024) select_centers_kernel(const float* __restrict__ core_den,
                                                              const float* __restrict__ g_in,
                                                              const int* __restrict__ k_in,
                                                              const int* __restrict__ core_idx, int core_nb,
                                                              int num_centers, unsigned char* __restrict__ chosen,
                                                              int* __restrict__ centers)
{
    __shared__ float sf[6][32];
    __shared__ int si[2][32];
    __shared__ float bsd[32];
    __shared__ int bidx[32];
    const int t = threadIdx.x, lane = t & 31, w = t >> 5, nw = blockDim.x >> 5;
    if (core_nb <= 0 || num_centers <= 0) return;
    // fills: max of the valid values, starting from -1 (dcreductioncuda.cu:559-564)
    float gmax = -1.0f;
    int kmax = -1;
    for (int i = t; i < core_nb; i += blockDim.x) {
        gmax = fmaxf(gmax, g_in[i]);
        kmax = max(kmax, k_in[i]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, off));
        kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, off));
    }
    if (lane == 0) {
        sf[0][w] = gmax;
        si[0][w] = kmax;
    }
    __syncthreads();
    float g_fill = -1.0f;
    int k_fill = -1;
    for (int i = 0; i < nw; ++i) {
        g_fill = fmaxf(g_fill, sf[0][i]);
        k_fill = max(k_fill, si[0][i]);
    }
    __syncthreads();
    float mn[3] = {FLT_MAX, FLT_MAX, FLT_MAX}, mx[3] = {-FLT_MAX, -FLT_MAX, -FLT_MAX};
    for (int i = t; i < core_nb; i += blockDim.x) {
        const float v[3] = {core_den[i], (g_in[i] < 0.0f) ? g_fill : g_in[i],
                            (float)((k_in[i] < 0) ? k_fill : k_in[i])};
#pragma unroll
        for (int q = 0; q < 3; ++q) {
            mn[q] = fminf(mn[q], v[q]);
            mx[q] = fmaxf(mx[q], v[q]);
        }
    }
#pragma unroll
    for (int q = 0; q < 3; ++q)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            mn[q] = fminf(mn[q], __shfl_xor_sync(0xffffffffu, mn[q], off));
            mx[q] = fmaxf(mx[q], __shfl_xor_sync(0xffffffffu, mx[q], off));
        }
    if (lane == 0)
        for (int q = 0; q < 3; ++q) {
            sf[q][w] = mn[q];
            sf[3 + q][w] = mx[q];
        }
    __syncthreads();
    float lo[3] = {FLT_MAX, FLT_MAX, FLT_MAX}, hi[3] = {-FLT_MAX, -FLT_MAX, -FLT_MAX};
    for (int i = 0; i < nw; ++i)
        for (int q = 0; q < 3; ++q) {
            lo[q] = fminf(lo[q], sf[q][i]);
            hi[q] = fmaxf(hi[q], sf[3 + q][i]);
        }
    const float den_range = __fsub_rn(hi[0], lo[0]);
    const float g_range = __fsub_rn(hi[1], lo[1]);
    const float k_range = __fsub_rn(hi[2], lo[2]);
    for (int i = t; i < core_nb; i += blockDim.x) chosen[i] = 0;
    __syncthreads();
    const int select_n = min(num_centers, core_nb);
    for (int sel = 0; sel < select_n; ++sel) {
        float best_sd = -FLT_MAX;
        int best = -1;
        for (int i = t; i < core_nb; i += blockDim.x) {
            if (chosen[i]) continue;
            const float dn = core_den[i];
            const float g = (g_in[i] < 0.0f) ? g_fill : g_in[i];
            const float kk = (float)((k_in[i] < 0) ? k_fill : k_in[i]);
            const float den_n = (den_range == 0.0f) ? 1.0f : __fdiv_rn(__fsub_rn(dn, lo[0]), den_range);
            const float g_n = (g_range == 0.0f) ? 1.0f : __fdiv_rn(__fsub_rn(g, lo[1]), g_range);
            const float k_n = (k_range == 0.0f) ? 1.0f : __fdiv_rn(__fsub_rn(kk, lo[2]), k_range);
            const float sd = __fmul_rn(__fmul_rn(den_n, g_n), k_n);
            if (sd > best_sd || (sd == best_sd && best < 0)) {
                best_sd = sd;
                best = i;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float osd = __shfl_xor_sync(0xffffffffu, best_sd, off);
            const int oi = __shfl_xor_sync(0xffffffffu, best, off);
            if (oi >= 0 && (best < 0 || osd > best_sd || (osd == best_sd && oi < best))) {
                best_sd = osd;
                best = oi;
            }
        }
        if (lane == 0) {
            bsd[w] = best_sd;
            bidx[w] = best;
        }
        __syncthreads();
        if (t == 0) {
            float bs = -FLT_MAX;
            int bi = -1;
            for (int i = 0; i < nw; ++i) {
                const int oi = bidx[i];
                const float osd = bsd[i];
                if (oi >= 0 && (bi < 0 || osd > bs || (osd == bs && oi < bi))) {
                    bs = osd;
                    bi = oi;
                }
            }
            centers[sel] = (bi >= 0) ? core_idx[bi] : -1;
            if (bi >= 0) chosen[bi] = 1;
        }
        __syncthreads();
    }
    for (int sel = select_n + t; sel < num_centers; sel += blockDim.x) centers[sel] = -1;
}

__global__ void scatter_kernel(const int* __restrict__ cores, const int* __restrict__ vals, int count,
                               int* __restrict__ out)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) out[cores[i]] = vals[i];
}

// ------------------------------------------------------------------ labels
__global__ void center_labels_kernel(const int* __restrict__ centers, int c, int n, int* __restrict__ lab)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < c && centers[i] >= 0 && centers[i] < n) lab[centers[i]] = i;
}

__global__ void init_roots_kernel(const int* __restrict__ parent, const int* __restrict__ clab, int n,
                                  int* __restrict__ root)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int p = parent[i];
    root[i] = (clab[i] >= 0 || p < 0 || p >= n) ? i : p;
}

__global__ void jump_kernel(const int* __restrict__ src, int n, int* __restrict__ dst)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = src[src[i]];
}

__global__ void assign_labels_kernel(const int* __restrict__ root, const int* __restrict__ clab, int n,
                                     int* __restrict__ labels, int* __restrict__ not_converged)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int r = root[i];
    if (root[r] != r) atomicOr(not_converged, 1);
    const int l = clab[r];
    labels[i] = (l >= 0) ? l : 0;
}

}  // namespace

namespace {

// scratch of the DC stages: the gathered core coordinates, dim-major (d x ldc)
struct DcScratch {
    int ldc;
    float* xc;
    float* core_den;   // written by the gather, unused by the stages
};

DcScratch dc_scratch(Workspace& ws, int core_nb, int d)
{
    DcScratch t;
    t.ldc = ((core_nb + kBlock - 1) / kBlock) * kBlock;
    const size_t xc_bytes = ((sizeof(float) * (size_t)t.ldc * d + 255) & ~size_t(255));
    // also room for dc_select's per-core scratch, which reuses this buffer once the stages are done
    const size_t sel_bytes = 3 * (((size_t)t.ldc * 4 + 255) & ~size_t(255)) + (size_t)t.ldc + 256;
    char* base = (char*)ws.dc_tmp.ensure(std::max(xc_bytes + sizeof(float) * (size_t)t.ldc + 256, sel_bytes));
    t.xc = (float*)base;
    t.core_den = (float*)(base + xc_bytes);
    return t;
}

void gather_cores(const DcScratch& t, const float* x, int ldx, int d, const float* den, const int* cores, int core_nb,
                  cudaStream_t s)
{
    FDB_CUDA(cudaMemsetAsync(t.xc, 0, sizeof(float) * (size_t)t.ldc * d, s));
    const size_t tot = (size_t)core_nb * d;
    gather_cores_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(x, ldx, d, cores, core_nb, t.ldc, t.xc, den,
                                                                       t.core_den);
    FDB_LAUNCHED();
}

void launch_stage(int stage, const DcScratch& t, const float* x, int ldx, int n, int d, const float* norms,
                  const float* den, const int* cores, int core_nb, int p_lo, int p_hi, uint64_t* best, int* rank,
                  cudaStream_t s)
{
    if (p_hi <= p_lo) return;
    DcArgs a{t.xc, t.ldc, core_nb, x, ldx, n, d, p_lo, p_hi, norms, den, cores, best, rank};
    dim3 grid((core_nb + kBlock - 1) / kBlock, (p_hi - p_lo + kBlock - 1) / kBlock);
    if (stage == 0) dc_stage_a_kernel<<<grid, kT, 0, s>>>(a);
    else dc_stage_b_kernel<<<grid, kT, 0, s>>>(a);
    FDB_LAUNCHED();
}

}  // namespace

void dc_reduction(Workspace& ws, const float* x, int ldx, int n, int d, const float* norms, const float* den,
                  const int* cores, int core_nb, int num_centers, int* core_parent, int* centers,
                  cudaStream_t s)
{
    FDB_REQUIRE(core_nb > 0 && num_centers > 0 && n > 0 && d > 0, "DC reduction: empty input");
    const DcScratch t = dc_scratch(ws, core_nb, d);
    uint64_t* best = ws.dc_sel.as<uint64_t>((size_t)2 * core_nb + 64);   // best keys, then ranks
    int* rank = reinterpret_cast<int*>(best + core_nb);
    gather_cores(t, x, ldx, d, den, cores, core_nb, s);
    FDB_CUDA(cudaMemsetAsync(best, 0xFF, sizeof(uint64_t) * core_nb, s));
    FDB_CUDA(cudaMemsetAsync(rank, 0, sizeof(int) * core_nb, s));
    launch_stage(0, t, x, ldx, n, d, norms, den, cores, core_nb, 0, n, best, rank, s);
    launch_stage(1, t, x, ldx, n, d, norms, den, cores, core_nb, 0, n, best, rank, s);
    dc_select(ws, den, cores, core_nb, best, rank, num_centers, core_parent, centers, s);
}

void dc_stage_range(Workspace& ws, int stage, const float* x, int ldx, int n, int d, const float* norms,
                    const float* den, const int* cores, int core_nb, int p_lo, int p_hi, uint64_t* best, int* rank,
                    cudaStream_t s)
{
    FDB_REQUIRE(core_nb > 0 && n > 0 && d > 0 && 0 <= p_lo && p_lo <= p_hi && p_hi <= n,
                "DC reduction stage: bad core count or point range");
    const DcScratch t = dc_scratch(ws, core_nb, d);
    gather_cores(t, x, ldx, d, den, cores, core_nb, s);
    if (stage == 0) FDB_CUDA(cudaMemsetAsync(best, 0xFF, sizeof(uint64_t) * core_nb, s));
    else FDB_CUDA(cudaMemsetAsync(rank, 0, sizeof(int) * core_nb, s));
    launch_stage(stage, t, x, ldx, n, d, norms, den, cores, core_nb, p_lo, p_hi, best, rank, s);
}

void dc_select(Workspace& ws, const float* den, const int* cores, int core_nb, const uint64_t* best, const int* rank_in,
               int num_centers, int* core_parent, int* centers, cudaStream_t s)
{
    FDB_REQUIRE(core_nb > 0 && num_centers > 0, "DC selection: empty input");
    // per core: density, delta, a working copy of the rank (finalize fills it), chosen flag -- after
    // the stages' best keys and ranks, which may live in the same buffer
    const size_t c4 = ((size_t)core_nb * 4 + 255) & ~size_t(255);
    char* base = (char*)ws.dc_tmp.ensure(3 * c4 + (size_t)core_nb + 256);
    float* core_den = (float*)base;
    float* delta = (float*)(base + c4);
    int* rank = (int*)(base + 2 * c4);
    unsigned char* chosen = (unsigned char*)(base + 3 * c4);
    core_den_kernel<<<(core_nb + 255) / 256, 256, 0, s>>>(den, cores, core_nb, core_den);
    FDB_LAUNCHED();
    FDB_CUDA(cudaMemcpyAsync(rank, rank_in, sizeof(int) * core_nb, cudaMemcpyDeviceToDevice, s));
    dc_finalize_kernel<<<(core_nb + 255) / 256, 256, 0, s>>>(best, rank, core_nb, core_parent, delta);
    FDB_LAUNCHED();
    select_centers_kernel<<<1, 1024, 0, s>>>(core_den, delta, rank, cores, core_nb, num_centers, chosen, centers);
    FDB_LAUNCHED();
}

void scatter_core_parents(const int* cores, const int* core_parent, int core_nb, int* parent, cudaStream_t s)
{
    if (core_nb <= 0) return;
    scatter_kernel<<<(core_nb + 255) / 256, 256, 0, s>>>(cores, core_parent, core_nb, parent);
    FDB_LAUNCHED();
}

void final_cluster(Workspace& ws, const int* parent, int n, const int* centers, int c, int* labels,
                   cudaStream_t s)
{
    if (n <= 0) return;
    int* clab = ws.labels_tmp.as<int>(3 * (size_t)n + 32);
    int* r0 = clab + n;
    int* r1 = r0 + n;
    int* flag = r1 + n;
    FDB_CUDA(cudaMemsetAsync(clab, 0xFF, sizeof(int) * (size_t)n, s));
    FDB_CUDA(cudaMemsetAsync(flag, 0, sizeof(int), s));
    const int blocks = (n + 255) / 256;
    if (c > 0) {
        center_labels_kernel<<<(c + 255) / 256, 256, 0, s>>>(centers, c, n, clab);
        FDB_LAUNCHED();
    }
    init_roots_kernel<<<blocks, 256, 0, s>>>(parent, clab, n, r0);
    FDB_LAUNCHED();
    // every chain is at most n long; ceil(log2 n) doublings reach its end
    int rounds = 1;
    while ((1ll << rounds) < (long long)n) ++rounds;
    int* cur = r0;
    int* nxt = r1;
    for (int t = 0; t < rounds; ++t) {
        jump_kernel<<<blocks, 256, 0, s>>>(cur, n, nxt);
        FDB_LAUNCHED();
        std::swap(cur, nxt);
    }
    assign_labels_kernel<<<blocks, 256, 0, s>>>(cur, clab, n, labels, flag);
    FDB_LAUNCHED();
    FDB_CUDA(cudaMemcpyAsync(ws.pinned + 12, flag, sizeof(int), cudaMemcpyDeviceToHost, s));
    FDB_CUDA(cudaStreamSynchronize(s));
    if (ws.pinned[12])
        throw Error(FDB200_ECYCLE, "label propagation did not converge (cycle in the parent links)");
}

}  // namespace fdb
