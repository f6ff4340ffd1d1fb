// knn_tc.cu -- tcgen05 (5th-generation tensor core) distance-tile engine for sm_100a.
//
// What it computes is exactly what knn_tile_simt computes (the reference FDS build's d2 and the
// lexicographic admission, see knn.cu); only the way candidates are found differs:
//
//   1. TF32 filter on the tensor cores. Every coordinate is rounded to TF32 (nearest) once,
//      x~ = rna(x), and each point is stored twice, K = D + 6 padded to 8:
//          A row i = [-2 x~_i, 1, 1, 1, nh_i, nm_i, nl_i, 0...]
//          B row j = [x~_j, nh_j, nm_j, nl_j, 1, 1, 1, 0...]
//      with nh + nm + nl = |x~|^2 (fmaf chain) split into three TF32-exact parts. Every operand is
//      exactly representable in TF32, so the 128 x 256 x K TF32 MMA gives
//      acc(i, j) = |x~_i - x~_j|^2 up to FP32 accumulation, straight in TMEM.
//   2. Rigorous margin (filter_bound in knn_common.cuh): a candidate that can still enter point
//      i's list always has acc <= U_i, so filtering on acc <= U never changes the result.
//   3. Exact refine. A pair passing acc <= U_row or acc <= U_col is recomputed with the sequential
//      fmaf chain on the ORIGINAL FP32 coordinates (a point-major copy in global memory) and
//      admitted with the exact lexicographic test. Precision TF32 skips the refine and keeps
//      d2 = max(acc, 0).
//
// Kernel shape (persistent, one CTA per SM, 13 warps):
//   warp 0       producer: cp.async.bulk copies of the A tile (128 rows, resident for a work item)
//                and of three B stages (two 128-point blocks = 256 rows each), stored in global
//                memory as pre-swizzled 4 KB K panels (the SWIZZLE_32B K-major layout), plus the
//                filter bounds of the tile's rows and columns
//   warp 1       TMEM owner and MMA issuer (one thread): K/8 tcgen05.mma kind::tf32 per tile into
//                one of two 256-column TMEM accumulators, tcgen05.commit to an mbarrier
//   warps 2..9   filter: tcgen05.ld 32 columns at a time (two loads in flight), two-sided bound
//                test into per-row survivor masks, one queue entry per (row, 32 columns) with
//                survivors; then the accumulator and the B stage are released at once
//   warps 10..12 refine: warp r owns the tiles g = r mod 3 and drains their queues (exact refine
//                from global memory, admission, append), off the filter's critical path
// Every mbarrier wait is bounded (about a second); on a timeout the CTA records an error code,
// stops issuing work, frees its TMEM and returns, and the host reports the failure.
#include "knn_common.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace fdb {

namespace tc {

constexpr int kFilterWarps = 8;
constexpr int kRefineWarps = 3;
constexpr int kThreads = 32 * (2 + kFilterWarps + kRefineWarps);
constexpr int kRows = 128;               // A rows per tile
constexpr int kCols = 256;               // B rows per tile (two blocks)
constexpr int kStages = 3;               // B stages in shared memory
constexpr int kQueues = 4;               // survivor queues between filter and refine warps
constexpr int kQueueCap = 256;           // entries per queue
constexpr int kMaxKp = 64;               // K up to 64 floats (eight 32-byte panels)
constexpr long long kWaitCycles = 2000000000ll;   // ~1 s at 2 GHz
constexpr float kPoisonNorm = 1.2676506002282294e30f;   // 2^100, exact in TF32

struct Args {
    int n, d, kp, dp, T, b_lo, nb, cap, exact;
    int diag, delta0, ndelta, npairs, pairs_per_item, items;
    int row_pad;                 // Npad: first poison row of the B array
    const float* U;              // filter bounds (Npad + 128)
    const float* nrm;            // exact fp32 norms (Npad + 128)
    const uint64_t* thr;         // exact admission thresholds (Npad + 128)
    const float* xp;             // original coordinates, point-major, dp floats per row
    const unsigned char* aimg;   // A operand: per 128-row block, K/8 pre-swizzled 4 KB panels
    const unsigned char* bimg;   // B operand, same layout (Npad + 128 rows)
    uint64_t* cand;
    int* cnt;
    int* ovf;
    int* err;
    unsigned long long* counters;   // optional trace counters
};

// ------------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
// try_wait with a suspend-time hint: the thread sleeps until the phase completes (or ~1 ms
// passes) instead of spinning, so waiting roles do not take issue slots from the filter
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}

// trace-mode phase timers: cycles accumulated per role, added to counters[4 + slot] at the end
enum {
    kTProdWaitA, kTProdWaitB, kTMmaWaitA, kTMmaWaitB, kTMmaWaitAcc, kTFiltWait, kTFiltWork, kTRefWait, kTRefWork,
    kTNum
};

// bounded wait: false on timeout or when another role aborted the CTA
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code)
{
    const long long t0 = clock64();
    while (!mbar_try_wait(b, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > kWaitCycles) {
            *abort_flag = 1;
            atomicCAS(err, 0, code);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     su32(dst)),
                 "l"(src), "r"(bytes), "r"(su32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, SWIZZLE_32B panel: rows 32 B apart, 8-row groups 256 B apart
__device__ __forceinline__ uint64_t sw32_desc(uint32_t saddr)
{
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(256 >> 4) << 32;   // stride byte offset: 8 rows x 32 B
    d |= (uint64_t)1 << 46;            // descriptor version for sm_100
    d |= (uint64_t)6 << 61;            // SWIZZLE_32B
    return d;
}

// kind::tf32, D = F32, A = B = TF32, both K-major, M = 128, N = 256
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kCols >> 3) << 17) |
                            ((uint32_t)(kRows >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accum)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accum)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
                 : "memory");
}

// tcgen05.ld of 32 consecutive accumulator columns of this thread's TMEM lane; the registers are
// valid only after tmem_wait on the same array (the wait names them, so no use moves above it)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait(uint32_t (&r)[32])
{
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// ------------------------------------------------------------------ shared memory plan
struct Smem {
    // offsets in bytes from the 1024-aligned base
    uint32_t a, b[kStages], arow_u, bcol_u[kStages], queue, qcount, bars, misc, total;
};

__host__ __device__ inline Smem smem_plan(int kp)
{
    Smem s;
    const uint32_t panels = (uint32_t)kp / 8;
    uint32_t o = 0;
    s.a = o;
    o += panels * kRows * 32;
    for (int q = 0; q < kStages; ++q) {
        s.b[q] = o;
        o += panels * kCols * 32;
    }
    s.arow_u = o;
    o += kRows * 4;
    for (int q = 0; q < kStages; ++q) {
        s.bcol_u[q] = o;
        o += kCols * 4;
    }
    s.queue = o;                       // per queue: rows[cap], first columns[cap], row masks, column masks
    o += (uint32_t)kQueues * kQueueCap * 16u;
    s.qcount = o;
    o += 16 * 4;
    s.bars = o;
    o += 24 * 8;
    s.misc = o;
    o += 64;
    s.total = o;
    return s;
}

// unit (item, index inside item) -> Q block and the two R blocks (-1 = poison half)
struct Unit {
    int B, R0, R1;
};

__device__ __forceinline__ int item_units(const Args& a, int item, int& p_lo)
{
    if (a.diag) {
        p_lo = 0;
        return 1;
    }
    const int chunk = item / a.nb;
    p_lo = chunk * a.pairs_per_item;
    return min(a.npairs, p_lo + a.pairs_per_item) - p_lo;
}

__device__ __forceinline__ Unit make_unit(const Args& a, int item, int p)
{
    Unit u;
    u.B = a.b_lo + item % a.nb;
    if (a.diag) {
        u.R0 = u.B;
        u.R1 = -1;
        return u;
    }
    int Rs[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int off = 2 * p + h;
        const int dl = a.delta0 + off;
        int R = -1;
        if (off < a.ndelta && !((a.T & 1) == 0 && dl == a.T / 2 && u.B >= a.T / 2)) {
            R = u.B + dl;
            if (R >= a.T) R -= a.T;
        }
        Rs[h] = R;
    }
    u.R0 = Rs[0];
    u.R1 = Rs[1];
    return u;
}

__device__ __forceinline__ void tc_append(const Args& a, int p, uint64_t key)
{
    const int slot = atomicAdd(&a.cnt[p], 1);
    if (slot < a.cap) a.cand[(size_t)p * a.cap + slot] = key;
    else atomicOr(a.ovf, 1);
}

// exact d2 of two points from the point-major original coordinates: fmaf chain over d = 0..D-1
// (the zero padding is never fed to the chain: fmaf(0, 0, -0) would turn a -0 dot into +0)
__device__ __forceinline__ float refine_global(const Args& a, int gi, int gj)
{
    const float* xi = a.xp + (size_t)gi * a.dp;
    const float* xj = a.xp + (size_t)gj * a.dp;
    const float4* xi4 = reinterpret_cast<const float4*>(xi);
    const float4* xj4 = reinterpret_cast<const float4*>(xj);
    float dot = 0.0f;
    const int full = a.d >> 2;
    for (int c = 0; c < full; ++c) {
        const float4 u = __ldg(xi4 + c), v = __ldg(xj4 + c);
        dot = __fmaf_rn(u.x, v.x, dot);
        dot = __fmaf_rn(u.y, v.y, dot);
        dot = __fmaf_rn(u.z, v.z, dot);
        dot = __fmaf_rn(u.w, v.w, dot);
    }
    for (int k = full * 4; k < a.d; ++k) dot = __fmaf_rn(__ldg(xi + k), __ldg(xj + k), dot);
    return exact_d2(__ldg(a.nrm + gi), __ldg(a.nrm + gj), dot);
}

// the survivors of one (row gi, 32 columns from gj0): exact refine and admission on both sides
__device__ __forceinline__ void settle_exact(const Args& a, int gi, int gj0, unsigned mr, unsigned mc)
{
    for (unsigned mm = mr | mc; mm; mm &= mm - 1) {
        const int q = __ffs(mm) - 1;
        const int gj = gj0 + q;
        if (gj == gi || gj >= a.n) continue;
        const float d2 = refine_global(a, gi, gj);
        if ((mr >> q) & 1u) {
            const uint64_t key = pack_key(d2, gj);
            if (key < __ldg(a.thr + gi)) tc_append(a, gi, key);
        }
        if ((mc >> q) & 1u) {
            const uint64_t key = pack_key(d2, gi);
            if (key < __ldg(a.thr + gj)) tc_append(a, gj, key);
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1) knn_tile_tc(Args a)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* sm = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const Smem P = smem_plan(a.kp);
    const int panels = a.kp / 8;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + P.bars);
    uint64_t* a_full = bars + 0;
    uint64_t* a_empty = bars + 1;
    uint64_t* b_full = bars + 2;                     // [kStages]
    uint64_t* b_empty = b_full + kStages;            // [kStages]
    uint64_t* acc_full = b_empty + kStages;          // [2]
    uint64_t* acc_empty = acc_full + 2;              // [2]
    uint64_t* q_full = acc_empty + 2;                // [kQueues]
    uint64_t* q_free = q_full + kQueues;             // [kQueues]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + P.misc);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + P.misc + 16);
    int* qcount = reinterpret_cast<int*>(sm + P.qcount);
    int* qbase = reinterpret_cast<int*>(sm + P.queue);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(a_full, 1);
        mbar_init(a_empty, kFilterWarps);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], kFilterWarps);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], kFilterWarps);
        }
        for (int q = 0; q < kQueues; ++q) {
            mbar_init(&q_full[q], kFilterWarps);
            mbar_init(&q_free[q], 1);
            qcount[q] = 0;
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const uint32_t a_bytes = (uint32_t)panels * kRows * 32;   // one 128-row block of an image

    if (warp == 0) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            int g = 0;
            bool ok = true;
            long long tw[2] = {0, 0};
            for (int t = 0, item = blockIdx.x; ok && item < a.items; ++t, item += gridDim.x) {
                long long c0 = clock64();
                if (!mbar_wait(a_empty, (t & 1) ^ 1, abort_flag, a.err, 1)) { ok = false; break; }
                tw[0] += clock64() - c0;
                const int B = a.b_lo + item % a.nb;
                mbar_expect_tx(a_full, a_bytes + kRows * 4);
                bulk_load(sm + P.a, a.aimg + (size_t)B * a_bytes, a_bytes, a_full);
                bulk_load(sm + P.arow_u, a.U + (size_t)B * kRows, kRows * 4, a_full);
                int p_lo;
                const int nu = item_units(a, item, p_lo);
                for (int uix = 0; uix < nu; ++uix, ++g) {
                    const int s = g % kStages;
                    c0 = clock64();
                    if (!mbar_wait(&b_empty[s], ((g / kStages) & 1) ^ 1, abort_flag, a.err, 2)) { ok = false; break; }
                    tw[1] += clock64() - c0;
                    const Unit u = make_unit(a, item, p_lo + uix);
                    unsigned char* bb = sm + P.b[s];
                    mbar_expect_tx(&b_full[s], 2 * a_bytes + 2 * kRows * 4);
                    const int blk0 = (u.R0 >= 0 ? u.R0 : a.row_pad / kRows);
                    const int blk1 = (u.R1 >= 0 ? u.R1 : a.row_pad / kRows);
                    const unsigned char* img0 = a.bimg + (size_t)blk0 * a_bytes;
                    const unsigned char* img1 = a.bimg + (size_t)blk1 * a_bytes;
                    for (int p = 0; p < panels; ++p) {
                        bulk_load(bb + p * kCols * 32, img0 + p * kRows * 32, kRows * 32, &b_full[s]);
                        bulk_load(bb + p * kCols * 32 + kRows * 32, img1 + p * kRows * 32, kRows * 32, &b_full[s]);
                    }
                    bulk_load(sm + P.bcol_u[s], a.U + (size_t)blk0 * kRows, kRows * 4, &b_full[s]);
                    bulk_load(sm + P.bcol_u[s] + kRows * 4, a.U + (size_t)blk1 * kRows, kRows * 4, &b_full[s]);
                }
            }
            if (a.counters) {
                atomicAdd(&a.counters[4 + kTProdWaitA], (unsigned long long)tw[0]);
                atomicAdd(&a.counters[4 + kTProdWaitB], (unsigned long long)tw[1]);
            }
            // on abort, let the copies already issued land before the CTA exits (bounded)
            if (!ok) {
                const long long t0 = clock64();
                for (int q = 0; q < kStages && q < g; ++q) {
                    const int gl = g - 1 - q;
                    while (!mbar_try_wait(&b_full[gl % kStages], (gl / kStages) & 1) && clock64() - t0 < kWaitCycles) {
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            int g = 0;
            bool ok = true;
            long long tw[3] = {0, 0, 0};
            for (int t = 0, item = blockIdx.x; ok && item < a.items; ++t, item += gridDim.x) {
                long long c0 = clock64();
                if (!mbar_wait(a_full, t & 1, abort_flag, a.err, 3)) { ok = false; break; }
                tw[0] += clock64() - c0;
                int p_lo;
                const int nu = item_units(a, item, p_lo);
                for (int uix = 0; uix < nu; ++uix, ++g) {
                    const int s = g % kStages, acc = g & 1;
                    c0 = clock64();
                    if (!mbar_wait(&b_full[s], (g / kStages) & 1, abort_flag, a.err, 4)) { ok = false; break; }
                    const long long c1 = clock64();
                    tw[1] += c1 - c0;
                    if (!mbar_wait(&acc_empty[acc], ((g >> 1) & 1) ^ 1, abort_flag, a.err, 5)) { ok = false; break; }
                    tw[2] += clock64() - c1;
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kCols);
                    const uint32_t abase = su32(sm + P.a), bbase = su32(sm + P.b[s]);
                    for (int p = 0; p < panels; ++p)
                        mma_tf32(d_tmem, sw32_desc(abase + p * kRows * 32), sw32_desc(bbase + p * kCols * 32),
                                 p > 0 ? 1u : 0u);
                    mma_commit(&acc_full[acc]);
                }
            }
            if (a.counters) {
                atomicAdd(&a.counters[4 + kTMmaWaitA], (unsigned long long)tw[0]);
                atomicAdd(&a.counters[4 + kTMmaWaitB], (unsigned long long)tw[1]);
                atomicAdd(&a.counters[4 + kTMmaWaitAcc], (unsigned long long)tw[2]);
            }
        }
        __syncwarp();
    } else if (warp < 2 + kFilterWarps) {
        // ---------------------------------------------------------------- filter
        const int e = warp - 2;                 // 0..7
        const int quad = warp & 3;              // the TMEM lane quarter this warp may read
        const int half = e >> 2;                // column half of the tile
        const int ra = quad * 32 + lane;        // this thread's A row (tile-local)
        int g = 0;
        bool ok = true;
        long long tw[2] = {0, 0};
        unsigned long long inline_entries = 0;
        for (int t = 0, item = blockIdx.x; ok && item < a.items; ++t, item += gridDim.x) {
            if (!mbar_wait(a_full, t & 1, abort_flag, a.err, 6)) { ok = false; break; }
            const float Ui = reinterpret_cast<const float*>(sm + P.arow_u)[ra];
            int p_lo;
            const int nu = item_units(a, item, p_lo);
            for (int uix = 0; uix < nu; ++uix, ++g) {
                const int s = g % kStages, acc = g & 1, qi = g % kQueues;
                const long long c0 = clock64();
                if (!mbar_wait(&acc_full[acc], (g >> 1) & 1, abort_flag, a.err, 7)) { ok = false; break; }
                if (!mbar_wait(&q_free[qi], ((g / kQueues) & 1) ^ 1, abort_flag, a.err, 8)) { ok = false; break; }
                const long long c1 = clock64();
                tw[0] += c1 - c0;
                tc_fence_after();
                const Unit u = make_unit(a, item, p_lo + uix);
                const int gi = u.B * kRows + ra;
                const bool row_real = gi < a.n;
                const float* cu = reinterpret_cast<const float*>(sm + P.bcol_u[s]);
                int* qgi = qbase + qi * 4 * kQueueCap;
                int* qgj = qgi + kQueueCap;
                unsigned* qmr = reinterpret_cast<unsigned*>(qgj + kQueueCap);
                unsigned* qmc = qmr + kQueueCap;
                const int rblk = half ? u.R1 : u.R0;
                auto process = [&](const uint32_t (&rv)[32], int c) {
                    const int cb = half * 128 + c * 32;
                    // four independent partial masks keep the dependency chains short
                    unsigned mr[4] = {0, 0, 0, 0}, mc[4] = {0, 0, 0, 0};
#pragma unroll
                    for (int q = 0; q < 32; q += 4) {
                        const float4 u4 = *reinterpret_cast<const float4*>(cu + cb + q);
                        const float uc[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            const float v = __uint_as_float(rv[q + w]);
                            if (v <= Ui) mr[w] |= 1u << (q + w);
                            if (v <= uc[w]) mc[w] |= 1u << (q + w);
                        }
                    }
                    unsigned mrow = (mr[0] | mr[1]) | (mr[2] | mr[3]);
                    unsigned mcol = (mc[0] | mc[1]) | (mc[2] | mc[3]);
                    if (!row_real) mrow = 0;
                    if (!row_real || a.diag) mcol = 0;   // diagonal tiles: both orders appear as rows
                    if (!__any_sync(0xffffffffu, (mrow | mcol) != 0u)) return;
                    const int gj0 = rblk * kRows + c * 32;
                    if (!a.exact) {
                        // precision TF32: the accumulator is the distance, admit right here
                        const unsigned mm = mrow | mcol;
                        if (mm) {
#pragma unroll
                            for (int q = 0; q < 32; ++q) {
                                if (!((mm >> q) & 1u)) continue;
                                const int gj = gj0 + q;
                                if (gj == gi || gj >= a.n) continue;
                                const float d2 = fmaxf(__uint_as_float(rv[q]), 0.0f);
                                if ((mrow >> q) & 1u) {
                                    const uint64_t key = pack_key(d2, gj);
                                    if (key < __ldg(a.thr + gi)) tc_append(a, gi, key);
                                }
                                if ((mcol >> q) & 1u) {
                                    const uint64_t key = pack_key(d2, gi);
                                    if (key < __ldg(a.thr + gj)) tc_append(a, gj, key);
                                }
                            }
                        }
                    } else if (mrow | mcol) {
                        const int slot = atomicAdd(&qcount[qi], 1);
                        if (slot < kQueueCap) {
                            qgi[slot] = gi;
                            qgj[slot] = gj0;
                            qmr[slot] = mrow;
                            qmc[slot] = mcol;
                        } else {
                            // queue full (dense early rounds): refine in place
                            settle_exact(a, gi, gj0, mrow, mcol);
                            ++inline_entries;
                        }
                    }
                    __syncwarp();
                };
                if (rblk >= 0) {
                    // two chunks in flight: the TMEM load of chunk c + 1 overlaps the filter of chunk c
                    const uint32_t tbase =
                        tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * kCols + half * 128);
                    uint32_t r0[32], r1[32];
                    tmem_ld32(tbase, r0);
                    tmem_wait(r0);
                    tmem_ld32(tbase + 32, r1);
                    process(r0, 0);
                    tmem_wait(r1);
                    tmem_ld32(tbase + 64, r0);
                    process(r1, 1);
                    tmem_wait(r0);
                    tmem_ld32(tbase + 96, r1);
                    process(r0, 2);
                    tmem_wait(r1);
                    process(r1, 3);
                }
                // the accumulator and the B stage are done with: release both, hand the queue over
                // (the proxy fence orders this warp's reads of the stage before the next bulk copy)
                tc_fence_before();
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                tw[1] += clock64() - c1;
                if (lane == 0) {
                    mbar_arrive(&acc_empty[acc]);
                    mbar_arrive(&b_empty[s]);
                    mbar_arrive(&q_full[qi]);
                }
            }
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(a_empty);
        }
        if (a.counters) {
            if (inline_entries) atomicAdd(&a.counters[1], inline_entries);
            if (lane == 0) {
                atomicAdd(&a.counters[4 + kTFiltWait], (unsigned long long)tw[0]);
                atomicAdd(&a.counters[4 + kTFiltWork], (unsigned long long)tw[1]);
            }
        }
    } else {
        // ---------------------------------------------------------------- refine
        const int r = warp - 2 - kFilterWarps;   // 0 .. kRefineWarps - 1
        int g = 0;
        bool ok = true;
        long long tw[2] = {0, 0};
        unsigned long long entries = 0;
        for (int t = 0, item = blockIdx.x; ok && item < a.items; ++t, item += gridDim.x) {
            int p_lo;
            const int nu = item_units(a, item, p_lo);
            for (int uix = 0; uix < nu; ++uix, ++g) {
                if (g % kRefineWarps != r) continue;
                const int qi = g % kQueues;
                const long long c0 = clock64();
                if (!mbar_wait(&q_full[qi], (g / kQueues) & 1, abort_flag, a.err, 9)) { ok = false; break; }
                const long long c1 = clock64();
                tw[0] += c1 - c0;
                const int* qgi = qbase + qi * 4 * kQueueCap;
                const int* qgj = qgi + kQueueCap;
                const unsigned* qmr = reinterpret_cast<const unsigned*>(qgj + kQueueCap);
                const unsigned* qmc = qmr + kQueueCap;
                const int nq = min(qcount[qi], kQueueCap);
                entries += nq;
                for (int ei = lane; ei < nq; ei += 32) settle_exact(a, qgi[ei], qgj[ei], qmr[ei], qmc[ei]);
                __syncwarp();
                tw[1] += clock64() - c1;
                if (lane == 0) {
                    qcount[qi] = 0;
                    mbar_arrive(&q_free[qi]);
                }
                __syncwarp();
            }
        }
        if (a.counters && lane == 0) {
            atomicAdd(&a.counters[0], entries);
            atomicAdd(&a.counters[4 + kTRefWait], (unsigned long long)tw[0]);
            atomicAdd(&a.counters[4 + kTRefWork], (unsigned long long)tw[1]);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512) : "memory");
}

// ------------------------------------------------------------------ data preparation
__device__ __forceinline__ float rna_tf32(float x)
{
    // round the magnitude to 11 significant bits, ties away from zero
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

__device__ __forceinline__ void split3(float v, float& h, float& m, float& l)
{
    h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
    const float r = __fsub_rn(v, h);
    m = __uint_as_float(__float_as_uint(r) & 0xFFFFE000u);
    l = __fsub_rn(r, m);   // at most 2 significant bits remain: exact in TF32
}

// byte offset of element k of row i inside a blocked, pre-swizzled operand image: 128-row blocks
// of K/8 panels, each panel 128 rows x 32 bytes with the SWIZZLE_32B chunk order, so one contiguous
// bulk copy of a panel lands in shared memory exactly as the MMA descriptor expects it
__device__ __forceinline__ size_t image_offset(int i, int k, int kp)
{
    const int blk = i >> 7, r = i & 127, p = k >> 3, c = k & 7;
    const int phys = ((c >> 2) ^ ((r >> 2) & 1));
    return (size_t)blk * (kp / 8) * 4096 + (size_t)p * 4096 + (size_t)r * 32 + phys * 16 + (c & 3) * 4;
}

// One thread per row: TF32-rounded A / B operand rows, the original coordinates point-major (zero
// padded to dp), and poison for padding rows (their product with any real row is 2^100, above every
// finite bound).
__global__ void build_rows_kernel(const float* __restrict__ x, int ldx, int n, int d, int kp, int dp,
                                  int rows_a, int rows_b, unsigned char* __restrict__ A,
                                  unsigned char* __restrict__ Bm, float* __restrict__ xp)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows_b) return;
    const bool has_a = i < rows_a;
    float* xr = xp + (size_t)i * dp;
    auto put = [&](unsigned char* img, int k, float v) { *reinterpret_cast<float*>(img + image_offset(i, k, kp)) = v; };
    if (i >= n) {
        for (int k = 0; k < kp; ++k) {
            if (has_a) put(A, k, (k == d + 3) ? kPoisonNorm : 0.0f);
            put(Bm, k, (k == d) ? kPoisonNorm : 0.0f);
        }
        for (int k = 0; k < dp; ++k) xr[k] = 0.0f;
        return;
    }
    float nt = 0.0f;
    for (int k = 0; k < d; ++k) {
        const float xv = x[(size_t)k * ldx + i];
        const float xt = rna_tf32(xv);
        nt = __fmaf_rn(xt, xt, nt);
        if (has_a) put(A, k, __fmul_rn(-2.0f, xt));
        put(Bm, k, xt);
        xr[k] = xv;
    }
    for (int k = d; k < dp; ++k) xr[k] = 0.0f;
    float h, m, l;
    split3(nt, h, m, l);
    const float av[6] = {1.0f, 1.0f, 1.0f, h, m, l};
    const float bv[6] = {h, m, l, 1.0f, 1.0f, 1.0f};
    for (int k = d; k < kp; ++k) {
        const int o = k - d;
        if (has_a) put(A, k, (o < 6) ? av[o] : 0.0f);
        put(Bm, k, (o < 6) ? bv[o] : 0.0f);
    }
}

}  // namespace tc

// ------------------------------------------------------------------ host side
namespace {

struct TcState {
    int n = 0, d = 0, kp = 0, dp = 0, npad = 0, sms = 0;
    unsigned char *A = nullptr, *B = nullptr;
    float* xp = nullptr;
    float *U = nullptr, *nrm = nullptr;   // U / nrm / thr belong to the scheduler
    uint64_t* thr = nullptr;
};

TcState g_state;   // the prepared operands of the current kNN call (one per process)

}  // namespace

bool tc_engine_supported(int d)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) return false;
    const int kp = tc_kp(d);
    return p.major == 10 && p.minor == 0 && kp <= tc::kMaxKp && tc::smem_plan(kp).total + 1024 <= 227 * 1024;
}

// Prepares the TF32 operand images and the point-major original coordinates for one kNN call; the
// per-point bounds, norms and thresholds (Npad + 128 entries each) belong to the scheduler.
void tc_prepare(Workspace& ws, const float* x, int ldx, int n, int d, const float* norms, const float* U,
                const uint64_t* thr, cudaStream_t s)
{
    TcState& st = g_state;
    const int kp = tc_kp(d);
    const int dp = ((d + 3) / 4) * 4;
    const int T = (n + kBlock - 1) / kBlock;
    const int npad = T * kBlock;
    const int rows_b = npad + kBlock;     // + one poison block
    const size_t a_bytes = sizeof(float) * (size_t)npad * kp;
    const size_t b_bytes = sizeof(float) * (size_t)rows_b * kp;
    const size_t x_bytes = sizeof(float) * (size_t)rows_b * dp;
    char* mem = (char*)ws.ops.ensure(a_bytes + b_bytes + x_bytes + 3072);
    auto align = [](char* p) { return (char*)(((uintptr_t)p + 1023) & ~(uintptr_t)1023); };
    st.A = (unsigned char*)align(mem);
    st.B = (unsigned char*)align((char*)st.A + a_bytes);
    st.xp = (float*)align((char*)st.B + b_bytes);
    // the images have no gaps: every element is written by the build kernel
    tc::build_rows_kernel<<<(rows_b + 127) / 128, 128, 0, s>>>(x, ldx, n, d, kp, dp, npad, rows_b, st.A, st.B,
                                                               st.xp);
    FDB_LAUNCHED();
    int dev = 0;
    FDB_CUDA(cudaGetDevice(&dev));
    FDB_CUDA(cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, dev));
    st.n = n;
    st.d = d;
    st.kp = kp;
    st.dp = dp;
    st.npad = npad;
    st.U = const_cast<float*>(U);
    st.nrm = const_cast<float*>(norms);
    st.thr = const_cast<uint64_t*>(thr);
}

void launch_tile_round_tc(const TileRound& r, int units, int precision, cudaStream_t s)
{
    (void)units;
    TcState& st = g_state;
    tc::Args a{};
    a.n = r.n;
    a.d = r.d;
    a.kp = st.kp;
    a.dp = st.dp;
    a.T = r.T;
    a.b_lo = r.b_lo;
    a.nb = r.nb;
    a.cap = r.cap;
    a.exact = precision == FDB200_FP32 ? 1 : 0;
    a.diag = r.diag;
    a.delta0 = r.delta0;
    a.ndelta = r.ndelta;
    a.row_pad = st.npad;
    a.U = st.U;
    a.nrm = st.nrm;
    a.thr = st.thr;
    a.xp = st.xp;
    a.aimg = st.A;
    a.bimg = st.B;
    a.cand = r.cand;
    a.cnt = r.cnt;
    a.ovf = r.ovf;
    a.err = r.ovf + 1;
    a.counters = r.counters;
    if (r.diag) {
        a.npairs = 1;
        a.pairs_per_item = 1;
        a.items = r.nb;
    } else {
        a.npairs = (r.ndelta + 1) / 2;
        // about 8 items per CTA so the tail of a round stays short
        const long long want_items = 8ll * st.sms;
        int ppi = (int)std::max<long long>(1, ((long long)a.npairs * r.nb + want_items - 1) / want_items);
        ppi = std::min(ppi, a.npairs);
        a.pairs_per_item = ppi;
        a.items = r.nb * ((a.npairs + ppi - 1) / ppi);
    }
    if (a.items <= 0) return;
    const tc::Smem P = tc::smem_plan(st.kp);
    const size_t smem = P.total + 1024;
    static bool attr_set = false;
    if (!attr_set) {
        FDB_CUDA(cudaFuncSetAttribute(tc::knn_tile_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        attr_set = true;
    }
    const int grid = std::min(a.items, st.sms);
    tc::knn_tile_tc<<<grid, tc::kThreads, smem, s>>>(a);
    FDB_LAUNCHED();
}

}  // namespace fdb
