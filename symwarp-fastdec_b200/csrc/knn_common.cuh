// knn_common.cuh -- the per-round tile contract shared by the SIMT and tcgen05 distance engines.
#pragma once

#include "fdb_internal.h"

namespace fdb {

__device__ __forceinline__ uint64_t pack_key(float d2, int idx)
{
    return ((uint64_t)__float_as_uint(d2) << 32) | (uint32_t)idx;
}

// symtriknnfds.h:23-26 -- two separately rounded adds, then clamp at zero
__device__ __forceinline__ float exact_d2(float na, float nb, float dot)
{
    return fmaxf(__fadd_rn(__fadd_rn(na, nb), __fmul_rn(-2.0f, dot)), 0.0f);
}

// ------------------------------------------------------------------ one round of tiles
struct TileRound {
    const float* x;
    int ldx, n, d;
    const float* norms;
    const uint64_t* thr;     // per-point admission bound: a key is admitted iff key < thr
    const float* U;          // per-point TF32 filter bound (tcgen05 engine)
    uint64_t* cand;          // n * cap candidate slots
    int* cnt;                // per-point slot counters
    int cap;
    int* ovf;                // set when any counter passes cap
    int T;                   // blocks in the triangle
    int b_lo, nb;            // this shard's row blocks
    int diag;                // 1: diagonal units (B, B), row side only
    int delta0;              // first block offset of the round
    int ndelta;              // block offsets in the round
};

__device__ __forceinline__ bool decode_unit(const TileRound& r, int u, int& B, int& R)
{
    if (r.diag) {
        B = r.b_lo + u;
        R = B;
        return true;
    }
    const int dl = r.delta0 + u / r.nb;
    B = r.b_lo + u % r.nb;
    // with an even block count the offset T/2 pairs every block twice; keep one copy
    if ((r.T & 1) == 0 && dl == r.T / 2 && B >= r.T / 2) return false;
    R = B + dl;
    if (R >= r.T) R -= r.T;
    return true;
}

__device__ __forceinline__ void append_at(const TileRound& r, int p, int slot, uint64_t key)
{
    if (slot < r.cap) r.cand[(size_t)p * r.cap + slot] = key;
    else atomicOr(r.ovf, 1);
}

__device__ __forceinline__ void append_keys(const TileRound& r, int p, const uint64_t* keys, int count)
{
    const int base = atomicAdd(&r.cnt[p], count);
    for (int t = 0; t < count; ++t) {
        const int slot = base + t;
        if (slot < r.cap) r.cand[(size_t)p * r.cap + slot] = keys[t];
        else atomicOr(r.ovf, 1);
    }
}

// Largest possible |acc - d2_ref| for a candidate that can enter point i's list, where acc is the
// tcgen05 TF32 value of the augmented product (knn_tc.cu) and d2_ref the reference's FP32 d2:
//   |acc - d2_ref| <= c1 |x_i||x_j| + c2 (n_i + n_j)
//     c1: TF32 rounding of both coordinates (<= 2^-10 relative each), times the factor 2
//     c2: FP32 accumulation of kp terms (generously 2^-21 each), the split norm's low part, and
//         the reference's own rounding of the norms and of d2
// and for an admissible candidate (d2_ref <= T) |x_j| <= |x_i| + sqrt(T + slack).
__device__ __forceinline__ float filter_bound(float T, float ni, int d, int kp, int exact)
{
    if (!exact) return T;
    if (isinf(T)) return T;
    const double n = (double)ni, t = (double)T;
    const double a = sqrt(n) * (1.0 + 1e-6);
    const double R = sqrt(t + 0x1p-10 * (n + t)) * (1.0 + 1e-6);
    const double b = a + R;
    const double c1 = 0x1p-8 * 1.01;
    const double c2 = 2.5 * kp * 0x1p-21 + (2.0 * d + 8.0) * 0x1p-24 + 0x1p-19;
    const double E = c1 * a * b + c2 * (n + b * b);
    return __double2float_ru(t + E);
}

void launch_tile_round_simt(const TileRound& r, int units, cudaStream_t s);
void launch_tile_round_tc(const TileRound& r, int units, int precision, cudaStream_t s);

}  // namespace fdb
