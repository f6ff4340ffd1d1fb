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
    const float* U;          // per-point folded filter bound V (tcgen05 engine)
    uint64_t* cand;          // n * cap candidate slots
    int* cnt;                // per-point slot counters
    int cap;
    int* ovf;                // [0]: tag of the round in which a counter passed cap; [1]: tcgen05 error
    int tag;                 // this round's tag (its index in the host's batch of rounds + 1)
    int T;                   // blocks in the triangle
    int b_lo, nb;            // this shard's row blocks
    int diag;                // 1: diagonal units (B, B), row side only
    int rows_only;           // SIMT tiles: 1 = each unit updates its row block only, and the round covers
                             // the offsets in both directions (a shard's rows get every candidate
                             // without updating other shards' points); 0 = symmetric units
    int delta0;              // first block offset of the round
    int ndelta;              // block offsets in the round
    int sym;                 // tcgen05 engine: 1 = each unordered block pair once, both sides tested
                             // (unfolded operands, U strict); 0 = ordered pairs, rows only (folded)
    unsigned long long* counters;   // optional tcgen05 diagnostics (FDB200_TRACE=1), else null
};

__device__ __forceinline__ bool decode_unit(const TileRound& r, int u, int& B, int& R)
{
    if (r.diag) {
        B = r.b_lo + u;
        R = B;
        return true;
    }
    if (r.rows_only) {
        // units [0, nb * ndelta): R = B + delta; [nb * ndelta, 2 nb * ndelta): R = B - delta; with an
        // even block count the offset T/2 reaches the same block both ways, so its second copy goes
        const int per = r.nb * r.ndelta;
        const int back = u >= per ? 1 : 0;
        const int v = u - back * per;
        const int dl = r.delta0 + v / r.nb;
        B = r.b_lo + v % r.nb;
        if (back && (r.T & 1) == 0 && dl == r.T / 2) return false;
        R = back ? B - dl : B + dl;
        if (R >= r.T) R -= r.T;
        if (R < 0) R += r.T;
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
    else atomicExch(r.ovf, r.tag);
}

// K of the tcgen05 operand rows: D coordinates + 3 norm columns + 3 ones, padded to 8
__host__ __device__ inline int tc_kp(int d) { return ((d + 6 + 7) / 8) * 8; }

// Filter bound of point i for the tcgen05 engine. The MMA sees x~ = x rounded to TF32 (nearest,
// relative error <= 2^-11 per coordinate) and the norms of x~ split into three TF32-exact parts,
// so acc(i, j) = |x~_i - x~_j|^2 up to FP32 accumulation. With r = |x_i - x_j| (real):
//   |x~_i - x~_j| <= r + eps (|x_i| + |x_j|)                                  (triangle inequality)
//   acc <= r^2 + 2 r eps (a + b) + eps^2 (a + b)^2 + acc_err + norm_err
//   d2_ref >= r^2 - e_ref       (the reference's own FP32 rounding of n_i + n_j - 2 dot)
// A candidate that can enter the list has d2_ref <= T, hence r <= R = sqrt(T + e_ref) and
// b = |x_j| <= a + R, so acc <= U_i = T + E(a, R) for every such candidate: the filter never drops
// one. acc_err allows 2^-20 of the summed term magnitudes per K-step of 8 (four times the FP32
// truncation error of one tensor-core K-step), norm_err the fmaf-chain norm of x~.
__device__ __forceinline__ float filter_bound(float T, float ni, int d, int kp, int exact)
{
    if (!exact) return T;
    if (isinf(T)) return T;
    const double n = (double)ni, t = (double)T;
    const double a = sqrt(n) * (1.0 + 1e-6);
    const double eps = 0x1p-11 * (1.0 + 0x1p-10);
    const double c_ref = (2.0 * d + 8.0) * 0x1p-24;
    const double c_acc = (double)(kp / 8) * 0x1p-20;
    const double c_nrm = (d + 2.0) * 0x1p-24;
    double R = sqrt(t), b = a + R;
    for (int it = 0; it < 2; ++it) {
        const double e_ref = c_ref * (n + b * b);
        R = sqrt(t + e_ref) * (1.0 + 1e-6);
        b = a + R;
    }
    const double nt_i = n * (1.0 + 0x1p-9), nt_j = b * b * (1.0 + 0x1p-9);   // norms of x~
    const double E = c_ref * (n + b * b) + 2.0 * R * eps * (a + b) + eps * eps * (a + b) * (a + b) +
                     c_acc * 2.0 * (nt_i + nt_j) + c_nrm * (nt_i + nt_j);
    return __double2float_ru(t + E);
}

// byte offset of element k of row i inside a blocked, pre-swizzled tcgen05 operand image: 128-row
// blocks of K/8 panels, each panel 128 rows x 32 bytes with the SWIZZLE_32B chunk order, so one
// contiguous bulk copy of a panel lands in shared memory exactly as the MMA descriptor expects it
__host__ __device__ __forceinline__ size_t image_offset(int i, int k, int kp)
{
    const int blk = i >> 7, r = i & 127, p = k >> 3, c = k & 7;
    const int phys = ((c >> 2) ^ ((r >> 2) & 1));
    return (size_t)blk * (kp / 8) * 4096 + (size_t)p * 4096 + (size_t)r * 32 + phys * 16 + (c & 3) * 4;
}

// v = h + m + l exactly, each part exact in TF32 (11 significant bits, then 11, then at most 2)
__device__ __forceinline__ void split3(float v, float& h, float& m, float& l)
{
    h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
    const float r = __fsub_rn(v, h);
    m = __uint_as_float(__float_as_uint(r) & 0xFFFFE000u);
    l = __fsub_rn(r, m);
}

// The tcgen05 engine folds point i's filter bound into its A operand row: the three "norm of i"
// entries hold w_i = n~_i - V_i instead, so the MMA yields acc'(i, j) = |x~_i - x~_j|^2 - V_i and a
// candidate survives iff acc' is negative (its sign bit). With U = filter_bound(T) covering the
// accumulation error of the plain sum, the extra term w_i adds at most c_acc |w_i| <= c_acc (n~ + V)
// of error; V also adds 2^-100 so that a survivor's acc' is strictly below zero. Infinite bounds
// (empty lists) become w = -2^120: everything survives. Precision TF32 folds the plain threshold.
constexpr float kFoldAll = -1.329227995784916e36f;   // -2^120, exact in TF32

__device__ __forceinline__ void fold_bound(float U, float nt, int kp, int exact, float& V, float& w)
{
    if (!(U < __int_as_float(0x7f800000))) {
        V = __int_as_float(0x7f800000);
        w = kFoldAll;
        return;
    }
    if (!exact) {
        V = U;
        w = __fsub_rn(nt, U);
        return;
    }
    const float c_acc = (float)(kp / 8) * 0x1p-20f * 1.01f;
    V = __fadd_ru(U, __fmul_ru(c_acc, __fadd_ru(nt, U)));
    V = __fadd_ru(V, 0x1p-100f);
    w = __fsub_rd(nt, V);
}

// The symmetric schedule leaves the operands unfolded, so acc(i, j) = |x~_i - x~_j|^2 up to FP32
// accumulation, and tests each unordered pair for both endpoints at once: the pair survives iff
// acc < max(U_i, U_j), with U the filter bound made strict (its next float up, so that acc <= bound
// is acc < U). One rounded subtraction acc - max(U_i, U_j) has the sign of the exact difference
// (a negative difference never rounds to +0), so the sign bit is the survivor bit as in the folded
// form. Infinite bounds stay infinite (everything survives).
__device__ __forceinline__ float strict_bound(float U)
{
    if (!(U < __int_as_float(0x7f800000))) return __int_as_float(0x7f800000);
    return __uint_as_float(__float_as_uint(U) + 1u);   // U >= 0
}

// writes w's three TF32 parts into row i of the A operand image (columns d + 3 .. d + 5)
__device__ __forceinline__ void store_fold(unsigned char* aimg, int i, int d, int kp, float w)
{
    float h, m, l;
    split3(w, h, m, l);
    *reinterpret_cast<float*>(aimg + image_offset(i, d + 3, kp)) = h;
    *reinterpret_cast<float*>(aimg + image_offset(i, d + 4, kp)) = m;
    *reinterpret_cast<float*>(aimg + image_offset(i, d + 5, kp)) = l;
}

void launch_tile_round_simt(const TileRound& r, int units, cudaStream_t s);
void launch_tile_round_tc(const TileRound& r, int units, int precision, cudaStream_t s);

}  // namespace fdb
