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
    uint64_t* cand;          // n * cap candidate slots
    int* cnt;                // per-point slot counters
    int cap;
    int* ovf;                // set when any counter passes cap
    int T;                   // blocks in the triangle
    int b_lo, nb;            // this shard's row blocks
    int diag;                // 1: diagonal units (B, B), row side only
    int delta0;              // first block offset of the round
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

__device__ __forceinline__ void append_keys(const TileRound& r, int p, const uint64_t* keys, int count)
{
    const int base = atomicAdd(&r.cnt[p], count);
    for (int t = 0; t < count; ++t) {
        const int slot = base + t;
        if (slot < r.cap) r.cand[(size_t)p * r.cap + slot] = keys[t];
        else atomicOr(r.ovf, 1);
    }
}

void launch_tile_round_simt(const TileRound& r, int units, cudaStream_t s);
void launch_tile_round_tc(const TileRound& r, int units, int precision, cudaStream_t s);

}  // namespace fdb
