// knn_tc_schedule.h -- the tcgen05 engine's tile schedule: which tiles a round's launch covers, how
// they group into work items, and how an item maps to its tiles. Device code (every role of the tile
// kernel walks it) and host code (the launcher, and a host test that checks coverage) share it.
//
// A round covers the block offsets [delta0, delta0 + ndelta) of T blocks of 128 points. A tile is one
// row block X against two adjacent column blocks (Y, Y + 1) = (X + delta, X + delta + 1) (mod T); a work
// item keeps (Y, Y + 1) and walks up to ppi such offset pairs, i.e. the row blocks X = Y - delta.
//   symmetric: forward offsets only, so each unordered block pair is covered once (by the shard that
//     owns its first block, X); with an even T the offset T/2 reaches {X, X + T/2} from both blocks,
//     and only X < T/2 keeps it.
//   ordered (a shard of row blocks [b_lo, b_lo + nb)): the offsets and their mirrors T - delta, so each
//     ordered pair of a shard row block is covered once; T/2 once.
//   diagonal round: item b is the tile (b_lo + b, b_lo + b), column half 0 only.
#pragma once

#if defined(__CUDACC__)
#define FDB_SCHED_HD __host__ __device__ __forceinline__
#else
#define FDB_SCHED_HD inline
#endif

namespace fdb {
namespace tc {

// Offset pairs (tiles) per work item, at most: the items in flight, claimed in order, then stream a
// window of about 148 + 2 * 256 row blocks (19 MB at d = 50) that L2 holds, where whole-range items made
// the 148 CTAs drift apart over the row blocks (101 GB of DRAM reads in the largest round of the
// headline fit). Each item reloads its column pair, and the tensor pipe idles while it lands (no room
// for a second column stage), so items are not made shorter: 64 pairs cost 5 % in that round.
constexpr int kMaxItemPairs = 256;

struct Sched {
    int T;                       // blocks in the triangle
    int diag;                    // 1: the diagonal round (X against X)
    int sym;                     // 1: symmetric schedule (forward offsets only, both endpoints tested)
    int b_lo, nb;                // row blocks of this shard
    int r0[2], len[2], np[2];    // forward / backward offset ranges: first offset, length, pairs
    int ppi, nchunk0, items;     // pairs per work item, items of the forward range, all items
    int ywin;                    // column blocks per offset chunk: T, or the window a shard's rows reach
};

struct Tile {
    int X, Y;     // row block, first column block
    int h0, h1;   // whether column block Y (Y + 1) belongs to the round
};

FDB_SCHED_HD int sched_min(int a, int b) { return a < b ? a : b; }

// the schedule of one launch (host side): round offsets [delta0, delta0 + ndelta), or the diagonal
// round, over the row blocks [b_lo, b_lo + nb), with about 8 items per CTA on `ctas` CTAs
inline void plan_schedule(Sched& a, int T, int diag, int sym, int b_lo, int nb, int delta0, int ndelta, int ctas)
{
    a.T = T;
    a.diag = diag;
    a.sym = sym;
    a.b_lo = b_lo;
    a.nb = nb;
    a.r0[0] = a.r0[1] = a.len[0] = a.len[1] = a.np[0] = a.np[1] = 0;
    a.nchunk0 = 0;
    a.ywin = T;
    if (diag) {
        a.items = nb;
        a.ppi = 1;
        return;
    }
    const long long want_items = 8ll * ctas;
    long long pairs;
    if (sym) {
        // forward offsets [d0, d0 + L) only: the tile of rows X and columns X + delta tests both
        a.r0[0] = delta0;
        a.len[0] = ndelta;
        a.np[0] = (ndelta + 1) / 2;
        pairs = (long long)nb * a.np[0];
    } else {
        // forward offsets [d0, d0 + L) and their mirrors T - delta, the offset T/2 only once
        const int e = ((T & 1) == 0 && delta0 + ndelta - 1 == T / 2) ? 1 : 0;
        a.r0[0] = delta0;
        a.len[0] = ndelta;
        a.r0[1] = T - (delta0 + ndelta - 1) + e;
        a.len[1] = ndelta - e;
        a.np[0] = (a.len[0] + 1) / 2;
        a.np[1] = (a.len[1] + 1) / 2;
        pairs = (long long)nb * (a.np[0] + a.np[1]);
    }
    // about 8 items of real tiles per CTA so the tail of a round stays short, kMaxItemPairs at most
    long long ppi = (pairs + want_items - 1) / want_items;
    if (ppi < 1) ppi = 1;
    if (ppi > kMaxItemPairs) ppi = kMaxItemPairs;
    a.ppi = sched_min((int)ppi, a.np[0] > 1 ? a.np[0] : 1);
    a.nchunk0 = (a.np[0] + a.ppi - 1) / a.ppi;
    // a shard's rows X in [b_lo, b_lo + nb) meet, for one chunk of ppi offset pairs, the column blocks
    // Y = X + delta: a window of nb + 2 ppi - 1 blocks (all T when unsharded)
    a.ywin = (nb == T) ? T : sched_min(T, nb + 2 * a.ppi - 1);
    a.items = a.ywin * (a.nchunk0 + (sym ? 0 : (a.np[1] + a.ppi - 1) / a.ppi));
}

// Work item -> (offset range rho, resident column block Y, its pair indices [p_lo, p_lo + count)).
// Every role walks the same items and tiles in the same order, so tile counters agree.
FDB_SCHED_HD int item_span(const Sched& a, int item, int& rho, int& Y, int& p_lo)
{
    if (a.diag) {
        rho = 0;
        Y = a.b_lo + item;
        p_lo = 0;
        return 1;
    }
    const int gc = item / a.ywin;
    const int w = item - gc * a.ywin;
    rho = gc < a.nchunk0 ? 0 : 1;
    p_lo = (rho ? gc - a.nchunk0 : gc) * a.ppi;
    if (a.ywin == a.T) {
        Y = w;
    } else {
        // a shard: only the column blocks Y whose rows X = Y - delta (delta = r0 + 2p over the chunk)
        // can fall in the shard's row blocks
        Y = a.b_lo + a.r0[rho] + 2 * p_lo + w;
        Y %= a.T;
    }
    return sched_min(a.np[rho], p_lo + a.ppi) - p_lo;
}

// pair p of an item covers the offsets (delta, delta + 1) = r0 + 2p (+1): rows X = Y - delta;
// false when X lies outside this shard's row blocks. Under the symmetric schedule an even block
// count reaches the pair {X, X + T/2} from both of its blocks: only X < T/2 keeps it.
FDB_SCHED_HD bool tile_of(const Sched& a, int rho, int Y, int p, Tile& t)
{
    t.Y = Y;
    if (a.diag) {
        t.X = Y;
        t.h0 = 1;
        t.h1 = 0;
        return true;
    }
    const int off = 2 * p;
    const int dl = a.r0[rho] + off;
    int X = Y - dl;
    if (X < 0) X += a.T;
    t.X = X;
    t.h0 = 1;
    t.h1 = (off + 1 < a.len[rho]) ? 1 : 0;
    if (a.sym && (a.T & 1) == 0 && X >= (a.T >> 1)) {
        if (dl == (a.T >> 1)) t.h0 = 0;
        if (dl + 1 == (a.T >> 1)) t.h1 = 0;
    }
    return (unsigned)(X - a.b_lo) < (unsigned)a.nb && (t.h0 | t.h1);
}

// how many of an item's nu pairs tile_of accepts: all of them unsharded, except under the symmetric
// schedule the one pair whose first offset is T/2 when its row block is X >= T/2; a shard counts
FDB_SCHED_HD int item_tiles(const Sched& a, int rho, int Y, int p_lo, int nu)
{
    if (a.nb == a.T) {
        if (!a.sym || a.diag || (a.T & 1)) return nu;
        const int hT = a.T >> 1, off = hT - a.r0[rho];
        if (off < 0 || (off & 1) || (off >> 1) < p_lo || (off >> 1) >= p_lo + nu) return nu;
        const int X = Y >= hT ? Y - hT : Y + hT;
        return X >= hT ? nu - 1 : nu;
    }
    int c = 0;
    for (int u = 0; u < nu; ++u) {
        Tile t;
        c += tile_of(a, rho, Y, p_lo + u, t) ? 1 : 0;
    }
    return c;
}

}  // namespace tc
}  // namespace fdb
