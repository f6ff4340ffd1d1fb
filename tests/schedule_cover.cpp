// Host check of the tcgen05 tile schedule (symwarp-fastdec_b200/csrc/knn_tc_schedule.h), built and run
// by tests/test_schedule.py. For many block counts T, round partitions of the offsets, shard splits
// and CTA counts it walks every work item and tile of every round exactly as the kernel's roles do and
// checks:
//   * the symmetric schedule (whole triangle): every unordered pair of distinct blocks is covered by
//     exactly one tile column half over all rounds, and the diagonal round covers each block once;
//   * the ordered schedule of a shard: every ordered pair (X, Y) with X in the shard's row blocks is
//     covered exactly once (X = Y by the diagonal round), and no other row block is ever covered;
//   * the symmetric schedule split over 2, 3 or 8 shards: the shards' tiles together cover every
//     unordered pair exactly once, and each shard's tiles have their row block in the shard;
//   * item_tiles (the MMA issuer's count) equals the number of pairs tile_of accepts in every item;
//   * every tile's row block lies in the shard and its column blocks in [0, T).
// Prints "ok <cases>" or the first failure, and exits non-zero on a failure.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "knn_tc_schedule.h"

using fdb::tc::Sched;
using fdb::tc::Tile;

static int fail(const char* what, int T, int b_lo, int nb, int sym, int ctas, int a = -1, int b = -1)
{
    std::printf("FAIL %s: T=%d shard=[%d,%d) sym=%d ctas=%d (%d, %d)\n", what, T, b_lo, b_lo + nb, sym, ctas, a, b);
    return 1;
}

// walks one launch; cov[X * T + Y] counts the (row block, column block) pairs covered
static int walk(const Sched& s, std::vector<int>& cov, int ctas)
{
    const int T = s.T;
    for (int item = 0; item < s.items; ++item) {
        int rho, Y, p_lo;
        const int nu = fdb::tc::item_span(s, item, rho, Y, p_lo);
        if (nu < 1 || Y < 0 || Y >= T) return fail("item span", T, s.b_lo, s.nb, s.sym, ctas, item, Y);
        int accepted = 0;
        for (int u = 0; u < nu; ++u) {
            Tile t;
            if (!fdb::tc::tile_of(s, rho, Y, p_lo + u, t)) continue;
            ++accepted;
            if (t.X < s.b_lo || t.X >= s.b_lo + s.nb) return fail("row outside shard", T, s.b_lo, s.nb, s.sym, ctas, t.X, t.Y);
            if (t.h0) ++cov[(size_t)t.X * T + t.Y];
            if (t.h1) ++cov[(size_t)t.X * T + (t.Y + 1) % T];
        }
        if (fdb::tc::item_tiles(s, rho, Y, p_lo, nu) != accepted)
            return fail("item_tiles != accepted tiles", T, s.b_lo, s.nb, s.sym, ctas, item, accepted);
    }
    return 0;
}

// the offsets 1 .. T/2 cut into consecutive rounds (delta0, ndelta), as the planner cuts them
static std::vector<std::pair<int, int>> partition(int T, std::mt19937& rng)
{
    std::vector<std::pair<int, int>> r;
    const int dmax = T / 2;
    int d0 = 1;
    while (d0 <= dmax) {
        std::uniform_int_distribution<int> len(1, std::max(1, std::min(dmax - d0 + 1, 1 + (int)(rng() % 600))));
        const int L = std::min(len(rng), dmax - d0 + 1);
        r.push_back({d0, L});
        d0 += L;
    }
    return r;
}

// one shard's fit: the diagonal round, then the rounds of the partition, into cov
static int cover(int T, int b_lo, int nb, int sym, int ctas, const std::vector<std::pair<int, int>>& rounds,
                 std::vector<int>& cov)
{
    Sched s;
    fdb::tc::plan_schedule(s, T, 1, sym, b_lo, nb, 0, 0, ctas);
    if (walk(s, cov, ctas)) return 1;
    for (const auto& r : rounds) {
        fdb::tc::plan_schedule(s, T, 0, sym, b_lo, nb, r.first, r.second, ctas);
        if (walk(s, cov, ctas)) return 1;
    }
    return 0;
}

// symmetric coverage: (X, Y) and (Y, X) together once, the diagonal once
static int check_unordered(const std::vector<int>& cov, int T, int world, int ctas)
{
    for (int X = 0; X < T; ++X)
        for (int Y = X; Y < T; ++Y) {
            const int both = X == Y ? cov[(size_t)X * T + X] : cov[(size_t)X * T + Y] + cov[(size_t)Y * T + X];
            if (both != 1) return fail("symmetric coverage", T, 0, T, 1, ctas, X, Y + 1000000 * world);
        }
    return 0;
}

// the symmetric schedule split over `world` shards of even block ranges
static int sym_shards(int T, int world, int ctas, std::mt19937& rng)
{
    std::vector<int> cov((size_t)T * T, 0);
    const auto rounds = partition(T, rng);
    for (int rank = 0; rank < world; ++rank) {
        const int lo = (int)((long)T * rank / world), hi = (int)((long)T * (rank + 1) / world);
        if (hi > lo && cover(T, lo, hi - lo, 1, ctas, rounds, cov)) return 1;
    }
    return check_unordered(cov, T, world, ctas);
}

// one fit of one shard (the whole triangle when nb == T)
static int fit(int T, int b_lo, int nb, int sym, int ctas, std::mt19937& rng)
{
    std::vector<int> cov((size_t)T * T, 0);
    if (cover(T, b_lo, nb, sym, ctas, partition(T, rng), cov)) return 1;
    for (int X = 0; X < T; ++X)
        for (int Y = 0; Y < T; ++Y) {
            const int c = cov[(size_t)X * T + Y];
            if (sym) {
                // unordered coverage: (X, Y) and (Y, X) together once; the diagonal once
                const int both = X == Y ? c : c + cov[(size_t)Y * T + X];
                if (both != 1) return fail("symmetric coverage", T, b_lo, nb, sym, ctas, X, Y);
            } else {
                const bool own = X >= b_lo && X < b_lo + nb;
                if (c != (own ? 1 : 0)) return fail("ordered coverage", T, b_lo, nb, sym, ctas, X, Y);
            }
        }
    return 0;
}

int main()
{
    std::mt19937 rng(12345);
    long cases = 0;
    const int ctas_list[] = {1, 3, 148};
    std::vector<int> Ts;
    for (int T = 1; T <= 70; ++T) Ts.push_back(T);
    for (int T : {127, 128, 255, 256, 513, 1000, 1563, 2048}) Ts.push_back(T);
    for (int T : Ts)
        for (int ctas : ctas_list) {
            const int reps = T <= 70 ? 3 : 1;
            for (int r = 0; r < reps; ++r) {
                // the whole triangle under the symmetric schedule
                if (fit(T, 0, T, 1, ctas, rng)) return 1;
                ++cases;
                // the whole triangle and 2-8 shards under the ordered schedule
                if (fit(T, 0, T, 0, ctas, rng)) return 1;
                ++cases;
                for (int world : {2, 3, 8}) {
                    if (world > T) continue;
                    if (sym_shards(T, world, ctas, rng)) return 1;
                    ++cases;
                    for (int rank = 0; rank < world; ++rank) {
                        const int lo = (int)((long)T * rank / world), hi = (int)((long)T * (rank + 1) / world);
                        if (hi > lo && fit(T, lo, hi - lo, 0, ctas, rng)) return 1;
                        ++cases;
                    }
                }
            }
        }
    std::printf("ok %ld\n", cases);
    return 0;
}
