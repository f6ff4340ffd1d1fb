"""The symmetric shards' threshold protocol, simulated on the host: each rank owns the block pairs whose
first block is its own, admits a candidate for a point only if its packed (d2, index) key is below the
point's threshold as combined at the start of the round, keeps the k smallest admitted keys per point,
and after every round the ranks' thresholds (the k-th key of each rank's partial list, or the empty key)
combine by unsigned MIN; at the end the partial lists merge. The result must be exactly the k smallest
keys of every point, whatever the number of ranks and the cut of the offsets into rounds: a threshold
combined this way is never below the true k-th key, so no true neighbour is ever refused. (The library
runs this protocol with its tiles and the round hook; this checks the protocol itself.)"""
import numpy as np
import pytest

EMPTY = np.uint64(0xFFFFFFFFFFFFFFFF)


def keys_of(x):
    """packed (float32 d2 bits << 32 | index) keys of every ordered pair, n x n; the diagonal empty"""
    d2 = ((x[:, None, :] - x[None, :, :]) ** 2).sum(-1).astype(np.float32)
    idx = np.arange(x.shape[0], dtype=np.uint64)
    keys = (d2.view(np.uint32).astype(np.uint64) << np.uint64(32)) | idx[None, :]
    np.fill_diagonal(keys, EMPTY)
    return keys


def simulate(x, k, world, block, rounds, rng):
    n = x.shape[0]
    keys = keys_of(x)
    T = (n + block - 1) // block
    blk = np.arange(n) // block
    owner_of_block = np.minimum(np.arange(T) * world // T, world - 1)
    lists = np.full((world, n, k), EMPTY, dtype=np.uint64)
    thr = np.full(n, EMPTY, dtype=np.uint64)          # combined, as every rank sees it
    # the offsets of the round plan: delta = 0 (the diagonal blocks) then 1 .. T // 2 in `rounds` cuts
    deltas = list(range(1, T // 2 + 1))
    cuts = sorted(rng.choice(np.arange(1, len(deltas)), size=min(rounds - 1, max(len(deltas) - 1, 0)),
                         replace=False).tolist()) if len(deltas) > 1 else []
    plan = [[0]] + [deltas[a:b] for a, b in zip([0] + cuts, cuts + [len(deltas)]) if b > a]
    for offs in plan:
        start = thr.copy()
        for r in range(world):
            cand = [[] for _ in range(n)]
            for X in np.nonzero(owner_of_block == r)[0]:
                for dl in offs:
                    Y = (X + dl) % T
                    if dl and T % 2 == 0 and dl == T // 2 and X >= T // 2:
                        continue                        # the pair {X, X + T/2} once, from X < T/2
                    rows = np.nonzero(blk == X)[0]
                    cols = np.nonzero(blk == Y)[0]
                    for i in rows:
                        for j in cols:
                            if i == j or (dl == 0 and j < i):
                                continue                # a diagonal block's pairs once each
                            if keys[i, j] < start[i]:
                                cand[i].append(keys[i, j])
                            if keys[j, i] < start[j]:
                                cand[j].append(keys[j, i])
            for p in range(n):
                if cand[p]:
                    merged = np.sort(np.concatenate([lists[r, p], np.array(cand[p], dtype=np.uint64)]))
                    lists[r, p] = merged[:k]
        thr = np.minimum.reduce([lists[r, :, k - 1] for r in range(world)])
    final = np.sort(np.concatenate([lists[r] for r in range(world)], axis=1), axis=1)[:, :k]
    return final, np.sort(keys, axis=1)[:, :k]


@pytest.mark.parametrize("seed,world,block,rounds", [(0, 2, 8, 3), (1, 3, 8, 5), (2, 4, 6, 2), (3, 5, 5, 9),
                                                     (4, 3, 7, 1)])
def test_symmetric_shard_protocol_gives_the_exact_lists(seed, world, block, rounds):
    rng = np.random.default_rng(seed)
    n, d, k = 120, 3, 6
    x = rng.standard_normal((n, d)).astype(np.float32)
    x[rng.integers(0, n, 10)] = x[rng.integers(0, n, 10)]   # duplicates: ties broken by index
    got, want = simulate(x, k, world, block, rounds, rng)
    assert np.array_equal(got, want)
