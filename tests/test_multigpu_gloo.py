"""Host-side logic of the sharded kNN (fastdec_b200.multigpu) on CPU: two gloo ranks exchange partial
per-point lists to their owners and gather the merged ranges on rank 0. The k-smallest selection that
fdb200_merge_lists performs on the GPU is restated here with numpy, so the test checks that the exchange
delivers every rank's partial list of every point to exactly the owner of that point, and that the
gathered result equals the k-smallest over all shards (what a single-GPU run computes)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fastdec_b200.multigpu import exchange_to_owners, gather_to_root, owner_ranges

EMPTY = np.uint64(0xFFFFFFFFFFFFFFFF)


def partial_lists(n, k, world, seed):
    """Packed (d2 bits << 32 | idx) partial lists per shard, sorted, with empty tails."""
    rng = np.random.default_rng(seed)
    out = []
    for s in range(world):
        keys = np.full((n, k), EMPTY, dtype=np.uint64)
        for i in range(n):
            m = int(rng.integers(0, k + 1))
            d2 = np.sort(rng.random(m).astype(np.float32))
            idx = rng.integers(0, n, size=m).astype(np.uint64)
            keys[i, :m] = np.sort((d2.view(np.uint32).astype(np.uint64) << np.uint64(32)) | idx)
        out.append(keys)
    return out


def k_smallest(blocks, k):
    cat = np.concatenate(blocks, axis=1)
    return np.sort(cat, axis=1)[:, :k]


def _worker(rank, world, port, n, k, seed, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        parts = partial_lists(n, k, world, seed)
        mine = torch.from_numpy(parts[rank].view(np.int64).copy())
        blocks = exchange_to_owners(mine, rank, world)
        a, b = owner_ranges(n, world)[rank]
        assert blocks.shape == (world, b - a, k)
        for s in range(world):
            assert np.array_equal(blocks[s].numpy().view(np.uint64), parts[s][a:b])
        merged = torch.from_numpy(k_smallest([blocks[s].numpy().view(np.uint64) for s in range(world)], k)
                                  .view(np.int64).copy())
        full = gather_to_root(merged, n, rank, world)
        if rank == 0:
            want = k_smallest(parts, k)
            assert np.array_equal(full.numpy().view(np.uint64), want)
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n,k", [(37, 5), (256, 12), (3, 4)])
def test_exchange_and_gather_two_ranks(n, k):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, k, 7 + n, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}


def test_owner_ranges_cover_every_point_once():
    for n in (1, 5, 128, 1_291_147):
        for world in (1, 2, 3, 8):
            rng = owner_ranges(n, world)
            assert rng[0][0] == 0 and rng[-1][1] == n
            assert all(rng[i][1] == rng[i + 1][0] for i in range(world - 1))


def test_block_ranges_follow_the_kernel_row_block_split():
    from fastdec_b200.multigpu import block_ranges
    for n in (1, 127, 128, 129, 1_291_147):
        for world in (1, 2, 3, 8):
            rng = block_ranges(n, world)
            assert rng[0][0] == 0 and rng[-1][1] == n
            assert all(rng[i][1] == rng[i + 1][0] for i in range(world - 1))
            T = (n + 127) // 128
            assert all(a == min(n, 128 * (T * r // world)) for r, (a, _) in enumerate(rng))


def test_weighted_block_split_gives_rank_0_less():
    from fastdec_b200.multigpu import block_split
    for n in (129, 5000, 1_291_147):
        T = (n + 127) // 128
        for world in (2, 3, 8):
            for share in (0.5, 0.9, 0.96):
                sp = block_split(n, world, share)
                assert sp[0][0] == 0 and sp[-1][1] == T
                assert all(sp[i][1] == sp[i + 1][0] for i in range(world - 1))
                sizes = [b - a for a, b in sp]
                assert abs(sizes[0] - share * T / world) <= 0.5 + 1e-9
                assert max(sizes[1:]) - min(sizes[1:]) <= 1


def _gather_worker(rank, world, port, n, k, q):
    from fastdec_b200.multigpu import block_ranges
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        full = rng.integers(0, 2 ** 62, size=(n, k), dtype=np.int64)   # every rank draws the same lists
        ranges = block_ranges(n, world)
        a, b = ranges[rank]
        got = gather_to_root(torch.from_numpy(full[a:b].copy()), n, rank, world, ranges)
        if rank == 0:
            assert np.array_equal(got.numpy(), full)
        else:
            assert got is None
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n,world", [(1000, 3), (129, 2), (300, 3), (100, 3)])
def test_gather_of_row_block_ranges(n, world):
    """The tcgen05 path of the sharded fit: each rank's own row-block range is final and rank 0
    collects the ranges (uneven widths, a rank with a short or empty range)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, n, 5, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results == {r: "ok" for r in range(world)}


def _dead_peer_worker(rank, world, port, q):
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()
        os._exit(0)   # the peer leaves between steps, before the gather
    try:
        gather_to_root(torch.zeros((5, 3), dtype=torch.int64), 10, rank, world)
        q.put((rank, "no error"))
    except Exception as e:  # the collective must fail, not wait forever
        q.put((rank, "error:" + type(e).__name__))


def test_gather_with_a_dead_peer_fails_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert results[1] == "left"
    assert results[0].startswith("error:")


def test_signed_key_mapping_keeps_the_unsigned_order():
    from fastdec_b200.multigpu import keys_to_signed
    rng = np.random.default_rng(5)
    d2 = np.abs(rng.standard_normal(2000)).astype(np.float32)
    d2[:3] = [0.0, np.float32(np.inf), np.float32(3.4e38)]
    keys = (d2.view(np.uint32).astype(np.uint64) << np.uint64(32)) | rng.integers(0, 2 ** 31, 2000).astype(np.uint64)
    keys[5] = EMPTY
    s = keys_to_signed(torch.from_numpy(keys.view(np.int64).copy())).numpy()
    assert np.array_equal(keys[np.argsort(keys, kind="stable")], keys[np.argsort(s, kind="stable")])
    assert s[5] == np.iinfo(np.int64).max
    assert np.array_equal(keys_to_signed(torch.from_numpy(s.copy())).numpy().view(np.uint64), keys)


def _dc_combine_worker(rank, world, port, q):
    from fastdec_b200.multigpu import all_reduce_keys_min
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(3)
        parts = []
        for s in range(world):   # every rank draws every rank's partial keys, keeps its own
            d2 = np.abs(rng.standard_normal(300)).astype(np.float32)
            k = (d2.view(np.uint32).astype(np.uint64) << np.uint64(32)) | rng.integers(0, 10 ** 6, 300).astype(np.uint64)
            k[rng.random(300) < 0.3] = EMPTY   # cores with no denser point in this rank's range
            parts.append(k)
        mine = torch.from_numpy(parts[rank].view(np.int64).copy())
        all_reduce_keys_min(mine)
        assert np.array_equal(mine.numpy().view(np.uint64), np.minimum.reduce(parts))
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_dc_partial_keys_combine_by_unsigned_min_over_ranks():
    """The sharded DC reduction's stage-A keys (packed uint64 in int64 tensors, UINT64_MAX = no denser
    point) combine across ranks by an all-reduce MIN after the signed mapping."""
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dc_combine_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results == {r: "ok" for r in range(world)}


def _round_hook_worker(rank, world, port, q):
    import fastdec_b200 as fdb
    from fastdec_b200.multigpu import RoundHook
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        hook = RoundHook(torch.device("cpu"))
        # flags: overflow tag and error code, combined by MAX (rank 1 overflowed in round 3)
        flags = torch.tensor([3 if rank == 1 else 0, 0], dtype=torch.int32)
        hook.combine(fdb.HOOK_FLAGS, flags)
        assert flags.tolist() == [3, 0]
        # thresholds: packed keys, unsigned MIN; an empty list's key (UINT64_MAX) loses to any real key
        rng = np.random.default_rng(11)
        parts = []
        for s in range(world):
            d2 = np.abs(rng.standard_normal(500)).astype(np.float32)
            k = (d2.view(np.uint32).astype(np.uint64) << np.uint64(32)) | rng.integers(0, 10 ** 6, 500).astype(np.uint64)
            k[rng.random(500) < 0.2] = EMPTY
            parts.append(k)
        mine = torch.from_numpy(parts[rank].view(np.int64).copy())
        hook.combine(fdb.HOOK_THRESHOLDS, mine)
        assert np.array_equal(mine.numpy().view(np.uint64), np.minimum.reduce(parts))
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_round_hook_combines_flags_by_max_and_thresholds_by_unsigned_min():
    """The symmetric shards' round hook: the round's flags combine by MAX (so every rank sees an
    overflow any rank had), the per-point thresholds by unsigned MIN of the packed keys (each rank's
    k-th key bounds the union's; UINT64_MAX = a list not yet full)."""
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_round_hook_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results == {r: "ok" for r in range(world)}
