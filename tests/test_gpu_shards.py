"""Every shard of the sharded self-kNN run one after another on ONE GPU (fdb200_knn_partial with
shard = (rank, world)), so the sharded kernel path is covered on a one-GPU box. With the tcgen05 engine
a shard tests its own row blocks against every column block, so the lists of its own points are final
and the shards' ranges put together equal the unsharded lists. With the SIMT engine (symmetric tiles)
every shard holds partial lists for all points, and their per-point merge by the library
(fdb200_merge_lists, the k smallest keys) equals the unsharded lists."""
import numpy as np
import pytest

from fastdec_b200.datasets import embedding_cloud, scale_out
from fastdec_b200.multigpu import block_ranges, owner_ranges

pytestmark = pytest.mark.gpu


def _lists(fdb, xd, k, shard, engine, precision="fp32"):
    import torch
    n = xd.shape[1]
    out = torch.empty((n, k), dtype=torch.int64, device=xd.device)
    st = fdb.knn_partial_device(xd, k, out, shard, engine=engine, precision=precision)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint64), st


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("engine", ["tcgen05", "auto", "simt"])
def test_shards_on_one_gpu_equal_the_unsharded_lists(fdb, world, engine):
    """auto: a shard's dense first rounds run on rows-only SIMT tiles, the rest on tcgen05 -- its own
    rows are final either way"""
    import torch
    n, k = 40_000, 45
    xd = torch.from_numpy(embedding_cloud(n=n, d=50, seed=31)).cuda()
    full, _ = _lists(fdb, xd, k, (0, 1), engine)
    parts = [_lists(fdb, xd, k, (r, world), engine) for r in range(world)]
    assert all(st["engine_used"] == (1 if engine == "simt" else 2) for _, st in parts)
    assert sum(st["pairs"] for _, st in parts) == n * (n - 1) // 2
    if engine != "simt":
        got = np.concatenate([p[a:b] for (p, _), (a, b) in zip(parts, block_ranges(n, world))])
    else:
        # the owners' merge of the exchanged partial lists, by the library (fdb200_merge_lists), for
        # each owner range as ShardedFit runs it after the all-to-all
        got = np.empty_like(full)
        for a, b in owner_ranges(n, world):
            own = torch.from_numpy(parts[0][0][a:b].view(np.int64).copy()).cuda()
            srcs = torch.from_numpy(np.stack([p[a:b].view(np.int64) for p, _ in parts[1:]])).cuda()
            fdb.merge_lists_device(own, srcs, world - 1, b - a, k)
            got[a:b] = own.cpu().numpy().view(np.uint64)
        # and the same selection restated on the host
        assert np.array_equal(np.sort(np.concatenate([p for p, _ in parts], axis=1), axis=1)[:, :k], full)
    assert np.array_equal(got, full)


def test_weighted_shards_with_overflow_reruns_stay_exact(fdb):
    """explicit (uneven) row-block ranges, rows-only SIMT rounds that overflow a small candidate buffer
    and are re-planned in halves: the shards' own rows still equal the unsharded lists"""
    import torch
    from fastdec_b200.multigpu import block_split
    n, k, world = 6000, 8, 3
    x = np.zeros((2, n), np.float32)
    x[0] = np.random.default_rng(1).integers(0, 2, n)
    xd = torch.from_numpy(x).cuda()
    full, _ = _lists(fdb, xd, k, (0, 1), "simt")
    got = []
    for r, (b0, b1) in enumerate(block_split(n, world, 0.5)):
        out = torch.empty((n, k), dtype=torch.int64, device=xd.device)
        st = fdb.knn_partial_device(xd, k, out, (r, world), engine="auto", cand_capacity=256, blocks=(b0, b1))
        torch.cuda.synchronize()
        got.append(out.cpu().numpy().view(np.uint64)[128 * b0:min(n, 128 * b1)])
    assert np.array_equal(np.concatenate(got), full)


def test_shards_at_128_dimensions_split_k(fdb):
    """The split-K tile shape (K = 136) on shards, in TF32 mode as the scale-out configuration runs."""
    import torch
    n, k, world = 30_000, 64, 4
    xd = torch.from_numpy(scale_out(n=n, d=128, seed=32)).cuda()
    full, _ = _lists(fdb, xd, k, (0, 1), "tcgen05", "tf32")
    parts = [_lists(fdb, xd, k, (r, world), "tcgen05", "tf32")[0] for r in range(world)]
    got = np.concatenate([p[a:b] for p, (a, b) in zip(parts, block_ranges(n, world))])
    assert np.array_equal(got, full)
