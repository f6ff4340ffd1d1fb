"""Multi-GPU self-kNN: one process per GPU, the triangle sharded by row blocks.

The reference is single-GPU (its sources use no NCCL or MPI). Here every rank evaluates the block
pairs of its share of the triangle (fdb200_knn_partial with shard = (rank, world)) into partial
lists for ALL points; a partial list is a lexicographic (d2, index) k-smallest of the candidates the
rank saw, so the k-smallest of all ranks' partial lists is the exact answer (the selection is
associative and commutative). Points are owned by contiguous ranges; one all-to-all moves every
partial list to its owner, the owner merges the `world` copies on the GPU, and rank 0 gathers the
merged ranges and runs the O(n k) tail (density, DC detection / reduction, labels) alone.

With the tcgen05 engine a rank tests only the rows of its own blocks against every column block, so
the lists of its own points are already complete and every other list it holds is empty: the
all-to-all and the merge are skipped and each rank contributes its block rows to the gather.

The exchange (`exchange_to_owners`, `gather_to_root`) only uses torch.distributed collectives, so
the same code runs over NCCL on B200s and over gloo on CPU tensors in the tests.
"""
from __future__ import annotations

import os
import sys
import time

import torch
import torch.distributed as dist


def _log(rank, *msg):
    """per-phase stderr line when FASTDEC_BENCH_LOG=1"""
    if os.environ.get("FASTDEC_BENCH_LOG") == "1":
        print(f"[rank {rank} {time.time():.3f}]", *msg, file=sys.stderr, flush=True)


def owner_ranges(n: int, world: int):
    """[start, stop) of the points owned by each rank (balanced contiguous ranges)."""
    return [(n * r // world, n * (r + 1) // world) for r in range(world)]


def exchange_to_owners(lists: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """lists: (n, k) int64 partial lists of all points on this rank. Returns (world, n_own, k):
    block s is rank s's partial list for the points this rank owns."""
    n, k = lists.shape
    rng = owner_ranges(n, world)
    n_own = rng[rank][1] - rng[rank][0]
    out = torch.empty((world, n_own, k), dtype=lists.dtype, device=lists.device)
    dist.all_to_all_single(out.view(-1), lists.reshape(-1),
                           output_split_sizes=[n_own * k] * world,
                           input_split_sizes=[(b - a) * k for a, b in rng])
    return out


def block_ranges(n: int, world: int, block: int = 128):
    """[start, stop) of the points in each rank's row blocks (the split fdb200_knn_partial uses)."""
    T = (n + block - 1) // block
    return [(min(n, block * (T * r // world)), min(n, block * (T * (r + 1) // world))) for r in range(world)]


def gather_to_root(merged: torch.Tensor, n: int, rank: int, world: int, ranges=None):
    """merged: (n_own, k) final lists of this rank's points (its range in `ranges`, the owner ranges
    by default). Rank 0 receives the full (n, k).

    A collective (a gather of equal, padded blocks to rank 0) rather than point-to-point sends:
    collectives on one communicator run in the same order on every rank, so a rank that has already
    moved on to the next step's kernels cannot hold back the transfer that rank 0 is waiting for.
    Only rank 0 receives (and allocates room for) the other ranks' blocks."""
    k = merged.shape[1]
    rng = ranges if ranges is not None else owner_ranges(n, world)
    width = max(b - a for a, b in rng)
    if merged.shape[0] == width and merged.is_contiguous():
        pad = merged
    else:
        pad = torch.empty((width, k), dtype=merged.dtype, device=merged.device)
        pad[:merged.shape[0]].copy_(merged)
    parts = [torch.empty_like(pad) for _ in range(world)] if rank == 0 else None
    dist.gather(pad, gather_list=parts, dst=0)
    if rank != 0:
        return None
    return torch.cat([parts[s][:b - a] for s, (a, b) in enumerate(rng)], dim=0)


class ShardedFit:
    """One fit across `world` GPUs (see the module docstring). step() returns rank-local stats."""

    def __init__(self, n, d, k, c, rank, world, device, stream_ptr, **opts):
        import fastdec_b200 as fdb
        self.fdb = fdb
        self.n, self.d, self.k, self.c = n, d, k, c
        self.rank, self.world, self.dev, self.sp = rank, world, device, stream_ptr
        self.opts = opts
        self.lists = torch.empty((n, k), dtype=torch.int64, device=device)
        if rank == 0:
            self.dist = torch.empty((k, n), dtype=torch.float32, device=device)
            self.idx = torch.empty((k, n), dtype=torch.int32, device=device)

    def step(self, x_dev, centers, labels):
        fdb, n, k = self.fdb, self.n, self.k
        _log(self.rank, "step: partial kNN")
        st = fdb.knn_partial_device(x_dev, k, self.lists, (self.rank, self.world), stream=self.sp, **self.opts)
        n_own = 0
        if st.get("engine_used") == 2:
            # rows-only engine: this rank's block rows are final, nothing to exchange or merge
            rng = block_ranges(n, self.world)
            a, b = rng[self.rank]
            _log(self.rank, "step: gather")
            full = gather_to_root(self.lists[a:b], n, self.rank, self.world, rng)
        else:
            _log(self.rank, "step: exchange", st.get("knn_ms"))
            blocks = exchange_to_owners(self.lists, self.rank, self.world)
            n_own = blocks.shape[1]
            _log(self.rank, "step: merge")
            if n_own > 0:
                fdb.merge_lists_device(blocks[0], blocks[1:], self.world - 1, n_own, k, stream=self.sp,
                                       device=self.dev.index or 0)
            _log(self.rank, "step: gather")
            full = gather_to_root(blocks[0], n, self.rank, self.world)
        _log(self.rank, "step: tail")
        if self.rank == 0:
            fdb.lists_to_knn_device(full, n, k, self.dist, self.idx, stream=self.sp, device=self.dev.index or 0)
            tail = fdb.fit_from_knn_device(x_dev, self.dist, self.idx, k, self.c, centers, labels, stream=self.sp,
                                           **{kk: v for kk, v in self.opts.items() if kk != "engine"})
            for key in ("density_ms", "dc_ms", "labels_ms", "num_cores", "final_k"):
                st[key] = tail[key]
            st["launches"] = st.get("launches", 0) + tail.get("launches", 0) + 1   # + lists_to_knn
        if n_own > 0:
            st["launches"] = st.get("launches", 0) + 1                              # + merge
        _log(self.rank, "step: done")
        return st

    def close(self):
        self.lists = None
