"""Multi-GPU fit: one process per GPU, the kNN triangle sharded by row blocks, the DC reduction sharded
by points.

The reference is single-GPU (its sources use no NCCL or MPI). Here every rank evaluates the block pairs
of its share of the triangle (fdb200_knn_partial on its row blocks), in one of two ways:
  ordered shards (`sym_shards=False`, or FASTDEC_SYM_SHARDS=0): with the tcgen05 engine and the
    automatic engine (whose dense first rounds run on rows-only SIMT tiles when sharded) a rank tests
    its own rows against every column block, so the lists of its own points are final when its rounds
    end; rank 0 gathers them.
  symmetric shards (the default with the tcgen05 and automatic engines): a rank multiplies only the block pairs
    whose first block is its own, once, and tests both endpoints, as the one-GPU schedule does, so the
    shards together do half the tensor work. Its tiles then update points of every rank: after every
    round the library calls back (`round_hook`) and the ranks combine the round's overflow flags (MAX,
    so an overflowed round is discarded and re-planned alike everywhere) and every point's threshold
    (unsigned MIN of the packed keys: each rank's k-th key bounds the union's, so each rank filters with
    the tightest). At the end the partial lists go to their owners as below.
With the SIMT engine (and with symmetric shards) a rank's tiles update points of every rank, so its
partial lists go to their owners with one all-to-all and the owners merge them (the lexicographic
(d2, index) k-smallest is associative and commutative, so the merged lists equal the single-GPU ones).

After the kNN, rank 0 computes the densities and the DC detection with the k-halving loop (O(n k):
the exact sequential-double mean needs the whole graph in order). The DC reduction -- a cores x N
contraction -- is sharded: rank 0 broadcasts the densities and the cores, every rank reduces its own
range of points (fdb200_dc_stage), the packed (d2, index) minimum combines with one all-reduce MIN and
the rank counts with one all-reduce SUM, and rank 0 selects the centers and propagates the labels.
Rank 0 carries the last of that tail alone, so its share of the triangle can be made smaller
(`rank0_share`, relative to an even split).

Every collective (`exchange_to_owners`, `gather_to_root`, the broadcasts and all-reduces) is a
torch.distributed collective issued in the same order on every rank, so the same code runs over NCCL on
B200s and over gloo on CPU tensors in the tests.
"""
from __future__ import annotations

import os
import sys
import time

import torch
import torch.distributed as dist

BLOCK = 128


def _log(rank, *msg):
    """per-phase stderr line when FASTDEC_BENCH_LOG=1"""
    if os.environ.get("FASTDEC_BENCH_LOG") == "1":
        print(f"[rank {rank} {time.time():.3f}]", *msg, file=sys.stderr, flush=True)


def owner_ranges(n: int, world: int):
    """[start, stop) of the points owned by each rank (balanced contiguous ranges)."""
    return [(n * r // world, n * (r + 1) // world) for r in range(world)]


def block_split(n: int, world: int, rank0_share: float = 1.0, block: int = BLOCK):
    """[b_lo, b_hi) row blocks of each rank: the even split of the T = ceil(n / block) blocks that
    fdb200_knn_partial makes from (rank, world), or, with rank0_share < 1, rank 0 taking that fraction
    of an even share and the other ranks splitting the rest evenly."""
    T = (n + block - 1) // block
    if world == 1:
        return [(0, T)]
    if rank0_share >= 1.0:
        return [(T * r // world, T * (r + 1) // world) for r in range(world)]
    b0 = int(round(max(rank0_share, 0.0) * T / world))
    rest = T - b0
    return [(0, b0)] + [(b0 + rest * (r - 1) // (world - 1), b0 + rest * r // (world - 1)) for r in range(1, world)]


def block_ranges(n: int, world: int, block: int = BLOCK, rank0_share: float = 1.0):
    """[start, stop) of the points in each rank's row blocks (block_split in points)."""
    return [(min(n, block * a), min(n, block * b)) for a, b in block_split(n, world, rank0_share, block)]


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


_SIGN = -(1 << 63)   # int64 with only the top bit set


def keys_to_signed(best: torch.Tensor) -> torch.Tensor:
    """Packed uint64 keys (held in int64) mapped so that a signed MIN is the unsigned MIN: a valid key
    has a clear top bit (d2 >= 0), the empty key UINT64_MAX has every bit set; flipping the top bit
    keeps the unsigned order and sends the empty key to INT64_MAX. The map is its own inverse."""
    return torch.bitwise_xor(best, _SIGN)


def all_reduce_keys_min(best: torch.Tensor):
    """in place: the minimum over ranks of packed uint64 keys (held in int64)"""
    s = keys_to_signed(best)
    dist.all_reduce(s, op=dist.ReduceOp.MIN)
    best.copy_(keys_to_signed(s))


class _DeviceArray:
    """CUDA array interface over `count` elements at a device pointer of the library (no copy)"""

    def __init__(self, ptr, count, typestr):
        self.__cuda_array_interface__ = {"shape": (int(count),), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 2}


class RoundHook:
    """The symmetric shards' round hook: combines the library's per-round flags (MAX) and per-point
    thresholds (unsigned MIN) over all ranks with torch.distributed, on the current stream (which is
    the stream the library runs on). Errors inside the callback are kept and raised after the call."""

    def __init__(self, device):
        import fastdec_b200 as fdb
        self.device = device
        self.errors = []
        self.calls = 0
        self.flags_kind = fdb.HOOK_FLAGS
        self.c_hook = fdb.ROUND_HOOK(self._hook)

    def combine(self, kind, t: torch.Tensor):
        """in place over all ranks: int32 flags by MAX, packed uint64 keys (held in int64) by unsigned MIN"""
        if kind == self.flags_kind:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        else:
            all_reduce_keys_min(t)

    def _hook(self, ctx, kind, ptr, count, stream):
        try:
            self.calls += 1
            typestr = "<i4" if kind == self.flags_kind else "<i8"
            self.combine(kind, torch.as_tensor(_DeviceArray(ptr, count, typestr), device=self.device))
        except Exception as e:   # an exception cannot cross the C call; raise it after the call returns
            self.errors.append(e)

    def check(self):
        if self.errors:
            err, self.errors = self.errors[0], []
            raise RuntimeError(f"round hook failed: {err!r}")


class ShardedFit:
    """One fit across `world` GPUs (see the module docstring). step() returns rank-local stats."""

    def __init__(self, n, d, k, c, rank, world, device, stream_ptr, rank0_share=None, sym_shards=None, **opts):
        import fastdec_b200 as fdb
        self.fdb = fdb
        self.n, self.d, self.k, self.c = n, d, k, c
        self.rank, self.world, self.dev, self.sp = rank, world, device, stream_ptr
        self.dev_index = device.index or 0
        self.opts = opts
        if rank0_share is None:
            rank0_share = float(os.environ.get("FASTDEC_RANK0_SHARE", "1.0"))
        self.set_rank0_share(rank0_share)
        if sym_shards is None:
            sym_shards = os.environ.get("FASTDEC_SYM_SHARDS", "1") == "1"
        self.sym = bool(sym_shards) and world > 1 and opts.get("engine", "auto") != "simt"
        self.hook = RoundHook(device) if self.sym else None
        self.lists = torch.empty((n, k), dtype=torch.int64, device=device)
        if rank == 0:
            self.dist = torch.empty((k, n), dtype=torch.float32, device=device)
            self.idx = torch.empty((k, n), dtype=torch.int32, device=device)
            self.parent = torch.empty(n, dtype=torch.int32, device=device)
        self.den = torch.empty(n, dtype=torch.float32, device=device)
        self.cores = torch.empty(n, dtype=torch.int32, device=device)
        self.meta = torch.zeros(2, dtype=torch.int64, device=device)

    def set_rank0_share(self, share):
        """rank 0's share of the triangle relative to an even split (must be the same on every rank)"""
        self.rank0_share = share
        self.blocks = block_split(self.n, self.world, share)
        self.ranges = block_ranges(self.n, self.world, rank0_share=share)

    def step(self, x_dev, centers, labels):
        fdb, n, k, c, rank, world, sp = self.fdb, self.n, self.k, self.c, self.rank, self.world, self.sp
        _log(rank, "step: partial kNN")
        hook = {"round_hook": self.hook.c_hook} if self.sym else {}
        st = fdb.knn_partial_device(x_dev, k, self.lists, (rank, world), stream=sp, blocks=self.blocks[rank],
                                    **hook, **self.opts)
        if self.sym:
            self.hook.check()
        n_own = 0
        if st.get("engine_used") == 2 and not self.sym:
            # rows-only schedule: this rank's block rows are final, nothing to exchange or merge
            a, b = self.ranges[rank]
            _log(rank, "step: gather")
            full = gather_to_root(self.lists[a:b], n, rank, world, self.ranges)
        else:
            _log(rank, "step: exchange", st.get("knn_ms"))
            blocks = exchange_to_owners(self.lists, rank, world)
            n_own = blocks.shape[1]
            _log(rank, "step: merge")
            if n_own > 0:
                fdb.merge_lists_device(blocks[0], blocks[1:], world - 1, n_own, k, stream=sp, device=self.dev_index)
            _log(rank, "step: gather")
            full = gather_to_root(blocks[0], n, rank, world)
        # densities and DC detection (k-halving included) on rank 0
        tail_opts = {kk: v for kk, v in self.opts.items() if kk != "engine"}
        launches = 0
        if rank == 0:
            fdb.lists_to_knn_device(full, n, k, self.dist, self.idx, stream=sp, device=self.dev_index)
            nc, fk = fdb.density_detection_device(self.dist, self.idx, k, c, self.den, self.parent, self.cores,
                                                  stream=sp, device=self.dev_index, **tail_opts)
            self.meta[0], self.meta[1] = nc, fk
            launches += 1 + 10
        _log(rank, "step: broadcast cores")
        dist.broadcast(self.meta, src=0)
        nc, fk = int(self.meta[0].item()), int(self.meta[1].item())
        st["num_cores"], st["final_k"] = nc, fk
        if nc > c:
            # the DC reduction sharded by points: stage A, all-reduce MIN, stage B, all-reduce SUM
            dist.broadcast(self.den, src=0)
            cores = self.cores[:nc]
            dist.broadcast(cores, src=0)
            p_lo, p_hi = owner_ranges(n, world)[rank]
            best = torch.empty(nc, dtype=torch.int64, device=self.dev)
            rk = torch.empty(nc, dtype=torch.int32, device=self.dev)
            _log(rank, "step: DC stage A")
            fdb.dc_stage_device(0, x_dev, self.den, cores, nc, p_lo, p_hi, best, stream=sp)
            all_reduce_keys_min(best)
            _log(rank, "step: DC stage B")
            fdb.dc_stage_device(1, x_dev, self.den, cores, nc, p_lo, p_hi, best, rk, stream=sp)
            dist.all_reduce(rk, op=dist.ReduceOp.SUM)
            launches += 6
            if rank == 0:
                core_parent = torch.empty(nc, dtype=torch.int32, device=self.dev)
                fdb.dc_select_device(self.den, cores, nc, best, rk, c, core_parent, centers, stream=sp,
                                     device=self.dev_index)
                self.parent[cores.long()] = core_parent
                launches += 3
        elif rank == 0:
            centers.copy_(self.cores[:c])
        if rank == 0:
            fdb.final_cluster_device(self.parent, centers, labels, stream=sp, device=self.dev_index)
            launches += 3 + max(1, (n - 1).bit_length())
        if n_own > 0:
            launches += 1
        st["launches"] = st.get("launches", 0) + launches
        _log(rank, "step: done")
        return st

    def close(self):
        self.lists = None
