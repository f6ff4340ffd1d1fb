"""The sharded fit on two GPUs (one process per GPU, NCCL): the kNN triangle split by row blocks, the
partial lists exchanged to their owners with an all-to-all (SIMT engine) and merged, gathered on rank
0, and the fit finished there must give exactly the single-GPU centers and labels. Skipped on a
one-GPU machine."""
import os
import socket

import numpy as np
import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, n, q, engine, share, sym, cap, c=10):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    import fastdec_b200 as fdb
    from fastdec_b200.datasets import embedding_cloud
    from fastdec_b200.multigpu import ShardedFit
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        x = embedding_cloud(n=n, d=50, seed=5)
        xd = torch.from_numpy(x).to(dev)
        k = 30
        sp = torch.cuda.current_stream(dev).cuda_stream
        runner = ShardedFit(n, 50, k, c, rank, world, dev, sp, rank0_share=share, engine=engine, sym_shards=sym,
                            cand_capacity=cap)
        centers = torch.empty(c, dtype=torch.int32, device=dev)
        labels = torch.empty(n, dtype=torch.int32, device=dev)
        for _ in range(2):   # twice: buffers and lists are reused across steps
            runner.step(xd, centers, labels)
        torch.cuda.synchronize(dev)
        if sym and not (runner.hook and runner.hook.calls > 0):
            raise RuntimeError("symmetric shards ran without their round hook")
        if rank == 0:
            ref = fdb.fit(x, k, c, engine=engine)
            same = (centers.cpu().numpy().tolist() == ref["centers"].tolist()
                    and np.array_equal(labels.cpu().numpy(), ref["labels"]))
            q.put((rank, "ok" if same else "mismatch"))
        else:
            q.put((rank, "ok"))
        dist.barrier()
        runner.close()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e)))


@pytest.mark.gpu
@pytest.mark.parametrize("engine,share,sym,cap", [("auto", 1.0, False, 0), ("auto", 0.8, False, 0),
                                                  ("simt", 1.0, False, 0), ("auto", 1.0, True, 0),
                                                  ("auto", 0.8, True, 0), ("auto", 1.0, True, 256)])
def test_sharded_fit_on_two_gpus_matches_one_gpu(engine, share, sym, cap):
    """engine auto: rows-only shards (SIMT tiles for the dense rounds, then tcgen05), each rank's rows
    final, gather only; share 0.8 gives rank 0 a smaller share of the triangle. engine simt: symmetric
    tiles, partial lists for every point, the NCCL all-to-all to the owners and fdb200_merge_lists.
    Symmetric shards (sym): each unordered block pair once over both GPUs, both endpoints tested,
    thresholds combined after every round through the round hook, partial lists exchanged to their
    owners; cap 256 makes candidate overflows (re-planned alike on both ranks) likely. Either way the
    DC reduction is sharded over both GPUs."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, 150_000 if engine == "auto" else 40_000, q, engine, share, sym, cap)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert results == {0: "ok", 1: "ok"}


@pytest.mark.gpu
def test_symmetric_shards_with_an_empty_shard_match_one_gpu():
    """300 points are 3 blocks of 128: with rank0_share 0.1 rank 0 gets no row blocks at all, yet under
    symmetric shards it must still make every round-hook call the other rank makes (or that rank's
    collectives would wait for it) and take part in the exchange; the fit equals the one-GPU fit."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from fastdec_b200.multigpu import block_split
    assert block_split(300, 2, 0.1)[0] == (0, 0)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, 300, q, "auto", 0.1, True, 0, 3)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert results == {0: "ok", 1: "ok"}
