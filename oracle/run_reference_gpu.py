#!/usr/bin/env python
"""Times the reference's own GPU path (cyberbull66/symwarp-fastdec, built unmodified from its sources
into oracle/_ref by `make -C oracle refgpu`) on this machine's GPU, on the seeded synthetic stand-in
of the headline workload. MEASUREMENT / TEST INFRASTRUCTURE: nothing in the product calls this.

    python oracle/run_reference_gpu.py [--binary oracle/_ref/symwarp-fastdec-fds] [--backend symwarp]
                                      [--n 1291147] [--d 50] [--k 45] [--c 20] [--runs 3]

It writes the dataset as the reference's CSV input (one point per line, shortest round-trip float
text, so the reference parses exactly the float32 values bench.py uses), a 4-line config (CSV path,
k, clusters, runs; test.cpp:314-335), runs the binary, and prints one JSON line with the wall time
of the whole process, the reference's own per-run timer lines ("Finished run i of ...", rusage CPU
seconds of the host thread; the CUDA runtime spin-waits, so they track wall time), its per-stage
timers (FASTDEC_STAGE_TIMING builds) and the centers. bench.py imports time_reference_gpu for its
reference_gpu field.
"""
from __future__ import annotations

import argparse
import json
import re
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "symwarp-fastdec_b200"))


def write_csv(x_dm, path):
    """the reference CLI's CSV input, written by the library (shortest round-trip float text, so
    read_data parses back the exact float32 values)"""
    import fastdec_b200 as fdb
    fdb.write_csv(path, x_dm)


def time_reference_gpu(x_dm, k, c, binary, runs=2, backend="symwarp", workdir="/tmp/fdb_refgpu",
                       density_threads=0, timeout=900):
    """Runs the reference binary on x_dm (dim-major float32) and returns its own timers: Fit seconds
    per run, the per-stage seconds (kNN on the GPU; density, DC detection and final clustering on the
    host cores, with FASTDEC_DENSITY_THREADS=density_threads, 0 = all cores), and the centers."""
    import os
    wd = Path(workdir)
    wd.mkdir(parents=True, exist_ok=True)
    d, n = x_dm.shape
    csv = wd / f"data_{n}x{d}.csv"
    t0 = time.time()
    write_csv(x_dm, csv)
    t_csv = time.time() - t0
    cfg = wd / "config.txt"
    cfg.write_text(f"{csv}\n{k}\n{c}\n{runs}\n")
    env = dict(os.environ, FASTDEC_DENSITY_THREADS=str(density_threads))
    t0 = time.time()
    r = subprocess.run([str(binary), "--backend", backend, str(cfg)], capture_output=True, text=True, env=env,
                       timeout=timeout)
    wall = time.time() - t0
    out = r.stdout
    fit = [float(m.group(2)) for m in re.finditer(r"Finished run (\d+) of [^:]*: ([0-9.eE+-]+)", out)]
    stages = {}
    for m in re.finditer(r"Finished (building kNN graph|density estimation|DC detection|DC reduction|final clustering): "
                         r"([0-9.eE+-]+)", out):
        stages.setdefault(m.group(1), []).append(float(m.group(2)))
    prep = re.search(r"Finished preparation of data including Transpose: ([0-9.eE+-]+)", out)
    centers = re.findall(r"Cluster centers found: \s*\nlength: \d+\n(\[.*\])", out)
    try:
        csv.unlink()
    except OSError:
        pass
    return {"binary": Path(binary).name, "backend": backend, "rc": r.returncode, "n": n, "d": d, "k": k, "c": c,
            "runs": runs, "process_wall_s": wall, "csv_write_s": t_csv,
            "prep_cpu_s": float(prep.group(1)) if prep else None, "fit_s_per_run": fit, "stage_s": stages,
            "density_threads": density_threads, "host_cores": os.cpu_count(),
            "centers": json.loads(centers[-1]) if centers else None,
            "stdout_tail": out[-600:] if r.returncode else "", "stderr_tail": r.stderr[-400:]}


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--binary", default=str(ROOT / "oracle" / "_ref" / "symwarp-fastdec-fds"))
    p.add_argument("--backend", default="symwarp")
    p.add_argument("--n", type=int, default=1_291_147)
    p.add_argument("--d", type=int, default=50)
    p.add_argument("--k", type=int, default=45)
    p.add_argument("--c", type=int, default=20)
    p.add_argument("--runs", type=int, default=3)
    p.add_argument("--seed", type=int, default=3)
    p.add_argument("--density-threads", type=int, default=0)
    p.add_argument("--workdir", default="/tmp/fdb_refgpu")
    a = p.parse_args()
    from fastdec_b200.datasets import embedding_cloud
    res = time_reference_gpu(embedding_cloud(n=a.n, d=a.d, seed=a.seed), a.k, a.c, a.binary, a.runs, a.backend,
                             a.workdir, a.density_threads)
    print(json.dumps(res), flush=True)
    return res["rc"]


if __name__ == "__main__":
    sys.exit(main())
