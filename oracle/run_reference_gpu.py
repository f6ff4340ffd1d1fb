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
seconds of the host thread; the CUDA runtime spin-waits, so they track wall time) and the centers.
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
    xt = x_dm.T
    with open(path, "w") as f:
        for s in range(0, xt.shape[0], 65536):
            blk = xt[s:s + 65536]
            f.write("\n".join(",".join(r) for r in blk.astype(str).tolist()) + "\n")


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
    p.add_argument("--workdir", default="/tmp/fdb_refgpu")
    a = p.parse_args()
    from fastdec_b200.datasets import embedding_cloud
    wd = Path(a.workdir)
    wd.mkdir(parents=True, exist_ok=True)
    csv = wd / f"cloud_{a.n}x{a.d}_s{a.seed}.csv"
    t0 = time.time()
    if not csv.exists():
        write_csv(embedding_cloud(n=a.n, d=a.d, seed=a.seed), csv)
    t_csv = time.time() - t0
    cfg = wd / "config.txt"
    cfg.write_text(f"{csv}\n{a.k}\n{a.c}\n{a.runs}\n")
    t0 = time.time()
    r = subprocess.run([a.binary, "--backend", a.backend, str(cfg)], capture_output=True, text=True)
    wall = time.time() - t0
    out = r.stdout
    runs = [float(m.group(2)) for m in re.finditer(r"Finished run (\d+) of [^:]*: ([0-9.eE+-]+)", out)]
    stages = {}
    for m in re.finditer(r"Finished (building kNN graph|density estimation|DC detection|DC reduction|final clustering): "
                         r"([0-9.eE+-]+)", out):
        stages.setdefault(m.group(1), []).append(float(m.group(2)))
    prep = re.search(r"Finished preparation of data including Transpose: ([0-9.eE+-]+)", out)
    centers = re.findall(r"Cluster centers found: \s*\nlength: \d+\n(\[.*\])", out)
    print(json.dumps({"binary": Path(a.binary).name, "backend": a.backend, "rc": r.returncode, "n": a.n, "d": a.d,
                      "k": a.k, "c": a.c, "runs": a.runs, "process_wall_s": wall, "csv_write_s": t_csv,
                      "prep_cpu_s": float(prep.group(1)) if prep else None, "fit_s_per_run": runs,
                      "stage_s": stages, "centers": json.loads(centers[-1]) if centers else None,
                      "stderr_tail": r.stderr[-400:]}), flush=True)
    if r.returncode != 0:
        print(out[-2000:], file=sys.stderr)
    return r.returncode


if __name__ == "__main__":
    sys.exit(main())
