"""The FAISS-style kNN baseline that bench.py reports beside the fit (brute-force GEMM distances plus a
top-k select, as the reference's faissgpu backend runs GpuIndexFlatL2): its lists must agree with the
exact engine's, so that the timing compares like with like. FP32 GEMM distances differ from the exact
fmaf-chain ones only by rounding (|q|^2 + |x|^2 - 2 q.x with another summation order), so the recall
must be near 1 and the k-th distance agree to the rounding scale; TF32 GEMMs round the coordinates to
11 bits, so they admit a looser tolerance and a lower recall."""
import sys
from pathlib import Path

import numpy as np
import pytest

import fastdec_b200.datasets as ds

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


# tolerance on the k-th squared distance: the GEMM form cancels |q|^2 + |x|^2 against 2 q.x, so its error
# scales with the norms: FP32 about 2^-24 per rounding, TF32 rounds the coordinates to 2^-11
@pytest.mark.parametrize("mode,min_recall,ntol", [("fp32", 0.995, 2.0 ** -18), ("tf32", 0.80, 2.0 ** -8)])
def test_faiss_style_baseline_agrees_with_the_exact_lists(fdb, mode, min_recall, ntol):
    import torch
    sys.path.insert(0, str(ROOT))
    import bench

    n, d, k = 20000, 50, 30
    x = ds.embedding_cloud(n=n, d=d, seed=4)
    dist, idx, _ = fdb.knn(x, k)              # exact: rank-major (k, n), sqrt distances
    dev = torch.device("cuda", 0)
    xd = torch.from_numpy(x).to(dev)
    stream = torch.cuda.current_stream(dev)
    summary, first = bench.run_faiss_style(xd, k, stream, sample=2048, batch=1024)
    assert summary[mode]["knn_s_all_points"] > 0
    qi, v, i = (t.cpu().numpy() for t in first[mode])
    nrm = (x.astype(np.float64) ** 2).sum(0)
    nmax = float(nrm.max())
    hits, total = 0, 0
    for r, q in enumerate(qi):
        # drop the query itself (distance 0 at rank 0, or tied with an exact duplicate)
        got = [j for j in i[r].tolist() if j != q][:k]
        want = idx[:, q].tolist()
        hits += len(set(got) & set(want))
        total += k
        # the k-th neighbour's squared distance: GEMM value vs exact value
        kth_exact = float(dist[k - 1, q]) ** 2
        kth_gemm = float(np.sort(v[r][i[r] != q])[k - 1])
        assert abs(kth_gemm - kth_exact) <= ntol * (nrm[q] + nmax), (mode, q, kth_gemm, kth_exact)
    assert hits / total >= min_recall, (mode, hits / total)
