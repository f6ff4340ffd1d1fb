"""Full-size end-to-end parity on the headline workload (1,291,147 x 50, k = 45, c = 20, the seeded
synthetic stand-in for GloVe 50d):

* the whole fit returns the cluster centers that the reference's own GPU Fit returned on a B200 for
  the same float32 data (fixture written by oracle/run_reference_gpu.py from the reference binaries
  built by `make -C oracle refgpu`; its FDS and cuBLAS FP32 builds agree);
* 2,000 random rows of the engine's kNN graph equal the CPU oracle's exact lists bit for bit;
* the reference's OWN host stages (fastdecbase.cpp compiled from its sources, oracle/_ref), run on the
  engine's kNN graph, give the same mean, densities, cores, parents (detection + DC reduction),
  labels and centers as the engine, bit for bit -- the north star's "density, parent and label
  arrays bit-exact given identical kNN lists" at the headline size. The densities use CUDA's double
  exp() where the reference uses the host C library's; the test prints how many of the 1.29M
  densities differ because of that (and fails if any does)."""
import json
from pathlib import Path

import numpy as np
import pytest

import fastdec_b200 as fdb
from fastdec_b200.datasets import embedding_cloud

GOLDEN = Path(__file__).parent / "golden" / "reference_gpu_cloud_1291147x50_k45_c20.json"
N, D, K, C = 1_291_147, 50, 45, 20

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def headline():
    return embedding_cloud(n=N, d=D, seed=3)


def test_fullsize_centers_match_reference_gpu_fit(headline):
    g = json.loads(GOLDEN.read_text())
    r = fdb.fit(headline, g["k"], g["c"])
    assert r["stats"]["engine_used"] == 2, "the tcgen05 engine should run this shape"
    assert r["centers"].tolist() == g["centers_fds_build"]
    assert r["centers"].tolist() == g["centers_cublas_fp32_build"]
    labels = r["labels"]
    assert labels.min() >= 0 and labels.max() < g["c"]
    # every center carries its own label
    assert np.array_equal(labels[r["centers"]], np.arange(g["c"]))


def test_fullsize_knn_rows_and_reference_host_stages(headline, oracle):
    x = headline
    dist, idx, st = fdb.knn(x, K)
    assert st["engine_used"] == 2 and st["pairs"] == N * (N - 1) // 2
    # 2,000 random rows against the oracle's exact per-row kNN, bit for bit (ties included)
    rows = np.random.default_rng(11).choice(N, 2000, replace=False).astype(np.int32)
    d2, ri = oracle.knn_rows(x, K, rows)
    assert np.array_equal(idx[:, rows].T, ri)
    assert np.array_equal(dist[:, rows].T.view(np.uint32), np.sqrt(d2).view(np.uint32))
    # whole-graph properties: ascending, no self, distinct neighbours
    assert (np.diff(dist, axis=0) >= 0).all()
    assert (idx != np.arange(N, dtype=np.int32)[None, :]).all()
    assert (np.diff(np.sort(idx, axis=0), axis=0) != 0).all()

    # the exact sequential-double mean of all N*K distances (fastdecbase.cpp:257-274)
    _, mean = fdb.density(dist)
    assert mean == oracle.mean_knn_dist(dist)

    # the reference's own stages on the engine's graph, against the engine's fit
    ref = oracle.ref_fit_from_knn(x, dist, idx, C)
    r = fdb.fit(x, K, C)
    fk = ref["final_k"]
    assert r["stats"]["final_k"] == fk and r["stats"]["num_cores"] == ref["num_cores"]
    mism = int(np.count_nonzero(r["densities"].view(np.uint32) != ref["densities"].view(np.uint32)))
    print(f"\nheadline densities differing between device exp() and the host C library's exp(): {mism} of {N}")
    assert mism == 0
    assert r["centers"].tolist() == ref["centers"].tolist()
    assert np.array_equal(r["labels"], ref["labels"])

    # cores and parents through the stage entry points: DC detection at the final k, then the DC
    # reduction's parents written into the cores' slots (fastdecbase.cpp:335-356)
    parent, cores = fdb.dc_detection(idx, r["densities"], k=fk)
    assert np.array_equal(cores, ref["cores"])
    if len(cores) > C:
        core_parent, centers = fdb.dc_reduction(x, r["densities"], cores, C)
        assert centers.tolist() == ref["centers"].tolist()
        parent[cores] = core_parent
    assert np.array_equal(parent, ref["parents"])
