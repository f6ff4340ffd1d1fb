"""Full-size end-to-end parity: the whole fit on the headline workload (1,291,147 x 50, k = 45,
c = 20, seeded synthetic stand-in) must return the cluster centers that the reference's own GPU Fit
returned on a B200 for the same float32 data (fixture written by oracle/run_reference_gpu.py from
the reference binaries built by `make -C oracle refgpu`; the FDS and the cuBLAS FP32 builds agree)."""
import json
from pathlib import Path

import numpy as np
import pytest

import fastdec_b200 as fdb
from fastdec_b200.datasets import embedding_cloud

GOLDEN = Path(__file__).parent / "golden" / "reference_gpu_cloud_1291147x50_k45_c20.json"


@pytest.mark.gpu
def test_fullsize_centers_match_reference_gpu_fit():
    g = json.loads(GOLDEN.read_text())
    x = embedding_cloud(n=1_291_147, d=50, seed=3)
    r = fdb.fit(x, g["k"], g["c"])
    assert r["stats"]["engine_used"] == 2, "the tcgen05 engine should run this shape"
    assert r["centers"].tolist() == g["centers_fds_build"]
    assert r["centers"].tolist() == g["centers_cublas_fp32_build"]
    labels = r["labels"]
    assert labels.min() >= 0 and labels.max() < g["c"]
    # every center carries its own label
    assert np.array_equal(labels[r["centers"]], np.arange(g["c"]))
