"""The drop-in boundary exercised through the reference's own types and programs.

* The reference's unmodified FastDECBase::Fit (fastdecbase.cpp:159-228, compiled from its sources by
  `make -C oracle refplugin`) with the kNN plug-in of symwarp-fastdec_b200/integration/b200knnfastdec.h
  (compute_knn -> fdb200_knn), once with the reference's own cuBLAS DC reduction (dcreductioncuda.cu)
  and once with integration/b200_dc_reduction.cpp (warp_parallel_dc_reduction_cuda ->
  fdb200_dc_reduction): the README spiral golden and a 20,000-point GMM against the oracle.
* The CLI (bin/fastdec_b200, which drives the C++ B200FastDEC) on the reference's config format with
  `--backend b200`: spiral.csv gives the README centers; a .fbin dataset with --save-knn, then
  --load-knn with another cluster count, gives the engine's fits.
* fdb200_fit_from_knn on a saved graph: a graph of 45 ranks serves k = 30 and k = 45.
"""
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import fastdec_b200 as fdb
import fastdec_b200.datasets as ds

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
REF = ROOT / "oracle" / "_ref"
CLI = ROOT / "symwarp-fastdec_b200" / "bin" / "fastdec_b200"


def _plugin_fit(binary, x, k, c, tmp_path):
    d, n = x.shape
    src, out = tmp_path / "x.f32", tmp_path / "out.bin"
    np.ascontiguousarray(x, np.float32).tofile(src)
    r = subprocess.run([str(binary), str(src), str(n), str(d), str(k), str(c), "0", str(out)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-1000:] + r.stderr[-1000:]
    v = np.fromfile(out, np.int32)
    return v[:c], v[c:]


@pytest.mark.parametrize("variant", ["refdc", "b200dc"])
def test_reference_fit_with_the_b200_knn_plugin(variant, spiral_dm, known, oracle, tmp_path):
    binary = REF / f"plugin_fit-{variant}"
    if not binary.exists():
        pytest.skip("reference plug-in driver not built (make -C oracle refplugin)")
    centers, labels = _plugin_fit(binary, spiral_dm, 7, 3, tmp_path)
    assert centers.tolist() == known["spiral"]["centers"]
    assert np.array_equal(labels, fdb.fit(spiral_dm, 7, 3)["labels"])
    g = ds.gmm_isotropic(n=20_000, d=16, seed=1)
    centers, labels = _plugin_fit(binary, g, 20, 10, tmp_path)
    o = oracle.fit(g, 20, 10)
    assert centers.tolist() == o["centers"].tolist()
    assert np.array_equal(labels, o["labels"])


def _run_cli(args, tmp_path):
    r = subprocess.run([str(CLI), *args], capture_output=True, text=True, timeout=600, cwd=tmp_path)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    m = re.findall(r"Cluster centers found: \s*\nlength: \d+\n\[([0-9,\-]*)\]", r.stdout)
    assert m, r.stdout[-2000:]
    return [[int(v) for v in s.split(",") if v] for s in m], r.stdout


def test_cli_backend_b200_on_the_reference_config_format(spiral_dm, known, tmp_path):
    # spiral.csv as the reference ships it: one point per line, shortest round-trip float text
    csv = tmp_path / "spiral.csv"
    csv.write_text("\n".join(",".join(r) for r in spiral_dm.T.astype(str).tolist()) + "\n")
    cfg = tmp_path / "config.txt"
    cfg.write_text(f"{csv}\n7\n3\n2\n")
    centers, out = _run_cli(["--backend", "b200", str(cfg)], tmp_path)
    assert centers == [known["spiral"]["centers"]] * 2, out[-1000:]
    assert "Backend: b200" in out


def test_cli_fbin_input_and_knn_graph_save_load(tmp_path):
    x = ds.gmm_isotropic(n=30_000, d=16, seed=4)
    data = tmp_path / "gmm.fbin"
    fdb.write_fbin(data, x)
    graph = tmp_path / "gmm.knng"
    cfg = tmp_path / "a.txt"
    cfg.write_text(f"{data}\n20\n10\n1\n")
    centers, out = _run_cli(["--save-knn", str(graph), str(cfg)], tmp_path)
    assert centers == [fdb.fit(x, 20, 10)["centers"].tolist()]
    # another cluster count and a smaller k from the saved graph: no kNN is computed
    cfg2 = tmp_path / "b.txt"
    cfg2.write_text(f"{data}\n12\n6\n1\n")
    centers, out = _run_cli(["--load-knn", str(graph), str(cfg2)], tmp_path)
    assert "Loaded a kNN graph of 20 ranks" in out
    assert centers == [fdb.fit(x, 12, 6)["centers"].tolist()]


def test_fit_from_a_saved_graph_serves_smaller_k(tmp_path):
    x = ds.embedding_cloud(n=60_000, d=50, seed=8)
    dist, idx, _ = fdb.knn(x, 45)
    p = tmp_path / "g.knng"
    fdb.save_knn_graph(p, dist, idx)
    gd, gi, _ = fdb.load_knn_graph(p)
    for k, c in [(45, 20), (30, 12)]:
        a = fdb.fit_from_knn(x, gd, gi, k, c)
        b = fdb.fit(x, k, c)
        assert a["centers"].tolist() == b["centers"].tolist()
        assert np.array_equal(a["labels"], b["labels"])
        assert np.array_equal(a["densities"].view(np.uint32), b["densities"].view(np.uint32))
