"""Whole-fit parity: centers, labels and densities against the oracle and the reference's own
host stages (oracle/_ref), plus the reference's golden answers."""
import numpy as np
import pytest

import fastdec_b200.datasets as ds

pytestmark = pytest.mark.gpu


def test_spiral_golden_centers(fdb, known, spiral_dm):
    r = fdb.fit(spiral_dm, known["spiral"]["k"], known["spiral"]["c"])
    assert r["centers"].tolist() == known["spiral"]["centers"]      # README.md:105-122


def test_two_blob_fit(fdb, known):
    tb = known["two_blob_fit"]
    pts = np.array(tb["row_major"], np.float32).reshape(-1, tb["dims"])
    r = fdb.fit(np.ascontiguousarray(pts.T), tb["k"], tb["c"])
    c = r["centers"]
    assert (c < tb["left_count"]).sum() == 1 and (c >= tb["left_count"]).sum() == 1
    assert set(r["labels"].tolist()) <= {0, 1}


@pytest.mark.parametrize("name,gauss", [("spiral3", False), ("spiral3", True), ("gmm", False),
                                        ("gmm", True), ("glove", False), ("grid", False)])
def test_fit_matches_oracle(fdb, oracle, name, gauss):
    if name == "spiral3":
        x, k, c = ds.spiral3(seed=9), 7, 3
    elif name == "gmm":
        x, k, c = ds.gmm_isotropic(n=20000, d=16, seed=31), 20, 10
    elif name == "glove":
        x, k, c = ds.embedding_cloud(n=10000, d=50, seed=32), 45, 20
    else:
        x, k, c = ds.small_integer_grid(3000, 3, levels=9, seed=8), 12, 5
    r = fdb.fit(x, k, c, density="gaussian" if gauss else "laplacian")
    o = oracle.fit(x, k, c, gaussian=gauss)
    assert r["centers"].tolist() == o["centers"].tolist()
    assert np.array_equal(r["labels"], o["labels"])
    assert r["stats"]["final_k"] == o["final_k"] and r["stats"]["num_cores"] == o["num_cores"]
    if oracle.ref_available(gauss):
        ref = oracle.ref_fit(x, k, c, gaussian=gauss)
        assert np.array_equal(r["densities"].view(np.uint32), ref["densities"].view(np.uint32))
        assert r["centers"].tolist() == ref["centers"].tolist()
        assert np.array_equal(r["labels"], ref["labels"])


def test_k_halving_path(fdb, oracle):
    # many clusters relative to k forces the "not enough cores" retry (fastdecbase.cpp:186-199)
    x = ds.gmm_isotropic(n=3000, d=4, comps=3, seed=5)
    r = fdb.fit(x, 64, 40)
    o = oracle.fit(x, 64, 40)
    assert o["final_k"] < 64
    assert r["stats"]["final_k"] == o["final_k"]
    assert r["centers"].tolist() == o["centers"].tolist()
    assert np.array_equal(r["labels"], o["labels"])


def test_not_enough_cores_error(fdb, oracle):
    # points 0, 1, 3, 7, ... (gaps doubling): every point's neighbours are denser except two
    x = np.array([[2.0 ** i - 1 for i in range(12)]], np.float32)
    with pytest.raises(RuntimeError):
        oracle.fit(x, 4, 3)
    with pytest.raises(fdb.FastDecError) as e:
        fdb.fit(x, 4, 3)
    assert e.value.code == -4


def test_b200fastdec_class_surface(fdb, known, spiral_dm):
    m = fdb.B200FastDEC(7, 3, "b200_unit_test", 0)
    m.Fit(spiral_dm, spiral_dm.shape[1], spiral_dm.shape[0])
    assert m.get_center_indices().tolist() == known["spiral"]["centers"]
    assert len(m.get_labels()) == spiral_dm.shape[1]
