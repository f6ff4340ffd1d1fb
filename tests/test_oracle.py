"""CPU oracle pinned against the reference's golden vectors and the reference's own host code."""
import numpy as np
import pytest

import fastdec_b200.datasets as ds


def test_spiral_golden_centers(oracle, known, spiral_dm):
    # README.md:105-122: spiral.csv, k=7, c=3, FP32 -> [101, 304, 203]
    r = oracle.fit(spiral_dm, known["spiral"]["k"], known["spiral"]["c"])
    assert r["centers"].tolist() == known["spiral"]["centers"]


def test_dc_reduction_known_case(oracle, known):
    kc = known["dc_known_case"]          # symwarp_unit_test.cu:21-59
    x = np.array([kc["points_1d"]], np.float32)
    cp, delta, rank, centers = oracle.dc_reduction(x, np.array(kc["densities"], np.float32), kc["cores"],
                                                   kc["num_centers"])
    assert cp.tolist() == kc["expected_parents"]
    assert centers.tolist() == [kc["expected_center"]]


def test_dc_reduction_no_denser_point(oracle, known):
    kc = known["dc_no_denser"]           # symwarp_unit_test.cu:61-88
    x = np.array([kc["points_1d"]], np.float32)
    cp, delta, rank, centers = oracle.dc_reduction(x, np.array(kc["densities"], np.float32), kc["cores"],
                                                   kc["num_centers"])
    assert cp.tolist() == kc["expected_parents"]
    assert centers.tolist() == [kc["expected_center"]]
    assert delta.tolist() == [-1.0] and rank.tolist() == [-1]


def test_two_blob_fit(oracle, known):
    tb = known["two_blob_fit"]           # symwarp_unit_test.cu:90-144
    pts = np.array(tb["row_major"], np.float32).reshape(-1, tb["dims"])
    r = oracle.fit(np.ascontiguousarray(pts.T), tb["k"], tb["c"])
    c = r["centers"]
    assert len(c) == 2 and (c < tb["left_count"]).sum() == 1 and (c >= tb["left_count"]).sum() == 1
    assert set(r["labels"].tolist()) <= {0, 1}


def _numpy_knn_exact_small_ints(x_dm, k):
    """For small-integer data every float op is exact, so float64 gives the same d2; lexsort pins
    the (d2, index) tie order independently of the oracle's heap code."""
    x = x_dm.astype(np.float64)
    d, n = x.shape
    g = x.T @ x
    nrm = np.diag(g)
    d2 = np.maximum(nrm[:, None] + nrm[None, :] - 2 * g, 0)
    out_d, out_i = np.empty((k, n), np.float32), np.empty((k, n), np.int32)
    for i in range(n):
        cand = np.delete(np.arange(n), i)
        order = np.lexsort((cand, d2[i, cand]))[:k]
        out_i[:, i] = cand[order]
        out_d[:, i] = np.sqrt(d2[i, cand[order]]).astype(np.float32)
    return out_d, out_i


@pytest.mark.parametrize("n,d,k", [(2, 1, 1), (33, 3, 8), (200, 4, 31), (257, 2, 64), (300, 5, 299)])
def test_oracle_knn_ties_against_lexsort(oracle, n, d, k):
    x = ds.small_integer_grid(n, d, levels=4, seed=n + d)
    dist, idx = oracle.knn(x, k)
    ed, ei = _numpy_knn_exact_small_ints(x, k)
    assert np.array_equal(idx, ei)
    assert np.array_equal(dist, ed)


def test_oracle_knn_rows_match_full(oracle):
    x = ds.gmm_isotropic(n=3000, d=16, seed=11)
    dist, idx = oracle.knn(x, 20)
    rows = np.array([0, 5, 17, 2999, 1500], np.int32)
    d2, ri = oracle.knn_rows(x, 20, rows)
    assert np.array_equal(ri, idx[:, rows].T)
    assert np.array_equal(np.sqrt(d2), dist[:, rows].T)


needs_ref = pytest.mark.skipif(not __import__("oracle").ref_available(), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("gen,k,c,gauss", [
    ("spiral", 7, 3, False),
    ("spiral3", 7, 3, False),
    ("spiral3", 7, 3, True),
    ("gmm", 20, 10, False),
    ("grid", 12, 5, False),
])
def test_oracle_matches_reference_host_stages(oracle, spiral_dm, gen, k, c, gauss):
    """The reference's FastDECBase::Fit (compiled from its sources) and the oracle agree on every
    output given the same kNN and DC-reduction stand-ins: densities bit for bit (sequential mean,
    exp-sum), cores, parents, centers and labels."""
    if gen == "spiral":
        x = spiral_dm
    elif gen == "spiral3":
        x = ds.spiral3(seed=4)
    elif gen == "gmm":
        x = ds.gmm_isotropic(n=4000, d=16, seed=12)
    else:
        x = ds.small_integer_grid(2000, 3, levels=9, seed=3)
    ref = oracle.ref_fit(x, k, c, gaussian=gauss)
    dist, idx = oracle.knn(x, k)
    kk = ref["final_k"]
    den = oracle.density(dist[:kk], gaussian=gauss)
    assert np.array_equal(den.view(np.uint32), ref["densities"].view(np.uint32))
    parent, cores = oracle.dc_detection(idx[:kk], den)
    assert np.array_equal(cores, ref["cores"])
    r = oracle.fit(x, k, c, gaussian=gauss)
    assert r["centers"].tolist() == ref["centers"].tolist()
    assert np.array_equal(r["labels"], ref["labels"])
    assert r["final_k"] == kk


def test_oracle_mean_is_sequential_double(oracle):
    rng = np.random.default_rng(0)
    dist = rng.random((7, 1001)).astype(np.float32) * 3
    s = 0.0
    for i in range(1001):
        for q in range(7):
            s += float(dist[q, i])
    assert oracle.mean_knn_dist(dist) == s / (1001 * 7)
