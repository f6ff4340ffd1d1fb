"""tcgen05 engine: bit-exact FP32 parity with the oracle (TF32 filter + exact refine), and the
TF32 distance mode against exact distances within TF32 error."""
import numpy as np
import pytest

import fastdec_b200.datasets as ds

pytestmark = pytest.mark.gpu


def _exact(fdb, oracle, x, k, **kw):
    dist, idx, st = fdb.knn(x, k, engine="tcgen05", **kw)
    assert st["engine_used"] == 2
    od, oi = oracle.knn(x, k)
    assert np.array_equal(idx, oi), f"first index mismatch at {np.argwhere(idx != oi)[:3].tolist()}"
    assert np.array_equal(dist.view(np.uint32), od.view(np.uint32))
    return st


@pytest.mark.parametrize("n,d,k", [(2, 1, 1), (129, 3, 5), (300, 2, 7), (1000, 16, 20), (2049, 50, 45),
                                   (5000, 8, 31), (3000, 50, 10), (777, 47, 30)])
def test_tc_bit_exact_small(fdb, oracle, n, d, k):
    rng = np.random.default_rng(7 * n + d)
    x = rng.uniform(-1, 1, (d, n)).astype(np.float32)
    _exact(fdb, oracle, x, k)


def test_tc_spiral(fdb, oracle, spiral_dm):
    _exact(fdb, oracle, spiral_dm, 7)


def test_tc_ties_and_duplicates(fdb, oracle):
    _exact(fdb, oracle, ds.small_integer_grid(2500, 5, levels=4, seed=2), 60)


def test_tc_offset_data_large_norms(fdb, oracle):
    # far from the origin: large |x| stresses the dot-product form of the TF32 margin
    x = ds.gmm_isotropic(n=6000, d=16, seed=5) + 40.0
    _exact(fdb, oracle, x.astype(np.float32), 20)


def test_tc_glove_like(fdb, oracle):
    _exact(fdb, oracle, ds.embedding_cloud(n=30000, d=50, seed=8), 45)


def test_tc_matches_simt_on_large_input(fdb):
    x = ds.embedding_cloud(n=150_000, d=50, seed=9)
    a = fdb.knn(x, 45, engine="tcgen05")
    b = fdb.knn(x, 45, engine="simt")
    assert np.array_equal(a[1], b[1]) and np.array_equal(a[0], b[0])
    assert a[2]["pairs"] == b[2]["pairs"]


def test_tf32_mode_distances_close(fdb, oracle):
    x = ds.gmm_isotropic(n=8000, d=16, seed=3)
    dist, idx, st = fdb.knn(x, 20, engine="tcgen05", precision="tf32")
    od, oi = oracle.knn(x, 20)
    # each returned neighbour's squared distance is within the TF32 error model of its exact d2:
    # |d2_tf32 - d2| <= 2^-8 |x_i||x_j| (coordinate rounding) + 1e-4 (n_i + n_j) (accumulation)
    nrm = oracle.norms(x)
    xc = np.ascontiguousarray(x)
    for i in range(0, 8000, 97):
        for q in range(20):
            j = int(idx[q, i])
            exact_d2 = oracle.lib().or_pair_d2(xc, 8000, 16, nrm, i, j)
            bound = 2 ** -8 * 1.01 * np.sqrt(nrm[i] * nrm[j]) + 1e-4 * (nrm[i] + nrm[j])
            assert abs(float(dist[q, i]) ** 2 - exact_d2) <= bound
    recall = np.mean([len(set(idx[:, i]) & set(oi[:, i])) / 20 for i in range(8000)])
    assert recall > 0.95
    assert (np.diff(dist, axis=0) >= 0).all()


def test_auto_engine_mixes_rounds_and_stays_exact(fdb):
    """The automatic engine runs the first (dense) rounds on the SIMT tiles and the rest on tcgen05;
    the lists must be identical to an all-tcgen05 and an all-SIMT run."""
    x = ds.embedding_cloud(n=120_000, d=50, seed=13)
    a = fdb.knn(x, 45)
    b = fdb.knn(x, 45, engine="tcgen05")
    assert a[2]["engine_used"] == 2 and a[2]["rounds"] == b[2]["rounds"]
    assert np.array_equal(a[1], b[1]) and np.array_equal(a[0], b[0])


@pytest.mark.parametrize("d", [59, 78, 100, 128, 150, 178])
def test_tc_large_dimensions_bit_exact(fdb, oracle, d):
    """K = d + 6 padded to 8. Up to K = 80 two whole row blocks are staged beside the resident column
    pair; beyond that a row stage holds a group of K panels (6 of 11 at d = 78, 7 of 14 at d = 100,
    6 of 17 at d = 128, 4 of 20 at d = 150, 1 of 23 at d = 178, the largest K that fits) and a tile
    takes several stages. The lists stay bit-exact."""
    rng = np.random.default_rng(d)
    x = rng.uniform(-1, 1, (d, 3000)).astype(np.float32)
    _exact(fdb, oracle, x, 20)


def test_tc_scale_out_mixture_sample(fdb, oracle):
    # the 128-dimensional scale-out mixture (k = 64) at a size the oracle finishes in seconds
    _exact(fdb, oracle, ds.scale_out(n=12000, d=128, seed=4), 64)


def test_tc_matches_simt_at_128_dimensions(fdb):
    x = ds.scale_out(n=60000, d=128, seed=6)
    a = fdb.knn(x, 64, engine="tcgen05")
    b = fdb.knn(x, 64, engine="simt")
    assert np.array_equal(a[1], b[1]) and np.array_equal(a[0], b[0])


def test_tf32_mode_at_128_dimensions_close(fdb, oracle):
    x = ds.scale_out(n=6000, d=128, seed=7)
    dist, idx, st = fdb.knn(x, 64, engine="tcgen05", precision="tf32")
    assert st["engine_used"] == 2
    nrm = oracle.norms(x)
    xc = np.ascontiguousarray(x)
    for i in range(0, 6000, 211):
        for q in range(0, 64, 7):
            j = int(idx[q, i])
            exact_d2 = oracle.lib().or_pair_d2(xc, 6000, 128, nrm, i, j)
            bound = 2 ** -8 * 1.01 * np.sqrt(nrm[i] * nrm[j]) + 1e-4 * (nrm[i] + nrm[j])
            assert abs(float(dist[q, i]) ** 2 - exact_d2) <= bound
    od, oi = oracle.knn(x, 64)
    recall = np.mean([len(set(idx[:, i]) & set(oi[:, i])) / 64 for i in range(6000)])
    assert recall > 0.95
    assert (np.diff(dist, axis=0) >= 0).all()
