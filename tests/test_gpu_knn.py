"""Self-kNN parity: the CUDA engine against the CPU oracle, bit for bit (FP32 mode).

The oracle restates the reference FDS build (fmaf-chain dot, two rounded adds, lexicographic
(d2, index) top-k), so equality here is equality with that build, ties included."""
import numpy as np
import pytest

import fastdec_b200.datasets as ds

pytestmark = pytest.mark.gpu


ENGINES = ["simt", "tcgen05"]


def _check_equal(fdb, oracle, x, k, **kw):
    dist, idx, st = fdb.knn(x, k, **kw)
    od, oi = oracle.knn(x, k)
    assert np.array_equal(idx, oi), f"index mismatch at {np.argwhere(idx != oi)[:5]}"
    assert np.array_equal(dist.view(np.uint32), od.view(np.uint32))
    return st


def test_spiral_knn_bit_exact(fdb, oracle, spiral_dm):
    _check_equal(fdb, oracle, spiral_dm, 7)


@pytest.mark.parametrize("n,d,k", [
    (2, 1, 1), (3, 2, 2), (33, 3, 8), (129, 1, 5), (257, 8, 64), (1000, 33, 20),
    (1000, 50, 45), (3001, 16, 20), (640, 100, 10), (5000, 2, 7), (300, 64, 299),
])
@pytest.mark.parametrize("engine", ENGINES)
def test_random_shapes_bit_exact(fdb, oracle, n, d, k, engine):
    rng = np.random.default_rng(n * 131 + d)
    x = rng.uniform(-1, 1, (d, n)).astype(np.float32)
    _check_equal(fdb, oracle, x, k, engine=engine)


@pytest.mark.parametrize("k", [1, 8, 64, 200])
@pytest.mark.parametrize("engine", ENGINES)
def test_integer_grid_ties_bit_exact(fdb, oracle, k, engine):
    # small-integer coordinates: many exact ties and duplicate points (zero distances)
    x = ds.small_integer_grid(1500, 4, levels=5, seed=k)
    _check_equal(fdb, oracle, x, k, engine=engine)


def test_gmm_20k_bit_exact(fdb, oracle):
    x = ds.gmm_isotropic(n=20000, d=16, seed=21)
    st = _check_equal(fdb, oracle, x, 20)
    assert st["pairs"] == 20000 * 19999 // 2


def test_glove_like_sample_bit_exact(fdb, oracle):
    x = ds.embedding_cloud(n=12000, d=50, seed=22)
    _check_equal(fdb, oracle, x, 45)


@pytest.mark.parametrize("engine", ["simt", "tcgen05", "auto"])
def test_small_capacity_forces_overflow_reruns_and_stays_exact(fdb, oracle, engine):
    # two groups of identical points: every candidate from a lower-indexed block beats the current
    # k-th key (all distances tie at 0), so the multi-offset rounds overflow a 256-slot buffer and
    # are re-planned in halves (22 re-runs in a host restatement of the schedule), several of them
    # in the middle of a queued batch of rounds
    x = np.zeros((2, 3000), np.float32)
    x[0] = np.random.default_rng(1).integers(0, 2, 3000)
    st = _check_equal(fdb, oracle, x, 8, cand_capacity=256, engine=engine)
    assert st["overflow_reruns"] > 0


def test_knn_argument_errors(fdb):
    x = np.zeros((2, 10), np.float32)
    with pytest.raises(fdb.FastDecError) as e:
        fdb.knn(x, 10)          # k >= n (symtriknncuda.cu:322-324)
    assert e.value.code == -1
    d, i, _ = fdb.knn(np.zeros((2, 1), np.float32), 3)   # n <= 1: no-op success (:319-321)
    assert d.shape == (3, 1)


@pytest.mark.parametrize("engine", ["simt", "tcgen05"])
def test_large_properties_and_sampled_rows(fdb, oracle, engine):
    """200k x 50 (larger than L2): sorted lists, no self, distinct neighbours, and exact
    agreement with the oracle on sampled rows."""
    n, k = 200_000, 45
    x = ds.embedding_cloud(n=n, d=50, seed=23)
    dist, idx, st = fdb.knn(x, k, engine=engine)
    assert st["pairs"] == n * (n - 1) // 2
    assert (idx != np.arange(n)[None, :]).all()
    assert (np.diff(dist, axis=0) >= 0).all()
    srt = np.sort(idx, axis=0)
    assert (np.diff(srt, axis=0) != 0).all()
    rows = np.random.default_rng(1).choice(n, 400, replace=False).astype(np.int32)
    d2, ri = oracle.knn_rows(x, k, rows)
    assert np.array_equal(idx[:, rows].T, ri)
    assert np.array_equal(dist[:, rows].T, np.sqrt(d2))
