"""Audit of the tcgen05 filter's margin (FP32 mode), the assumption the engine's bit-exactness rests on.

The engine keeps a pair (i, j) for the exact refine iff the tensor cores' FP32 accumulation of
|x~_i - x~_j|^2 - V_i is negative, where x~ are the TF32-rounded coordinates and V_i is point i's
threshold plus a rigorous margin (knn_common.cuh: filter_bound, fold_bound). Part of that margin is an
error model of the tcgen05 kind::tf32 accumulation: at most 2^-20 of the summed term magnitudes per
K-step of 8. Here, for every ordered pair of small problems (fdb200_debug_tc_filter):
  * every admissible candidate (exact FP32 d2 <= the point's exact k-th d2) has a negative accumulator;
  * the observed accumulation error |acc - exact sum of the same TF32 operands (float64)| stays below
    the modelled bound, and the largest ratio is reported;
  * the tcgen05 engine's lists equal the oracle's, bit for bit,
on the benchmark-like clouds and on an adversarial cloud far from the origin (|x|^2 >> d2, which makes
the accumulation cancel heavily) at d = 16, 50 and 128."""
import numpy as np
import pytest

import fastdec_b200.datasets as ds

pytestmark = pytest.mark.gpu


def _data(kind, d, n, seed):
    if kind == "offset":
        rng = np.random.default_rng(seed)
        return (1000.0 + 0.01 * rng.standard_normal((d, n))).astype(np.float32)
    if d == 16:
        return ds.gmm_isotropic(n=n, d=16, seed=seed)
    if d == 50:
        return ds.embedding_cloud(n=n, d=50, seed=seed)
    return ds.scale_out(n=n, d=d, seed=seed)


@pytest.mark.parametrize("kind", ["cloud", "offset"])
@pytest.mark.parametrize("d", [16, 50, 128])
def test_filter_margin_covers_the_tf32_accumulation(fdb, oracle, kind, d):
    n, k = 1500, 10
    x = _data(kind, d, n, seed=d + (7 if kind == "offset" else 0))
    d2 = oracle.pair_d2_all(x)                               # the reference's exact FP32 d2
    np.fill_diagonal(d2, np.inf)
    thr = np.sort(d2, axis=1)[:, k - 1].astype(np.float32)  # each point's exact k-th neighbour d2
    acc, V, A, B = fdb.debug_tc_filter(x, thr)
    kp = A.shape[1]
    # 1. the filter keeps every admissible candidate
    adm = d2 <= thr[:, None]
    assert adm.sum() >= n * k
    missed = adm & ~(acc < 0)
    assert not missed.any(), f"{missed.sum()} admissible pairs with a non-negative accumulator"
    # 2. the accumulation error against the model (2^-20 of the summed term magnitudes per K-step of 8)
    A64, B64 = A.astype(np.float64), B.astype(np.float64)
    exact = A64 @ B64.T
    mag = np.abs(A64) @ np.abs(B64).T
    err = np.abs(acc.astype(np.float64) - exact)
    model = (kp / 8) * 2.0 ** -20 * mag
    ratio = float((err / model).max())
    kept = float((acc < 0).mean())
    print(f"\n[tc filter audit] {kind} d={d} K={kp}: max accumulation error / model = {ratio:.4f}; "
          f"pairs kept {kept:.4%}; admissible {adm.mean():.4%}")
    assert ratio < 1.0
    # 3. the engine's lists on the same data, bit for bit
    dist, idx, st = fdb.knn(x, k, engine="tcgen05")
    od, oi = oracle.knn(x, k)
    assert st["engine_used"] == 2
    assert np.array_equal(idx, oi) and np.array_equal(dist.view(np.uint32), od.view(np.uint32))
