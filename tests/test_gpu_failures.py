"""Failure paths that fault or hang no GPU: a device allocation that cannot be satisfied is reported
as FDB200_ENOMEM with a message, and a bounded wait of the tcgen05 kernel that runs out (a row copy
that is withheld on purpose, so nothing completes the barrier) ends the launch with an error code that
the host reports as FDB200_EINTERNAL. After either, the next call on the same device is exact."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_candidate_buffer_too_large_reports_enomem_and_recovers(fdb, oracle):
    # 1.6M points x 16,000 candidate slots x 8 bytes = 205 GB: more than a B200 holds, so the
    # candidate buffer's cudaMalloc fails before any kernel is launched
    x = np.zeros((1, 1_600_000), np.float32)
    with pytest.raises(fdb.FastDecError) as e:
        fdb.knn(x, 4, cand_capacity=16_000)
    assert e.value.code == -3   # FDB200_ENOMEM
    assert "cudaMalloc" in str(e.value)
    # the same device keeps working
    rng = np.random.default_rng(3)
    y = rng.uniform(-1, 1, (8, 2000)).astype(np.float32)
    d, i, _ = fdb.knn(y, 10)
    od, oi = oracle.knn(y, 10)
    assert np.array_equal(i, oi) and np.array_equal(d, od)


def test_tile_kernel_bounded_wait_runs_out_and_the_device_stays_usable(fdb, oracle, monkeypatch):
    """FDB200_FAULT_INJECT=withhold_row_copy: every CTA's first row stage is never filled, so the MMA
    issuer's wait for it runs out after about a second. The kernel records an error code, its other
    roles see the abort flag, copies in flight are drained and TMEM is freed; the rest of the queued
    rounds skip themselves, and the host reports FDB200_EINTERNAL. The next call is exact again."""
    rng = np.random.default_rng(5)
    x = rng.uniform(-1, 1, (16, 3000)).astype(np.float32)
    monkeypatch.setenv("FDB200_FAULT_INJECT", "withhold_row_copy")
    with pytest.raises(fdb.FastDecError) as e:
        fdb.knn(x, 10, engine="tcgen05")
    assert e.value.code == -6 and "bounded wait" in str(e.value)   # FDB200_EINTERNAL
    monkeypatch.delenv("FDB200_FAULT_INJECT")
    d, i, st = fdb.knn(x, 10, engine="tcgen05")
    od, oi = oracle.knn(x, 10)
    assert st["engine_used"] == 2
    assert np.array_equal(i, oi) and np.array_equal(d, od)
