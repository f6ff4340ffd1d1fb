"""Failure paths made on the host, none of which faults or hangs the GPU: a device allocation that
cannot be satisfied is reported as FDB200_ENOMEM with a message, and the library stays usable for
the next call on the same device (the workspace re-grows)."""
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
