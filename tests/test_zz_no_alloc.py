"""fdb200_density_noalloc through the C ABI: the same densities and mean as fdb200_density on two
calls in a row, no device memory obtained during a call, and a clear refusal above its fixed size.
(The file name sorts last so that it also runs after every other test in one session.)"""
import ctypes

import numpy as np
import pytest

import fastdec_b200 as fdb

MAX_POINTS = 4194304   # FDB200_NOALLOC_MAX_POINTS


def _knn_like(n, k, seed):
    """rank-major (k x n) ascending distances with ties and zeros, like a kNN graph"""
    rng = np.random.default_rng(seed)
    d = np.sort(rng.random((n, k), dtype=np.float32) * np.float32(3.0), axis=1)
    d[::97, 0] = 0.0
    d[::89, 1:4] = d[::89, 1:2]
    return np.ascontiguousarray(d.T)


@pytest.mark.gpu
@pytest.mark.parametrize("kernel", ["laplacian", "gaussian"])
def test_density_noalloc_matches_density_on_two_calls(kernel):
    import torch
    lib = fdb.lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    for call, (n, k) in enumerate([(300_001, 24), (65_536, 45)]):
        dist = _knn_like(n, k, seed=31 + call)
        want_den, want_mean = fdb.density(dist, density=kernel)
        d_dev = torch.from_numpy(dist).to(dev)
        den = torch.full((n,), -1.0, dtype=torch.float32, device=dev)
        mean = torch.zeros(1, dtype=torch.float64, device=dev)
        o = fdb.make_opts(density=kernel, stream=stream.cuda_stream)
        torch.cuda.synchronize(dev)
        free0 = torch.cuda.mem_get_info(dev)[0]
        rc = lib.fdb200_density_noalloc(fdb._ptr(d_dev), n, k, ctypes.byref(o), fdb._ptr(den), fdb._ptr(mean))
        assert rc == 0, lib.fdb200_last_error().decode()
        torch.cuda.synchronize(dev)
        free1 = torch.cuda.mem_get_info(dev)[0]
        got_mean = float(mean.item())
        np.testing.assert_allclose(got_mean, want_mean, rtol=1e-12, atol=0)
        np.testing.assert_allclose(den.cpu().numpy(), want_den, rtol=1e-6, atol=1e-30)
        if call == 1:
            # the one-time address lookup happened on the first call; later calls obtain no memory
            assert free1 == free0


@pytest.mark.gpu
def test_density_noalloc_rejects_more_points_than_its_scratch():
    import torch
    lib = fdb.lib()
    dev = torch.device("cuda", 0)
    n = MAX_POINTS + 1
    # buffers of the full size, so that even a missing check could not read or write out of bounds
    dist = torch.ones(n, dtype=torch.float32, device=dev)
    den = torch.zeros(n, dtype=torch.float32, device=dev)
    mean = torch.zeros(1, dtype=torch.float64, device=dev)
    o = fdb.make_opts()
    rc = lib.fdb200_density_noalloc(fdb._ptr(dist), n, 1, ctypes.byref(o), fdb._ptr(den), fdb._ptr(mean))
    torch.cuda.synchronize(dev)
    assert rc == -1   # FDB200_EINVAL
    assert float(den.abs().max().item()) == 0.0   # nothing was launched
    assert "exceeds the fixed scratch" in lib.fdb200_last_error().decode()
