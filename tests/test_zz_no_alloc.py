"""fdb200_density_noalloc through the C ABI: the same densities and mean as fdb200_density, bit for
bit, on two calls in a row; no device memory obtained by a call after the first on a device, also
when the entry point is the first thing a fresh process calls; and a clear refusal above its fixed
size. (The file name sorts last so that it also runs after every other test in one session.)"""
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
        # the same kernels as fdb200_density: the mean and every density are bit-identical
        assert float(mean.item()) == want_mean
        assert np.array_equal(den.cpu().numpy().view(np.uint32), want_den.view(np.uint32))
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


_FIRST_CALL_SCRIPT = r"""
import ctypes, json, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
import fastdec_b200 as fdb
n, k = 200_003, 32
rng = np.random.default_rng(7)
dist = np.ascontiguousarray(np.sort(rng.random((n, k), dtype=np.float32) * np.float32(2.0), axis=1).T)
dev = torch.device("cuda", 0)
d_dev = torch.from_numpy(dist).to(dev)
outs = [(torch.full((n,), -1.0, dtype=torch.float32, device=dev), torch.zeros(1, dtype=torch.float64, device=dev))
        for _ in range(3)]
lib = fdb.lib()
o = fdb.make_opts()
torch.cuda.synchronize(dev)
free = [torch.cuda.mem_get_info(dev)[0]]
for den, mean in outs:
    # the library's first call in this process: nothing else of it has run or loaded kernels yet
    rc = lib.fdb200_density_noalloc(fdb._ptr(d_dev), n, k, ctypes.byref(o), fdb._ptr(den), fdb._ptr(mean))
    assert rc == 0, lib.fdb200_last_error().decode()
    torch.cuda.synchronize(dev)
    free.append(torch.cuda.mem_get_info(dev)[0])
want_den, want_mean = fdb.density(dist)
same = all(np.array_equal(den.cpu().numpy().view(np.uint32), want_den.view(np.uint32)) and
           float(mean.item()) == want_mean for den, mean in outs)
print("RESULT " + json.dumps({"free": free, "same": bool(same)}))
"""


@pytest.mark.gpu
def test_density_noalloc_as_the_first_call_of_a_fresh_process():
    """A process whose first library call is fdb200_density_noalloc: the first call's one-time set-up
    (the scratch address and the kernels' code) may obtain memory, the second and third obtain none,
    and all three give fdb200_density's bits."""
    import json
    import subprocess
    import sys
    from pathlib import Path
    pkg = Path(__file__).resolve().parent.parent / "symwarp-fastdec_b200"
    r = subprocess.run([sys.executable, "-c", _FIRST_CALL_SCRIPT, str(pkg)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads([l for l in r.stdout.splitlines() if l.startswith("RESULT ")][-1][len("RESULT "):])
    free = out["free"]
    assert free[2] == free[1] and free[3] == free[2], free
    assert out["same"]
