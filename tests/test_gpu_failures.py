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


_INJECT_SCRIPT = r"""
import sys, json
import numpy as np
sys.path[:0] = sys.argv[1:3]
import fastdec_b200 as fdb, oracle
rng = np.random.default_rng(5)
x = rng.uniform(-1, 1, (16, 3000)).astype(np.float32)
out = {}
try:
    fdb.knn(x, 10, engine="tcgen05")
    out["first"] = "ok"
except fdb.FastDecError as e:
    out["first"] = [e.code, str(e)]
d, i, st = fdb.knn(x, 10, engine="tcgen05")
od, oi = oracle.knn(x, 10)
out["engine"] = st["engine_used"]
out["exact"] = bool(np.array_equal(i, oi) and np.array_equal(d, od))
print("RESULT " + json.dumps(out))
"""


def test_tile_kernel_bounded_wait_runs_out_and_the_device_stays_usable():
    """FDB200_FAULT_INJECT=withhold_row_copy (read once per process): the first tcgen05 launch of the
    process never fills every CTA's first row stage, so the MMA issuer's wait for it runs out after
    about a second. The kernel records an error code, its other roles see the abort flag, copies in
    flight are drained and TMEM is freed; the rest of the queued rounds skip themselves, and the host
    reports FDB200_EINTERNAL. The next call in the same process is exact. Run in a child process so
    the variable is seen at the process's first launch."""
    import json
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    env = dict(os.environ, FDB200_FAULT_INJECT="withhold_row_copy")
    r = subprocess.run([sys.executable, "-c", _INJECT_SCRIPT, str(root / "symwarp-fastdec_b200"), str(root / "oracle")],
                       env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT ")][-1]
    out = json.loads(line[len("RESULT "):])
    code, msg = out["first"]
    assert code == -6 and "bounded wait" in msg, msg    # FDB200_EINTERNAL
    assert "unsafe" not in msg                            # the drain of the copies in flight finished
    assert out["engine"] == 2 and out["exact"]
