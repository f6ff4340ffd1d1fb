"""bench.py's reference arm on CPU: the JSON line the driver reads (keys, units, the reference-arm
extras) for a small configuration, and the silent exit of ranks other than 0 under torchrun."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                       env=env, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout


def test_reference_arm_prints_the_contract_line():
    out = _run(["--impl", "reference", "--config", "gmm100k", "--n", "4000", "--steps", "2", "--warmup", "1",
                "--cpu-seconds", "0.2"])
    line = json.loads(out.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "fit_distance_pairs_per_s" and line["unit"] == "pairs/s"
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert (line["n_gpus"], line["steps"], line["warmup"]) == (1, 2, 1)
    assert line["higher_is_better"] is True and line["scaling"] in ("weak", "strong")
    assert line["vs_baseline"] is None   # only the headline shape has a published number
    assert line["config"]["workload"].startswith("gmm100k 4,000 x 16")
    cpu = line["cpu_baseline"]
    assert cpu["value"] == line["value"] and cpu["unit"] == "pairs/s"
    assert cpu["kind"] in ("reference", "port") and cpu["cores"] >= 1 and cpu["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "pairs/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_silently():
    out = _run(["--impl", "reference", "--config", "gmm100k", "--n", "2000", "--steps", "1", "--warmup", "0"],
               {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert out.strip() == ""
