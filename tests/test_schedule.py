"""The tcgen05 tile schedule, checked on the host: tests/schedule_cover.cpp includes the same header the
tile kernel's roles walk (csrc/knn_tc_schedule.h) and, for block counts 1-70 and up to 2048, random
round partitions, 1/3/148 CTAs and 1-8 shards, checks that the symmetric schedule covers every
unordered block pair once, that a shard's ordered schedule covers every ordered pair of its rows once
and nothing else, and that the MMA issuer's per-item tile count matches the tiles the other roles
accept. No GPU needed."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs a host C++ compiler")
def test_tile_schedule_covers_every_pair_exactly_once(tmp_path):
    exe = tmp_path / "schedule_cover"
    subprocess.run(["g++", "-std=c++17", "-O2", "-I", str(ROOT / "symwarp-fastdec_b200" / "csrc"),
                    str(ROOT / "tests" / "schedule_cover.cpp"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.startswith("ok"), out.stdout + out.stderr
    assert int(out.stdout.split()[1]) > 9000
