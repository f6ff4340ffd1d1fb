"""Generate the committed golden fixtures from the reference tree (run in the build container).

Writes, next to this script:
  spiral.f32          spiral.csv parsed with the C library's strtof (as helper.cpp:9-63 reads it),
                      row-major float32 (312 x 2)
  known_answers.json  the reference's published/known answers for this path:
                        * spiral k=7 c=3 FP32 centers              README.md:105-122
                        * DC-reduction known case                  symwarp_unit_test.cu:21-59
                        * DC-reduction no-denser-point sentinels   symwarp_unit_test.cu:61-88
                        * two-blob Fit (points, k, c)              symwarp_unit_test.cu:90-144
The arrays are extracted from the reference files as text, so a change upstream shows up here.
Usage: python tests/golden/make_golden.py [/path/to/reference]
(default: $FASTDEC_REF, else a `reference/` directory beside this repository)
"""
import ctypes
import json
import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def c_floats(text):
    return [float(v.strip().rstrip("f")) for v in text.split(",") if v.strip()]


def c_ints(text):
    return [int(v.strip()) for v in text.split(",") if v.strip()]


def array_literal(src, name, start=0):
    m = re.search(r"%s\s*\[[^\]]*\]\s*=\s*\{([^}]*)\}" % re.escape(name), src[start:], re.S)
    if not m:
        raise SystemExit(f"array {name} not found")
    return m.group(1), start + m.end()


def main():
    import os
    default = os.environ.get("FASTDEC_REF") or str(HERE.parent.parent.parent / "reference")
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else default)
    libc = ctypes.CDLL(None)
    libc.strtof.restype = ctypes.c_float
    libc.strtof.argtypes = [ctypes.c_char_p, ctypes.c_void_p]

    rows = []
    for line in (ref / "spiral.csv").read_text().splitlines():
        if line.strip():
            rows.append([libc.strtof(tok.encode(), None) for tok in line.split(",")])
    spiral = np.asarray(rows, dtype=np.float32)
    spiral.tofile(HERE / "spiral.f32")

    readme = (ref / "README.md").read_text()
    m = re.search(r"Spiral \(FP32, FDS off\).*?Expected centers:\s*```text\s*\[([0-9,\s]+)\]", readme, re.S)
    spiral_centers = c_ints(m.group(1))

    src = (ref / "symwarp_unit_test.cu").read_text()
    t1 = src.index("test_dc_reduction_known_case()")
    ds1, p = array_literal(src, "ds_host", t1)
    den1, p = array_literal(src, "ds_den_host", p)
    cores1, p = array_literal(src, "core_indices_host", p)
    exp1, p = array_literal(src, "expected_idx", p)
    cen1 = int(re.search(r"center_indices_host\[0\]\s*!=\s*(\d+)", src[p:]).group(1))

    t2 = src.index("test_dc_reduction_no_cdh_case()")
    ds2, p = array_literal(src, "ds_host", t2)
    den2, p = array_literal(src, "ds_den_host", p)
    cores2, p = array_literal(src, "core_indices_host", p)
    m2 = re.search(r"cdh_index_host\[0\]\s*!=\s*(-?\d+)\s*\|\|\s*center_indices_host\[0\]\s*!=\s*(-?\d+)", src[p:])

    t3 = src.index("test_fit_small_dataset()")
    rm3, p = array_literal(src, "row_major", t3)
    km = re.search(r"SymWarpFastDEC model\((\d+),\s*(\d+)", src[p:])

    known = {
        "spiral": {"source": "README.md:105-122", "k": 7, "c": 3, "centers": spiral_centers,
                   "shape": list(spiral.shape)},
        "dc_known_case": {"source": "symwarp_unit_test.cu:21-59", "points_1d": c_floats(ds1),
                          "densities": c_floats(den1), "cores": c_ints(cores1), "num_centers": 1,
                          "expected_parents": c_ints(exp1), "expected_center": cen1},
        "dc_no_denser": {"source": "symwarp_unit_test.cu:61-88", "points_1d": c_floats(ds2),
                         "densities": c_floats(den2), "cores": c_ints(cores2), "num_centers": 1,
                         "expected_parents": [int(m2.group(1))],
                         "expected_center": int(m2.group(2))},
        "two_blob_fit": {"source": "symwarp_unit_test.cu:90-144", "row_major": c_floats(rm3),
                         "dims": 2, "k": int(km.group(1)), "c": int(km.group(2)),
                         "left_count": 4},
    }
    (HERE / "known_answers.json").write_text(json.dumps(known, indent=1) + "\n")
    print("wrote", HERE / "spiral.f32", HERE / "known_answers.json")


if __name__ == "__main__":
    main()
