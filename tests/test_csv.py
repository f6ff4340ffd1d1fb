"""The parallel CSV reader (fdb200_csv_shape / fdb200_read_csv) against the reference's own parser,
read_data (helper.cpp:30-63, compiled from the reference sources into oracle/_ref by the oracle build),
and against numpy; no GPU is involved."""
import ctypes
from pathlib import Path

import numpy as np
import pytest

import fastdec_b200 as fdb

REF_LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libfastdec_ref.so"


def _write(path, rows, fmt):
    with open(path, "w") as f:
        for r in rows:
            f.write(",".join(fmt(v) for v in r) + "\n")


def _ref_read(path, n, d):
    """row-major (n, d) float32 from the reference's read_data"""
    lib = ctypes.CDLL(str(REF_LIB))
    fn = getattr(lib, "_Z9read_dataPKcPfii")   # read_data(const char*, float*, int, int)
    out = np.zeros((n, d), np.float32)
    fn(str(path).encode(), out.ctypes.data_as(ctypes.c_void_p), n, d)
    return out


FORMATS = {
    "shortest": lambda v: repr(float(np.float32(v))),
    "fixed6": lambda v: f"{v:.6f}",
    "exp9": lambda v: f"{v:.9e}",
    "g17": lambda v: f"{v:.17g}",
}


@pytest.mark.parametrize("fmt", sorted(FORMATS))
def test_read_csv_matches_the_reference_parser(tmp_path, fmt):
    rng = np.random.default_rng(7)
    n, d = 2345, 13
    x = (rng.standard_normal((n, d)) * 10.0 ** rng.integers(-6, 6, size=(n, d))).astype(np.float64)
    x[0, 0] = 0.0
    x[1, 1] = -0.0
    p = tmp_path / "data.csv"
    _write(p, x, FORMATS[fmt])
    got = fdb.read_csv(p)
    assert got.shape == (d, n) and got.dtype == np.float32
    if REF_LIB.exists():
        ref = _ref_read(p, n, d)
        assert np.array_equal(got.T.view(np.uint32), ref.view(np.uint32))   # bit for bit, signed zeros too
    want = np.array([[np.float32(float(FORMATS[fmt](v))) for v in r] for r in x[:50]], np.float32)
    assert np.array_equal(got.T[:50].view(np.uint32), want.view(np.uint32))


def test_read_csv_threads_and_layout(tmp_path):
    rng = np.random.default_rng(3)
    x = rng.random((1001, 7)).astype(np.float32)
    p = tmp_path / "d.csv"
    _write(p, x, lambda v: repr(float(v)))
    a = fdb.read_csv(p, threads=1)
    b = fdb.read_csv(p, threads=13)
    assert np.array_equal(a, b)
    assert np.array_equal(a, x.T)   # dim-major: element (t, i) is point i's coordinate t


def test_read_csv_tolerates_crlf_spaces_and_missing_final_newline(tmp_path):
    p = tmp_path / "w.csv"
    p.write_bytes(b"1, 2 ,+3\r\n\r\n4,5,6e-1\r\n-7 ,8.5,9")
    x = fdb.read_csv(p)
    assert np.array_equal(x.T, np.array([[1, 2, 3], [4, 5, 0.6], [-7, 8.5, 9]], np.float32))


def test_read_csv_rejects_ragged_rows_and_missing_files(tmp_path):
    p = tmp_path / "r.csv"
    p.write_text("1,2,3\n4,5\n")
    with pytest.raises(fdb.FastDecError, match="line 2"):
        fdb.read_csv(p)
    with pytest.raises(fdb.FastDecError, match="cannot read"):
        fdb.read_csv(tmp_path / "missing.csv")


def test_write_csv_reads_back_exactly_with_the_reference_parser(tmp_path):
    """fdb200_write_csv: shortest round-trip text, so both the reference's read_data and the library's
    reader recover every float32 bit (subnormals, signed zero and extreme exponents included)."""
    rng = np.random.default_rng(11)
    n, d = 3001, 9
    x = (rng.standard_normal((d, n)) * 10.0 ** rng.integers(-30, 30, size=(d, n))).astype(np.float32)
    x[0, :6] = [0.0, -0.0, 1e-45, -3.4028235e38, 1.1754944e-38, np.float32(0.1)]
    p = tmp_path / "w.csv"
    for threads in (1, 5):
        fdb.write_csv(p, x, threads=threads)
        got = fdb.read_csv(p)
        assert np.array_equal(got.view(np.uint32), x.view(np.uint32))
    if REF_LIB.exists():
        ref = _ref_read(p, n, d)
        assert np.array_equal(ref.view(np.uint32), x.T.view(np.uint32))
    lines = p.read_text().splitlines()
    # line i is point i (column i of the dim-major array): point 1 starts with -0
    assert len(lines) == n and lines[1].split(",")[0] == "-0" and lines[0].split(",")[0] == "0"
