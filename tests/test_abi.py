"""The C-ABI library loads without a GPU and exports every function include/*.h declares."""
import ctypes
import re
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(fdb200_\w+)\s*\(", text, re.M))
    return names


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ["fdb200_knn", "fdb200_fit", "fdb200_dc_reduction", "fdb200_density",
                     "fdb200_dc_detection", "fdb200_final_cluster", "fdb200_last_error"]:
        assert required in names


def test_library_exports_every_declared_symbol(fdb):
    lib = fdb.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(fdb.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (fdb200_\w+)", out))
    assert declared_functions() <= exported
    assert set(fdb.EXPORTS) <= exported


def test_opts_init_and_version_need_no_gpu(fdb):
    lib = fdb.lib()
    o = fdb.Opts()
    assert lib.fdb200_opts_init(ctypes.byref(o)) == 0
    assert o.struct_size == ctypes.sizeof(fdb.Opts)
    assert o.shard_count == 1 and o.precision == fdb.FP32
    assert lib.fdb200_abi_version() == 3
    assert ctypes.sizeof(fdb.Stats) == 8 * 7 + 8 * 2 + 4 * 6 + 4 * 6  # matches FdB200Stats (120 bytes)


def test_python_package_has_no_cpu_fallback(fdb):
    import inspect
    src = inspect.getsource(fdb)
    assert "oracle" not in src
