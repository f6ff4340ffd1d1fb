"""ctypes bindings for the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg import this
module. It wraps oracle/libfastdec_oracle.so (a plain-C restatement of the reference's Fit, see
fastdec_oracle.h for the reference lines each function follows) and, when it was built,
oracle/_ref/libfastdec_ref*.so (the reference's own host stages, fastdecbase.cpp + helper.cpp,
compiled from the reference tree, with CPU stand-ins for its GPU calls).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")

_lib = None
_ref = {}


def reference_tree():
    """The reference checkout: $FASTDEC_REF, else a `reference/` directory beside this repository;
    None when neither holds the reference sources (as on a GPU box, which only uses the prebuilt
    oracle/_ref files)."""
    for cand in (os.environ.get("FASTDEC_REF"), str(HERE.parent.parent / "reference")):
        if cand and (Path(cand) / "fastdecbase.cpp").exists():
            return Path(cand)
    return None


def build():
    """Compile the oracle library (and oracle/_ref when the reference tree is present)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    ref = reference_tree()
    if ref is not None:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={ref}"], check=True)


def lib():
    global _lib
    if _lib is None:
        path = HERE / "libfastdec_oracle.so"
        if not path.exists():
            build()
        L = ctypes.CDLL(str(path))
        c_int, c_double = ctypes.c_int, ctypes.c_double
        L.or_norms.argtypes = [_f32p, c_int, c_int, _f32p]
        L.or_pair_d2.argtypes = [_f32p, c_int, c_int, _f32p, c_int, c_int]
        L.or_pair_d2.restype = ctypes.c_float
        L.or_knn.argtypes = [_f32p, c_int, c_int, c_int, c_int, _f32p, _i32p]
        L.or_pair_d2_all.argtypes = [_f32p, c_int, c_int, _f32p]
        L.or_knn_rows.argtypes = [_f32p, c_int, c_int, c_int, _i32p, c_int, c_int, _f32p, _i32p]
        L.or_mean_knn_dist.argtypes = [_f32p, c_int, c_int]
        L.or_mean_knn_dist.restype = c_double
        L.or_density.argtypes = [_f32p, c_int, c_int, c_int, _f32p]
        L.or_dc_detection.argtypes = [_i32p, _f32p, c_int, c_int, _i32p, _i32p]
        L.or_dc_reduction.argtypes = [_f32p, c_int, c_int, _f32p, _i32p, c_int, c_int, c_int,
                                      _i32p, _f32p, _i32p, _i32p]
        L.or_select_centers.argtypes = [_f32p, _f32p, _i32p, _i32p, c_int, c_int, _i32p]
        L.or_final_cluster.argtypes = [_f32p, _i32p, c_int, _i32p, c_int, _i32p]
        L.or_fit.argtypes = [_f32p, c_int, c_int, c_int, c_int, c_int, c_int, _i32p, _i32p,
                             ctypes.POINTER(c_int), ctypes.POINTER(c_int)]
        _lib = L
    return _lib


def threads():
    return max(1, os.cpu_count() or 1)


def _dm(x_dm):
    x = np.ascontiguousarray(x_dm, dtype=np.float32)
    assert x.ndim == 2
    return x


def norms(x_dm):
    x = _dm(x_dm)
    d, n = x.shape
    out = np.empty(n, np.float32)
    lib().or_norms(x, n, d, out)
    return out


def pair_d2_all(x_dm):
    """(n, n) squared distances of every ordered pair as the reference computes them (fmaf-chain dot,
    symtriknnfds.h:23-26). Small n only."""
    x = _dm(x_dm)
    d, n = x.shape
    out = np.empty((n, n), np.float32)
    lib().or_pair_d2_all(x, n, d, out)
    return out


def knn(x_dm, k, nthreads=None):
    """Exact self-kNN. Returns rank-major (k, n) sqrt'd distances and indices."""
    x = _dm(x_dm)
    d, n = x.shape
    dist = np.empty((k, n), np.float32)
    idx = np.empty((k, n), np.int32)
    rc = lib().or_knn(x, n, d, k, nthreads or threads(), dist, idx)
    if rc != 0:
        raise ValueError(f"or_knn rejected n={n} d={d} k={k}")
    return dist, idx


def knn_rows(x_dm, k, rows, nthreads=None):
    """Exact kNN of selected rows: (len(rows), k) squared distances and indices."""
    x = _dm(x_dm)
    d, n = x.shape
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    d2 = np.empty((len(rows), k), np.float32)
    idx = np.empty((len(rows), k), np.int32)
    rc = lib().or_knn_rows(x, n, d, k, rows, len(rows), nthreads or threads(), d2, idx)
    if rc != 0:
        raise ValueError("or_knn_rows rejected its arguments")
    return d2, idx


def mean_knn_dist(dist_rm, k=None):
    dist = np.ascontiguousarray(dist_rm, dtype=np.float32)
    kk, n = dist.shape
    return lib().or_mean_knn_dist(dist, n, k or kk)


def density(dist_rm, k=None, gaussian=False):
    dist = np.ascontiguousarray(dist_rm, dtype=np.float32)
    kk, n = dist.shape
    out = np.empty(n, np.float32)
    lib().or_density(dist, n, k or kk, int(bool(gaussian)), out)
    return out


def dc_detection(idx_rm, den, k=None):
    idx = np.ascontiguousarray(idx_rm, dtype=np.int32)
    kk, n = idx.shape
    parent = np.empty(n, np.int32)
    cores = np.empty(n, np.int32)
    nc = lib().or_dc_detection(idx, np.ascontiguousarray(den, np.float32), n, k or kk, parent, cores)
    return parent, cores[:nc].copy()


def dc_reduction(x_dm, den, cores, num_centers, nthreads=None):
    """Returns (core_parent, delta, rank, centers) as in warp_parallel_dc_reduction_cuda."""
    x = _dm(x_dm)
    d, n = x.shape
    cores = np.ascontiguousarray(cores, np.int32)
    nc = len(cores)
    cp = np.empty(nc, np.int32)
    dl = np.empty(nc, np.float32)
    rk = np.empty(nc, np.int32)
    ctr = np.empty(num_centers, np.int32)
    rc = lib().or_dc_reduction(x, n, d, np.ascontiguousarray(den, np.float32), cores, nc,
                               num_centers, nthreads or threads(), cp, dl, rk, ctr)
    if rc != 0:
        raise ValueError("or_dc_reduction rejected its arguments")
    return cp, dl, rk, ctr


def select_centers(core_den, delta, rank, core_idx, num_centers):
    out = np.empty(num_centers, np.int32)
    lib().or_select_centers(np.ascontiguousarray(core_den, np.float32),
                            np.ascontiguousarray(delta, np.float32),
                            np.ascontiguousarray(rank, np.int32),
                            np.ascontiguousarray(core_idx, np.int32), len(core_idx), num_centers, out)
    return out


def final_cluster(den, parent, centers):
    den = np.ascontiguousarray(den, np.float32)
    n = den.shape[0]
    labels = np.empty(n, np.int32)
    centers = np.ascontiguousarray(centers, np.int32)
    lib().or_final_cluster(den, np.ascontiguousarray(parent, np.int32), n, centers, len(centers), labels)
    return labels


def fit(x_dm, k, c, gaussian=False, nthreads=None):
    """Whole fit. Returns dict(centers, labels, final_k, num_cores)."""
    x = _dm(x_dm)
    d, n = x.shape
    centers = np.empty(c, np.int32)
    labels = np.empty(n, np.int32)
    fk, nc = ctypes.c_int(0), ctypes.c_int(0)
    rc = lib().or_fit(x, n, d, k, c, int(bool(gaussian)), nthreads or threads(), centers, labels,
                      ctypes.byref(fk), ctypes.byref(nc))
    if rc == -2:
        raise RuntimeError("Fit: not enough core points")
    if rc != 0:
        raise ValueError(f"or_fit rejected n={n} d={d} k={k} c={c}")
    return dict(centers=centers, labels=labels, final_k=fk.value, num_cores=nc.value)


# ---------------- the reference's own host stages (oracle/_ref) ----------------

def ref_available(gaussian=False):
    name = "libfastdec_ref_gauss.so" if gaussian else "libfastdec_ref.so"
    return (HERE / "_ref" / name).exists()


def _ref_lib(gaussian):
    name = "libfastdec_ref_gauss.so" if gaussian else "libfastdec_ref.so"
    if name not in _ref:
        L = ctypes.CDLL(str(HERE / "_ref" / name))
        ip = ctypes.POINTER(ctypes.c_int)
        tail = [_i32p, _i32p, _f32p, _i32p, _i32p, ip, ip, ctypes.c_char_p, ctypes.c_int]
        L.ref_fit.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int] + tail
        L.ref_fit_from_knn.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       _f32p, _i32p] + tail
        _ref[name] = L
    return _ref[name]


def _ref_call(fn, x, c, *lead):
    d, n = x.shape
    centers = np.full(c, -1, np.int32)
    labels = np.empty(n, np.int32)
    den = np.empty(n, np.float32)
    parents = np.empty(n, np.int32)
    cores = np.empty(n, np.int32)
    nc, fk = ctypes.c_int(0), ctypes.c_int(0)
    err = ctypes.create_string_buffer(256)
    rc = fn(*lead, centers, labels, den, parents, cores, ctypes.byref(nc), ctypes.byref(fk), err, 256)
    if rc != 0:
        raise RuntimeError(err.value.decode() or "ref_fit failed")
    return dict(centers=centers, labels=labels, densities=den, parents=parents,
                cores=cores[:nc.value].copy(), num_cores=nc.value, final_k=fk.value)


def ref_fit(x_dm, k, c, gaussian=False):
    """FastDECBase::Fit from the reference sources (CPU kNN and DC reduction stand-ins)."""
    x = _dm(x_dm)
    d, n = x.shape
    return _ref_call(_ref_lib(gaussian).ref_fit, x, c, x, n, d, k, c)


def ref_fit_from_knn(x_dm, knn_dist_rm, knn_idx_rm, c, gaussian=False):
    """FastDECBase::Fit from the reference sources on a given kNN graph (rank-major (k, n) distances
    and indices, e.g. the GPU engine's): the reference's own density, DC detection with k-halving,
    final clustering, and the oracle's DC reduction. `parents` is the reference's m_cdh_ids after the
    fit (detection parents, with the cores' DC-reduction parents written in)."""
    x = _dm(x_dm)
    d, n = x.shape
    dist = np.ascontiguousarray(knn_dist_rm, dtype=np.float32)
    idx = np.ascontiguousarray(knn_idx_rm, dtype=np.int32)
    k = dist.shape[0]
    assert dist.shape == (k, n) and idx.shape == (k, n)
    return _ref_call(_ref_lib(gaussian).ref_fit_from_knn, x, c, x, n, d, k, c, dist, idx)
