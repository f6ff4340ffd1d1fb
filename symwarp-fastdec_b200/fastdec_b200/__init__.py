"""Python bindings for the B200 FastDEC engine (libfastdec_b200.so, C ABI in include/fastdec_b200.h).

The engine is native code; this module only loads it with ctypes and converts numpy arrays or
torch CUDA tensors to pointers. There is no fallback: if the shared library is missing the import
of any entry point raises. Layouts follow the reference (cyberbull66/symwarp-fastdec): datasets
are dim-major (d, n) float32 (test.cpp:110-115); kNN results are rank-major (k, n)
(symtriknncuda.h:11-12).

    B200FastDEC(k, c, name, gpu).Fit(data_dm, n, d)   # mirrors SymWarpFullGpuFastDEC / FastDECBase
    fit(data_dm, k, c)                                 # -> dict(centers, labels, densities, stats)
    knn(data_dm, k)                                    # -> (dist (k, n), idx (k, n))
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

PKG_ROOT = Path(__file__).resolve().parent.parent          # symwarp-fastdec_b200/
LIB_PATH = PKG_ROOT / "lib" / "libfastdec_b200.so"
CSRC = PKG_ROOT / "csrc"

FP32, TF32 = 0, 1
LAPLACIAN, GAUSSIAN = 0, 1
ENGINE_AUTO, ENGINE_SIMT, ENGINE_TCGEN05 = 0, 1, 2
_PRECISION = {"fp32": FP32, "tf32": TF32}
_DENSITY = {"laplacian": LAPLACIAN, "gaussian": GAUSSIAN}
_ENGINE = {"auto": ENGINE_AUTO, "simt": ENGINE_SIMT, "tcgen05": ENGINE_TCGEN05}

ERRORS = {0: "ok", -1: "EINVAL", -2: "ECUDA", -3: "ENOMEM", -4: "ECORES", -5: "ECYCLE", -6: "EINTERNAL"}


class FastDecError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


# fdb200_round_hook(ctx, kind, dev_ptr, count, stream): kind HOOK_FLAGS = int32 flags to combine by MAX,
# HOOK_THRESHOLDS = packed uint64 keys to combine by unsigned MIN, over all shards, on `stream`
ROUND_HOOK = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong,
                              ctypes.c_void_p)
HOOK_FLAGS, HOOK_THRESHOLDS = 0, 1


class Opts(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_int), ("device", ctypes.c_int), ("precision", ctypes.c_int),
                ("density_kernel", ctypes.c_int), ("engine", ctypes.c_int),
                ("inputs_on_device", ctypes.c_int), ("outputs_on_device", ctypes.c_int),
                ("shard_rank", ctypes.c_int), ("shard_count", ctypes.c_int),
                ("cand_capacity", ctypes.c_int), ("stream", ctypes.c_void_p),
                ("shard_block_lo", ctypes.c_int), ("shard_block_hi", ctypes.c_int),
                ("round_hook", ROUND_HOOK), ("round_hook_ctx", ctypes.c_void_p)]


class Stats(ctypes.Structure):
    _fields_ = [("total_ms", ctypes.c_double), ("upload_ms", ctypes.c_double), ("knn_ms", ctypes.c_double),
                ("density_ms", ctypes.c_double), ("dc_ms", ctypes.c_double), ("labels_ms", ctypes.c_double),
                ("knn_tile_ms", ctypes.c_double), ("pairs", ctypes.c_longlong),
                ("candidates", ctypes.c_longlong), ("rounds", ctypes.c_int),
                ("overflow_reruns", ctypes.c_int), ("num_cores", ctypes.c_int), ("final_k", ctypes.c_int),
                ("engine_used", ctypes.c_int), ("launches", ctypes.c_int),
                ("reserved", ctypes.c_int * 6)]

    def as_dict(self):
        return {f: getattr(self, f) for f, _ in self._fields_ if f != "reserved"}


EXPORTS = ["fdb200_opts_init", "fdb200_last_error", "fdb200_abi_version", "fdb200_knn", "fdb200_fit",
           "fdb200_dc_reduction", "fdb200_density", "fdb200_dc_detection", "fdb200_final_cluster",
           "fdb200_knn_partial", "fdb200_merge_lists", "fdb200_lists_to_knn", "fdb200_fit_from_knn",
           "fdb200_release", "fdb200_density_noalloc", "fdb200_csv_shape", "fdb200_read_csv",
           "fdb200_write_csv", "fdb200_fbin_shape", "fdb200_read_fbin", "fdb200_write_fbin", "fdb200_knn_graph_save",
           "fdb200_knn_graph_shape", "fdb200_knn_graph_load", "fdb200_density_detection", "fdb200_dc_stage",
           "fdb200_dc_select", "fdb200_debug_tc_filter"]

_lib = None


def build(quiet=True):
    """Compile libfastdec_b200.so and the CLI for sm_100a (nvcc; no GPU needed)."""
    cmd = ["make", "-C", str(CSRC), "-j", str(max(1, min(8, os.cpu_count() or 1)))]
    subprocess.run(cmd, check=True, stdout=subprocess.DEVNULL if quiet else None)


def lib():
    """The loaded engine library. Raises if it has not been built -- there is no fallback."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FastDecError(-6, f"{LIB_PATH} is missing; run fastdec_b200.build() (or make -C {CSRC})")
        L = ctypes.CDLL(str(LIB_PATH))
        vp, ip, i = ctypes.c_void_p, ctypes.c_int, ctypes.c_int
        op, sp = ctypes.POINTER(Opts), ctypes.POINTER(Stats)
        L.fdb200_opts_init.argtypes = [op]
        L.fdb200_last_error.restype = ctypes.c_char_p
        L.fdb200_knn.argtypes = [vp, i, i, i, op, vp, vp, sp]
        L.fdb200_fit.argtypes = [vp, i, i, i, i, op, vp, vp, vp, sp]
        L.fdb200_dc_reduction.argtypes = [vp, i, i, vp, vp, i, i, op, vp, vp]
        L.fdb200_density.argtypes = [vp, i, i, op, vp, ctypes.POINTER(ctypes.c_double)]
        L.fdb200_dc_detection.argtypes = [vp, vp, i, i, op, vp, vp, ctypes.POINTER(ctypes.c_int)]
        L.fdb200_final_cluster.argtypes = [vp, i, vp, i, op, vp]
        L.fdb200_knn_partial.argtypes = [vp, i, i, i, op, vp, sp]
        L.fdb200_merge_lists.argtypes = [vp, vp, i, i, i, op]
        L.fdb200_lists_to_knn.argtypes = [vp, i, i, op, vp, vp]
        L.fdb200_fit_from_knn.argtypes = [vp, vp, vp, i, i, i, i, op, vp, vp, vp, sp]
        L.fdb200_release.argtypes = [op]
        cp, ipp = ctypes.c_char_p, ctypes.POINTER(ctypes.c_int)
        L.fdb200_csv_shape.argtypes = [cp, ipp, ipp]
        L.fdb200_read_csv.argtypes = [cp, i, i, vp, i]
        L.fdb200_write_csv.argtypes = [cp, vp, i, i, i]
        L.fdb200_fbin_shape.argtypes = [cp, ipp, ipp]
        L.fdb200_read_fbin.argtypes = [cp, i, i, vp, i]
        L.fdb200_write_fbin.argtypes = [cp, vp, i, i]
        L.fdb200_knn_graph_save.argtypes = [cp, vp, vp, i, i, i]
        L.fdb200_knn_graph_shape.argtypes = [cp, ipp, ipp, ipp]
        L.fdb200_knn_graph_load.argtypes = [cp, i, i, vp, vp]
        L.fdb200_density_detection.argtypes = [vp, vp, i, i, i, op, vp, vp, vp, ipp, ipp]
        L.fdb200_dc_stage.argtypes = [i, vp, i, i, vp, vp, i, i, i, op, vp, vp]
        L.fdb200_dc_select.argtypes = [vp, vp, i, vp, vp, i, op, vp, vp]
        L.fdb200_debug_tc_filter.argtypes = [vp, i, i, vp, op, vp, vp, vp, vp, ipp]
        _lib = L
    return _lib


_CUDA_STREAM_LEGACY = 0x1   # cudaStreamLegacy


def make_opts(device=0, precision="fp32", density="laplacian", engine="auto", on_device=False,
              shard=(0, 1), cand_capacity=0, stream=None, blocks=None, round_hook=None):
    o = Opts()
    lib().fdb200_opts_init(ctypes.byref(o))
    o.device = int(device)
    o.precision = _PRECISION[precision] if isinstance(precision, str) else int(precision)
    o.density_kernel = _DENSITY[density] if isinstance(density, str) else int(density)
    o.engine = _ENGINE[engine] if isinstance(engine, str) else int(engine)
    o.inputs_on_device = o.outputs_on_device = int(bool(on_device))
    o.shard_rank, o.shard_count = int(shard[0]), int(shard[1])
    o.cand_capacity = int(cand_capacity)
    if blocks is not None:   # explicit shard: row blocks [blocks[0], blocks[1])
        o.shard_block_lo, o.shard_block_hi = int(blocks[0]), int(blocks[1])
    if round_hook is not None:   # a ROUND_HOOK; the caller keeps it alive for the call
        o.round_hook = round_hook
    # stream: None = the library's own stream; an integer handle runs the call on that CUDA stream.
    # Handle 0 is the legacy default stream (torch's default stream reports 0); the ABI reserves a
    # NULL stream for "the library's own", so it is passed as cudaStreamLegacy.
    if stream is None:
        o.stream = None
    else:
        o.stream = _CUDA_STREAM_LEGACY if int(stream) == 0 else int(stream)
    return o


def _check(rc):
    if rc != 0:
        raise FastDecError(rc, lib().fdb200_last_error().decode())


def _ptr(a):
    """data pointer of a C-contiguous numpy array or torch tensor"""
    if hasattr(a, "data_ptr"):
        return ctypes.c_void_p(a.data_ptr())
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


# ---------------------------------------------------------------- host-array API
def knn(data_dm, k, **kw):
    """Exact self-kNN (symtri_knn_cuda). Returns rank-major (k, n) distances and indices."""
    x = _f32(data_dm)
    d, n = x.shape
    dist = np.zeros((max(k, 0), n), np.float32)
    idx = np.zeros((max(k, 0), n), np.int32)
    st = Stats()
    _check(lib().fdb200_knn(_ptr(x), n, d, k, ctypes.byref(make_opts(**kw)), _ptr(dist), _ptr(idx),
                            ctypes.byref(st)))
    return dist, idx, st.as_dict()


def read_csv(path, threads=0):
    """The reference CLI's dataset file (one point per line, comma-separated) as a dim-major
    (d, n) float32 array, parsed in parallel by the library (fdb200_csv_shape / fdb200_read_csv)."""
    n, d = ctypes.c_int(0), ctypes.c_int(0)
    p = str(path).encode()
    _check(lib().fdb200_csv_shape(p, ctypes.byref(n), ctypes.byref(d)))
    out = np.empty((d.value, n.value), np.float32)
    _check(lib().fdb200_read_csv(p, n.value, d.value, _ptr(out), int(threads)))
    return out


def write_csv(path, data_dm, threads=0):
    """Writes a dim-major (d, n) float32 array in the reference CLI's CSV format (fdb200_write_csv):
    one point per line, values as the shortest text that reads back to the same float."""
    x = _f32(data_dm)
    d, n = x.shape
    _check(lib().fdb200_write_csv(str(path).encode(), _ptr(x), n, d, int(threads)))


def read_fbin(path, threads=0):
    """A binary dataset file (int32 n, int32 d, then n x d float32 row-major) as a dim-major (d, n)
    float32 array (fdb200_fbin_shape / fdb200_read_fbin)."""
    n, d = ctypes.c_int(0), ctypes.c_int(0)
    p = str(path).encode()
    _check(lib().fdb200_fbin_shape(p, ctypes.byref(n), ctypes.byref(d)))
    out = np.empty((d.value, n.value), np.float32)
    _check(lib().fdb200_read_fbin(p, n.value, d.value, _ptr(out), int(threads)))
    return out


def write_fbin(path, data_dm):
    """Writes a dim-major (d, n) float32 array as a binary dataset file (fdb200_write_fbin)."""
    x = _f32(data_dm)
    d, n = x.shape
    _check(lib().fdb200_write_fbin(str(path).encode(), _ptr(x), n, d))


def save_knn_graph(path, dist_rm, idx_rm, flags=0):
    """Saves a rank-major (k, n) kNN graph (fdb200_knn_graph_save)."""
    dist, idx = _f32(dist_rm), _i32(idx_rm)
    k, n = dist.shape
    assert idx.shape == (k, n)
    _check(lib().fdb200_knn_graph_save(str(path).encode(), _ptr(dist), _ptr(idx), n, k, int(flags)))


def load_knn_graph(path):
    """Loads a saved kNN graph: (dist (k, n), idx (k, n), flags)."""
    n, k, fl = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    p = str(path).encode()
    _check(lib().fdb200_knn_graph_shape(p, ctypes.byref(n), ctypes.byref(k), ctypes.byref(fl)))
    dist = np.empty((k.value, n.value), np.float32)
    idx = np.empty((k.value, n.value), np.int32)
    _check(lib().fdb200_knn_graph_load(p, n.value, k.value, _ptr(dist), _ptr(idx)))
    return dist, idx, fl.value


def fit_from_knn(data_dm, dist_rm, idx_rm, k, c, **kw):
    """The fit's stages after the kNN on a given rank-major graph (host arrays): the first k ranks
    of dist / idx are used. Returns dict(centers, labels, densities, stats)."""
    x = _f32(data_dm)
    d, n = x.shape
    dist, idx = _f32(dist_rm), _i32(idx_rm)
    assert dist.shape[1] == n and idx.shape == dist.shape and k <= dist.shape[0]
    centers = np.full(c, -1, np.int32)
    labels = np.full(n, -1, np.int32)
    den = np.zeros(n, np.float32)
    st = Stats()
    _check(lib().fdb200_fit_from_knn(_ptr(x), _ptr(dist), _ptr(idx), n, d, k, c, ctypes.byref(make_opts(**kw)),
                                     _ptr(centers), _ptr(labels), _ptr(den), ctypes.byref(st)))
    return dict(centers=centers, labels=labels, densities=den, stats=st.as_dict())


def fit(data_dm, k, c, **kw):
    """The whole FastDEC fit. Returns dict(centers, labels, densities, stats)."""
    x = _f32(data_dm)
    d, n = x.shape
    centers = np.full(c, -1, np.int32)
    labels = np.full(n, -1, np.int32)
    den = np.zeros(n, np.float32)
    st = Stats()
    _check(lib().fdb200_fit(_ptr(x), n, d, k, c, ctypes.byref(make_opts(**kw)), _ptr(centers), _ptr(labels),
                            _ptr(den), ctypes.byref(st)))
    return dict(centers=centers, labels=labels, densities=den, stats=st.as_dict())


def density(dist_rm, k=None, gaussian=False, **kw):
    dist = _f32(dist_rm)
    kk, n = dist.shape
    out = np.zeros(n, np.float32)
    mean = ctypes.c_double(0.0)
    kw.setdefault("density", "gaussian" if gaussian else "laplacian")
    # the rank stride of the list is n, the first k ranks are used
    _check(lib().fdb200_density(_ptr(dist), n, k or kk, ctypes.byref(make_opts(**kw)), _ptr(out),
                                ctypes.byref(mean)))
    return out, mean.value


def dc_detection(idx_rm, den, k=None, **kw):
    idx = _i32(idx_rm)
    kk, n = idx.shape
    parent = np.zeros(n, np.int32)
    cores = np.zeros(n, np.int32)
    nc = ctypes.c_int(0)
    _check(lib().fdb200_dc_detection(_ptr(idx), _ptr(_f32(den)), n, k or kk, ctypes.byref(make_opts(**kw)),
                                     _ptr(parent), _ptr(cores), ctypes.byref(nc)))
    return parent, cores[:nc.value].copy()


def dc_reduction(data_dm, den, cores, num_centers, **kw):
    """warp_parallel_dc_reduction_cuda: returns (core_parent, centers)."""
    x = _f32(data_dm)
    d, n = x.shape
    cores = _i32(cores)
    cp = np.zeros(len(cores), np.int32)
    ctr = np.zeros(num_centers, np.int32)
    _check(lib().fdb200_dc_reduction(_ptr(x), n, d, _ptr(_f32(den)), _ptr(cores), len(cores), num_centers,
                                     ctypes.byref(make_opts(**kw)), _ptr(cp), _ptr(ctr)))
    return cp, ctr


def final_cluster(parent, centers, **kw):
    parent = _i32(parent)
    centers = _i32(centers)
    labels = np.zeros(len(parent), np.int32)
    _check(lib().fdb200_final_cluster(_ptr(parent), len(parent), _ptr(centers), len(centers),
                                      ctypes.byref(make_opts(**kw)), _ptr(labels)))
    return labels


# ---------------------------------------------------------------- device (torch) API
def fit_device(x_dm, k, c, centers, labels, densities=None, stream=None, **kw):
    """Fit on a dim-major float32 CUDA tensor; outputs are CUDA int32 tensors. Returns stats."""
    d, n = x_dm.shape
    st = Stats()
    o = make_opts(on_device=True, stream=stream, device=x_dm.device.index or 0, **kw)
    _check(lib().fdb200_fit(_ptr(x_dm), n, d, k, c, ctypes.byref(o), _ptr(centers), _ptr(labels),
                            _ptr(densities) if densities is not None else None, ctypes.byref(st)))
    return st.as_dict()


def knn_partial_device(x_dm, k, lists, shard, stream=None, **kw):
    """Packed partial lists (n, k) uint64-as-int64 tensor for shard=(rank, count). Returns stats."""
    d, n = x_dm.shape
    st = Stats()
    o = make_opts(on_device=True, stream=stream, shard=shard, device=x_dm.device.index or 0, **kw)
    _check(lib().fdb200_knn_partial(_ptr(x_dm), n, d, k, ctypes.byref(o), _ptr(lists), ctypes.byref(st)))
    return st.as_dict()


def merge_lists_device(lists, srcs, nsrc, n_points, k, stream=None, device=0):
    o = make_opts(on_device=True, stream=stream, device=device)
    _check(lib().fdb200_merge_lists(_ptr(lists), _ptr(srcs) if nsrc else None, nsrc, n_points, k,
                                    ctypes.byref(o)))


def lists_to_knn_device(lists, n, k, dist, idx, stream=None, device=0):
    o = make_opts(on_device=True, stream=stream, device=device)
    _check(lib().fdb200_lists_to_knn(_ptr(lists), n, k, ctypes.byref(o), _ptr(dist), _ptr(idx)))


def fit_from_knn_device(x_dm, dist, idx, k, c, centers, labels, densities=None, stream=None, **kw):
    d, n = x_dm.shape
    st = Stats()
    o = make_opts(on_device=True, stream=stream, device=x_dm.device.index or 0, **kw)
    _check(lib().fdb200_fit_from_knn(_ptr(x_dm), _ptr(dist), _ptr(idx), n, d, k, c, ctypes.byref(o),
                                     _ptr(centers), _ptr(labels),
                                     _ptr(densities) if densities is not None else None, ctypes.byref(st)))
    return st.as_dict()


def density_detection_device(dist, idx, k, c, den, parent, cores, stream=None, device=0, **kw):
    """Density + DC detection with the k-halving retry on device tensors (rank-major (>= k, n) dist / idx;
    den (n,) float32, parent (n,) int32, cores (n,) int32 outputs). Returns (num_cores, final_k)."""
    n = dist.shape[1]
    nc, fk = ctypes.c_int(0), ctypes.c_int(0)
    o = make_opts(on_device=True, stream=stream, device=device, **kw)
    _check(lib().fdb200_density_detection(_ptr(dist), _ptr(idx), n, k, c, ctypes.byref(o), _ptr(den), _ptr(parent),
                                          _ptr(cores), ctypes.byref(nc), ctypes.byref(fk)))
    return nc.value, fk.value


def dc_stage_device(stage, x_dm, den, cores, core_nb, p_lo, p_hi, best, rank=None, stream=None):
    """One stage of the DC reduction over the points [p_lo, p_hi) (device tensors; best: (core_nb,) int64
    holding packed uint64 keys, rank: (core_nb,) int32)."""
    d, n = x_dm.shape
    o = make_opts(on_device=True, stream=stream, device=x_dm.device.index or 0)
    _check(lib().fdb200_dc_stage(int(stage), _ptr(x_dm), n, d, _ptr(den), _ptr(cores), int(core_nb), int(p_lo),
                                 int(p_hi), ctypes.byref(o), _ptr(best), _ptr(rank) if rank is not None else None))


def dc_select_device(den, cores, core_nb, best, rank, c, core_parent, centers, stream=None, device=0):
    o = make_opts(on_device=True, stream=stream, device=device)
    _check(lib().fdb200_dc_select(_ptr(den), _ptr(cores), int(core_nb), _ptr(best), _ptr(rank), int(c),
                                  ctypes.byref(o), _ptr(core_parent), _ptr(centers)))


def final_cluster_device(parent, centers, labels, stream=None, device=0):
    o = make_opts(on_device=True, stream=stream, device=device)
    _check(lib().fdb200_final_cluster(_ptr(parent), parent.shape[0], _ptr(centers), centers.shape[0],
                                      ctypes.byref(o), _ptr(labels)))


def debug_tc_filter(x_dm, thr_d2, precision="fp32"):
    """Diagnostics (fdb200_debug_tc_filter): the raw tcgen05 filter accumulators for every ordered pair
    of a small dim-major float32 dataset with per-point thresholds (squared distances) folded in.
    Returns (acc (n, n), V (n,), A rows (n, K), B rows (n, K)) as numpy arrays."""
    import torch
    x = torch.from_numpy(_f32(x_dm)).cuda()
    d, n = x.shape
    thr = torch.from_numpy(_f32(thr_d2)).cuda()
    kp = ((d + 6 + 7) // 8) * 8
    acc = torch.empty((n, n), dtype=torch.float32, device=x.device)
    V = torch.empty(n, dtype=torch.float32, device=x.device)
    ar = torch.empty((n, kp), dtype=torch.float32, device=x.device)
    br = torch.empty((n, kp), dtype=torch.float32, device=x.device)
    kpo = ctypes.c_int(0)
    o = make_opts(on_device=True, precision=precision, device=x.device.index or 0)
    _check(lib().fdb200_debug_tc_filter(_ptr(x), n, d, _ptr(thr), ctypes.byref(o), _ptr(acc), _ptr(V), _ptr(ar),
                                        _ptr(br), ctypes.byref(kpo)))
    assert kpo.value == kp
    return acc.cpu().numpy(), V.cpu().numpy(), ar.cpu().numpy(), br.cpu().numpy()


def release(device=0):
    _check(lib().fdb200_release(ctypes.byref(make_opts(device=device))))


class B200FastDEC:
    """Mirror of the reference's Fit surface (FastDECBase / SymWarpFullGpuFastDEC, test.cpp:124-140)."""

    def __init__(self, num_k_points, num_clusters, name="b200_fastdec", cuda_device_id=0, **opts):
        print("- %-17s : " % name)
        self.k, self.c, self.device, self.opts = num_k_points, num_clusters, cuda_device_id, opts
        self._centers = self._labels = self._den = None
        self.stats = None

    def Fit(self, data, num_points, num_dim):
        x = np.asarray(data, np.float32).reshape(num_dim, num_points)
        r = fit(x, self.k, self.c, device=self.device, **self.opts)
        self._centers, self._labels, self._den, self.stats = r["centers"], r["labels"], r["densities"], r["stats"]

    def get_center_indices(self):
        return self._centers

    def get_labels(self):
        return self._labels

    def get_densities(self):
        return self._den
