"""Binary files around the fit, host-only (no GPU): the .fbin dataset input (int32 n, int32 d, then
row-major float32) and kNN-graph persistence (fdb200_knn_graph_save / _shape / _load), including the
damaged-file cases the loader must reject instead of fitting on wrong data."""
import numpy as np
import pytest

import fastdec_b200 as fdb


def test_fbin_round_trip_and_layout(tmp_path):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((7, 5003)).astype(np.float32)          # dim-major (d, n)
    x[0, :5] = [0.0, -0.0, np.inf, -np.inf, 1e-45]
    p = tmp_path / "a.fbin"
    fdb.write_fbin(p, x)
    raw = np.fromfile(p, np.uint8)
    assert raw[:8].view(np.int32).tolist() == [5003, 7]
    assert np.array_equal(raw[8:].view(np.float32).reshape(5003, 7), x.T)   # row-major body
    for threads in (1, 3, 0):
        y = fdb.read_fbin(p, threads=threads)
        assert np.array_equal(y.view(np.uint32), x.view(np.uint32))
    # a file written by numpy reads the same
    q = tmp_path / "b.fbin"
    with open(q, "wb") as f:
        np.asarray([5003, 7], np.int32).tofile(f)
        np.ascontiguousarray(x.T).tofile(f)
    assert np.array_equal(fdb.read_fbin(q).view(np.uint32), x.view(np.uint32))


def test_fbin_rejects_a_size_that_disagrees_with_its_header(tmp_path):
    p = tmp_path / "bad.fbin"
    with open(p, "wb") as f:
        np.asarray([100, 4], np.int32).tofile(f)
        np.zeros(399, np.float32).tofile(f)
    with pytest.raises(fdb.FastDecError) as e:
        fdb.read_fbin(p)
    assert e.value.code == -1 and "header says 100 x 4" in str(e.value)
    with pytest.raises(fdb.FastDecError):
        fdb.read_fbin(tmp_path / "missing.fbin")


def _graph(n, k, seed):
    rng = np.random.default_rng(seed)
    dist = np.sort(rng.random((n, k), dtype=np.float32), axis=1).T.copy()
    idx = rng.integers(0, n, (k, n)).astype(np.int32)
    return dist, idx


def test_knn_graph_round_trip(tmp_path):
    dist, idx = _graph(4001, 12, 1)
    p = tmp_path / "g.knng"
    fdb.save_knn_graph(p, dist, idx, flags=1)
    d2, i2, fl = fdb.load_knn_graph(p)
    assert fl == 1
    assert np.array_equal(d2.view(np.uint32), dist.view(np.uint32)) and np.array_equal(i2, idx)
    raw = np.fromfile(p, np.uint8)
    assert raw[:8].tobytes() == b"FDBKNNG1" and raw.size == 32 + 8 * 4001 * 12
    # rank-major payload, distances then indices
    assert np.array_equal(raw[32:32 + 4 * 4001 * 12].view(np.float32).reshape(12, 4001), dist)


def test_knn_graph_loader_rejects_damaged_files(tmp_path):
    dist, idx = _graph(1000, 8, 2)
    p = tmp_path / "g.knng"
    fdb.save_knn_graph(p, dist, idx)
    raw = np.fromfile(p, np.uint8)
    # one flipped bit in the payload: the hash no longer matches
    bad = raw.copy()
    bad[32 + 4 * 1234] ^= 1
    bad.tofile(tmp_path / "flip.knng")
    with pytest.raises(fdb.FastDecError) as e:
        fdb.load_knn_graph(tmp_path / "flip.knng")
    assert e.value.code == -1 and "hash" in str(e.value)
    # truncated
    raw[:-4].tofile(tmp_path / "short.knng")
    with pytest.raises(fdb.FastDecError) as e:
        fdb.load_knn_graph(tmp_path / "short.knng")
    assert "truncated" in str(e.value)
    # not a graph file
    np.zeros(64, np.uint8).tofile(tmp_path / "zero.knng")
    with pytest.raises(fdb.FastDecError) as e:
        fdb.load_knn_graph(tmp_path / "zero.knng")
    assert "not a kNN graph" in str(e.value)
    # an index out of range (with a matching hash: written through the library)
    idx2 = idx.copy()
    idx2[3, 5] = 1000
    fdb.save_knn_graph(tmp_path / "oob.knng", dist, idx2)
    with pytest.raises(fdb.FastDecError) as e:
        fdb.load_knn_graph(tmp_path / "oob.knng")
    assert "out of range" in str(e.value)
