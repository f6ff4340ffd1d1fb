"""Stage-level parity for the post-kNN kernels, given identical inputs."""
import numpy as np
import pytest

import fastdec_b200.datasets as ds

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,k,gauss", [(1, 1, False), (31, 3, False), (1000, 7, True), (100003, 45, False),
                                       (250000, 20, True)])
def test_density_and_mean_bit_exact(fdb, oracle, n, k, gauss):
    rng = np.random.default_rng(n + k)
    dist = np.sort(rng.gamma(2.0, 0.3, (k, n)).astype(np.float32), axis=0)
    den, mean = fdb.density(dist, gaussian=gauss)
    assert mean == oracle.mean_knn_dist(dist)
    assert np.array_equal(den.view(np.uint32), oracle.density(dist, gaussian=gauss).view(np.uint32))


def test_mean_with_ties_and_zeros(fdb, oracle):
    # values on a coarse grid hit exact half-ulp ties in the running sum; zeros are identities
    rng = np.random.default_rng(3)
    dist = (rng.integers(0, 9, (16, 60000)) * 0.25).astype(np.float32)
    dist[:, :1000] = 0
    _, mean = fdb.density(dist)
    assert mean == oracle.mean_knn_dist(dist)


def test_truncated_ranks(fdb, oracle):
    rng = np.random.default_rng(4)
    dist = np.sort(rng.random((20, 5000)).astype(np.float32), axis=0)
    den, mean = fdb.density(dist, k=10)
    assert mean == oracle.mean_knn_dist(dist, k=10)
    assert np.array_equal(den, oracle.density(dist, k=10))


def test_detection_matches_oracle(fdb, oracle):
    x = ds.gmm_isotropic(n=8000, d=8, seed=3)
    dist, idx = oracle.knn(x, 15)
    den = oracle.density(dist)
    p, cores = fdb.dc_detection(idx, den)
    op, ocores = oracle.dc_detection(idx, den)
    assert np.array_equal(p, op) and np.array_equal(cores, ocores)


def test_dc_reduction_known_answers(fdb, known):
    for key in ("dc_known_case", "dc_no_denser"):
        kc = known[key]
        x = np.array([kc["points_1d"]], np.float32)
        cp, centers = fdb.dc_reduction(x, np.array(kc["densities"], np.float32), kc["cores"], kc["num_centers"])
        assert cp.tolist() == kc["expected_parents"]
        assert centers.tolist() == [kc["expected_center"]]


@pytest.mark.parametrize("n,d,c", [(3000, 2, 5), (20000, 16, 10), (6000, 50, 40)])
def test_dc_reduction_matches_oracle(fdb, oracle, n, d, c):
    x = ds.gmm_isotropic(n=n, d=d, comps=12, seed=n)
    dist, idx = oracle.knn(x, 10)
    den = oracle.density(dist)
    _, cores = oracle.dc_detection(idx, den)
    cp, ctr = fdb.dc_reduction(x, den, cores, c)
    ocp, _, _, octr = oracle.dc_reduction(x, den, cores, c)
    assert np.array_equal(cp, ocp)
    assert np.array_equal(ctr, octr)


def test_final_cluster_matches_oracle(fdb, oracle):
    rng = np.random.default_rng(9)
    n = 50000
    den = rng.random(n).astype(np.float32)
    order = np.argsort(-den, kind="stable")
    parent = np.full(n, -1, np.int32)
    for t in range(1, n):                 # each point's parent is a denser point (or none)
        if rng.random() < 0.97:
            parent[order[t]] = order[rng.integers(0, t)]
    centers = order[:7].astype(np.int32)
    assert np.array_equal(fdb.final_cluster(parent, centers), oracle.final_cluster(den, parent, centers))


def test_final_cluster_detects_cycles(fdb):
    parent = np.array([1, 2, 0, -1], np.int32)
    with pytest.raises(fdb.FastDecError) as e:
        fdb.final_cluster(parent, np.array([3], np.int32))
    assert e.value.code == -5


@pytest.mark.parametrize("ranges", [3, 8])
def test_sharded_dc_reduction_stages_equal_the_whole(fdb, oracle, ranges):
    """fdb200_dc_stage over disjoint point ranges, combined by minimum (stage A keys) and sum (stage B
    ranks) as the multi-GPU fit combines them, then fdb200_dc_select: the same core parents and
    centers as fdb200_dc_reduction and the reference's host stages. Also fdb200_density_detection
    against the reference (densities, cores, final k)."""
    import torch
    from fastdec_b200.multigpu import owner_ranges
    x = ds.embedding_cloud(n=30_000, d=50, seed=41)
    n, k, c = x.shape[1], 20, 12
    dist, idx, _ = fdb.knn(x, k)
    dd, di = torch.from_numpy(dist).cuda(), torch.from_numpy(idx).cuda()
    den = torch.empty(n, dtype=torch.float32, device="cuda")
    parent = torch.empty(n, dtype=torch.int32, device="cuda")
    cores = torch.empty(n, dtype=torch.int32, device="cuda")
    nc, fk = fdb.density_detection_device(dd, di, k, c, den, parent, cores)
    ref = oracle.ref_fit_from_knn(x, dist, idx, c)
    assert fk == ref["final_k"] and nc == ref["num_cores"] and nc > c
    assert np.array_equal(den.cpu().numpy().view(np.uint32), ref["densities"].view(np.uint32))
    assert np.array_equal(cores[:nc].cpu().numpy(), ref["cores"])
    xd = torch.from_numpy(x).cuda()
    cr = cores[:nc].contiguous()
    best = []
    for a, b in owner_ranges(n, ranges):
        t = torch.empty(nc, dtype=torch.int64, device="cuda")
        fdb.dc_stage_device(0, xd, den, cr, nc, a, b, t)
        best.append(t.cpu().numpy().view(np.uint64))
    comb = torch.from_numpy(np.minimum.reduce(best).view(np.int64).copy()).cuda()
    rk = np.zeros(nc, np.int64)
    for a, b in owner_ranges(n, ranges):
        t = torch.empty(nc, dtype=torch.int32, device="cuda")
        fdb.dc_stage_device(1, xd, den, cr, nc, a, b, comb, t)
        rk += t.cpu().numpy()
    rkd = torch.from_numpy(rk.astype(np.int32)).cuda()
    cp = torch.empty(nc, dtype=torch.int32, device="cuda")
    ctr = torch.empty(c, dtype=torch.int32, device="cuda")
    fdb.dc_select_device(den, cr, nc, comb, rkd, c, cp, ctr)
    wcp, wctr = fdb.dc_reduction(x, den.cpu().numpy(), cr.cpu().numpy(), c)
    assert np.array_equal(cp.cpu().numpy(), wcp) and np.array_equal(ctr.cpu().numpy(), wctr)
    assert ctr.cpu().numpy().tolist() == ref["centers"].tolist()
    p = parent.cpu().numpy()
    p[cr.cpu().numpy()] = cp.cpu().numpy()
    assert np.array_equal(p, ref["parents"])
