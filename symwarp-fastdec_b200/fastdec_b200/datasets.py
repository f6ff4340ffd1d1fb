"""Seeded synthetic datasets with the shapes and value distributions of the benchmark configs.

The reference's headline numbers are quoted on GloVe 50d (1,291,147 x 50, min-max scaled to
[-1, 1]); that file is not available here, so these generators stand in for it. Every function
returns a DIM-MAJOR float32 array of shape (d, n) -- the layout the reference's Fit receives
(test.cpp:110-115 transposes the CSV rows into it) -- with points in random order.
"""
from __future__ import annotations

import numpy as np


def _finish(points_rm: np.ndarray, rng: np.random.Generator) -> np.ndarray:
    perm = rng.permutation(points_rm.shape[0])
    return np.ascontiguousarray(points_rm[perm].T.astype(np.float32))


def _minmax_pm1(x: np.ndarray) -> np.ndarray:
    lo = x.min(axis=0, keepdims=True)
    hi = x.max(axis=0, keepdims=True)
    span = np.where(hi > lo, hi - lo, 1.0)
    return (x - lo) / span * 2.0 - 1.0


def spiral3(seed: int = 1, per_arm: int = 104, jitter: float = 0.3) -> np.ndarray:
    """Config 1: 2-D 3-arm spiral, theta ~ U[0.5, 4 pi], r = theta, arm i rotated by 2 pi i / 3."""
    rng = np.random.default_rng(seed)
    arms = []
    for a in range(3):
        th = rng.uniform(0.5, 4 * np.pi, per_arm)
        r = th * 1.0
        rot = 2 * np.pi * a / 3
        xy = np.stack([r * np.cos(th + rot), r * np.sin(th + rot)], axis=1)
        arms.append(xy + rng.normal(0.0, jitter, xy.shape))
    return _finish(np.concatenate(arms), rng)


def gmm_isotropic(n: int = 100_000, d: int = 16, comps: int = 10, seed: int = 2) -> np.ndarray:
    """Config 2: equal-weight isotropic Gaussian mixture, centers U[-10, 10]^d, sigma 1."""
    rng = np.random.default_rng(seed)
    centers = rng.uniform(-10.0, 10.0, (comps, d))
    lab = rng.integers(0, comps, n)
    x = centers[lab] + rng.normal(0.0, 1.0, (n, d))
    return _finish(x, rng)


def embedding_cloud(n: int = 1_291_147, d: int = 50, comps: int = 20, seed: int = 3,
                    heavy_frac: float = 0.05) -> np.ndarray:
    """Configs 3/4: 20 anisotropic Gaussians (per-dim sigma log-U[0.05, 0.5]) with Zipf(1.1)
    weights, plus a fraction of Student-t(3) heavy-tail points, min-max scaled to [-1, 1]."""
    rng = np.random.default_rng(seed)
    n_heavy = int(round(n * heavy_frac))
    n_main = n - n_heavy
    w = 1.0 / np.arange(1, comps + 1) ** 1.1
    w /= w.sum()
    counts = rng.multinomial(n_main, w)
    centers = rng.uniform(-1.0, 1.0, (comps, d))
    sig = np.exp(rng.uniform(np.log(0.05), np.log(0.5), (comps, d)))
    parts = [centers[c] + rng.standard_normal((counts[c], d)) * sig[c] for c in range(comps)]
    parts.append(rng.standard_t(3, (n_heavy, d)) * 0.5)
    x = _minmax_pm1(np.concatenate(parts))
    return _finish(x, rng)


def scale_out(n: int = 4_000_000, d: int = 128, comps: int = 50, seed: int = 5) -> np.ndarray:
    """Config 5: 50 anisotropic Gaussians with random orthogonal rotations (per-axis sigma
    log-U[0.1, 1.0]), min-max scaled to [-1, 1]^d."""
    rng = np.random.default_rng(seed)
    counts = rng.multinomial(n, np.full(comps, 1.0 / comps))
    out = np.empty((n, d), np.float32)
    pos = 0
    for c in range(comps):
        q, _ = np.linalg.qr(rng.standard_normal((d, d)))
        sig = np.exp(rng.uniform(np.log(0.1), np.log(1.0), d))
        z = rng.standard_normal((counts[c], d)).astype(np.float32) * sig.astype(np.float32)
        out[pos:pos + counts[c]] = z @ q.T.astype(np.float32) + rng.uniform(-4, 4, d).astype(np.float32)
        pos += counts[c]
    out = _minmax_pm1(out)
    return _finish(out, rng)


def small_integer_grid(n: int, d: int, levels: int = 6, seed: int = 7) -> np.ndarray:
    """Small-integer coordinates: many exact distance ties and duplicate points."""
    rng = np.random.default_rng(seed)
    return np.ascontiguousarray(rng.integers(0, levels, (d, n)).astype(np.float32))


CONFIGS = {
    "spiral3": dict(gen=spiral3, k=7, c=3),
    "gmm100k": dict(gen=gmm_isotropic, k=20, c=10),
    "glove_like": dict(gen=embedding_cloud, k=45, c=20),
    "scale_out": dict(gen=scale_out, k=64, c=50),
}
