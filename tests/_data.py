"""Seeded numpy generators with the value distributions of BASELINE.json's
configs, at sizes the CPU oracle checks in seconds."""

import numpy as np


def unit_gaussian(n, d, seed):
    """Config 1/4: i.i.d. N(0,1) per dim, then L2-normalised (fp32)."""
    x = np.random.default_rng(seed).standard_normal((n, d)).astype(np.float32)
    return (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32)


def sift_like(n, nq, d=128, centres=1000, seed=0):
    """Config 2: centres U[0,128]^d, noise sigma 20, clamp [0,255], round.

    Returns (base, queries); queries are drawn from the same mixture but are
    not base rows. Integer-valued data makes exact distance ties common.
    """
    rng = np.random.default_rng(seed)
    c = rng.uniform(0, 128, size=(centres, d)).astype(np.float32)

    def draw(m):
        lab = rng.integers(0, centres, size=m)
        x = c[lab] + rng.normal(0, 20, size=(m, d)).astype(np.float32)
        return np.rint(np.clip(x, 0, 255)).astype(np.float32)

    return draw(n), draw(nq)


def gaussian_mixture(n, nq, d=96, centres=10000, seed=0):
    """Config 5: centres N(0,1)*4, points = centre + N(0,1)."""
    rng = np.random.default_rng(seed)
    c = (rng.standard_normal((centres, d)) * 4).astype(np.float32)

    def draw(m):
        lab = rng.integers(0, centres, size=m)
        return (c[lab] + rng.standard_normal((m, d))).astype(np.float32)

    return draw(n), draw(nq)
