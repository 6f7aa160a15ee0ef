"""Seeded inputs of the simd-layout fixtures: make_golden.py builds the
fixtures from them and the tests regenerate them (only outputs are stored)."""

import numpy as np


def layout_inputs():
    rng = np.random.default_rng(12)
    tok = rng.standard_normal((7, 48))
    W = rng.standard_normal((48, 48))
    q = rng.standard_normal((5, 768))
    k = rng.standard_normal((7, 768))
    Tc = 20
    weights = np.tril(rng.random((12, Tc, Tc)))
    weights /= weights.sum(axis=2, keepdims=True)
    values = rng.standard_normal((12, Tc, 64))
    return tok, W, q, k, weights, values
