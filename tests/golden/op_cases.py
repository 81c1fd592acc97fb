"""Seeded inputs of the op-level fixtures in ops_htdemucs.npz: the attention and
LayerNorm shapes that HTDemucs' transformer feeds to the reference's shared ops
(ops::scaled_dot_product_attention and ops::layer_norm, called from
src/model_htdemucs.cu:555-659 with dim 384 over 8 heads, so head_dim 48, and
cross-attention between branches of different lengths).

The fixture stores only the reference's outputs; make_golden.py and the tests
rebuild the inputs from the seeds below.
"""
from __future__ import annotations

import numpy as np

# name: (seed, B, H, Nq, Nk, D, scale); scale 0 selects the op's default 1/sqrt(D)
SDPA_CASES = {
    "self48": (31, 1, 8, 160, 160, 48, 0.0),
    "cross48": (32, 2, 8, 96, 131, 48, 0.0),
    "cross64": (33, 1, 4, 200, 77, 64, 0.125),
    "self32": (34, 3, 2, 45, 45, 32, 0.0),
}

# name: (seed, rows, D)
LN_CASES = {
    "ln384": (41, 128, 384),
    "ln512": (42, 64, 512),
    "ln200": (43, 33, 200),
}

LN_EPS = 1e-5


def sdpa_inputs(name: str):
    seed, B, H, Nq, Nk, D, scale = SDPA_CASES[name]
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, H, Nq, D)).astype(np.float32)
    k = rng.standard_normal((B, H, Nk, D)).astype(np.float32)
    v = rng.standard_normal((B, H, Nk, D)).astype(np.float32)
    return q, k, v, scale


def default_scale(D: int) -> float:
    return float(1.0 / np.sqrt(np.float32(D)))


def ln_inputs(name: str):
    seed, rows, D = LN_CASES[name]
    rng = np.random.default_rng(seed)
    x = (0.5 + 2.0 * rng.standard_normal((rows, D))).astype(np.float32)
    g = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    b = (0.1 * rng.standard_normal(D)).astype(np.float32)
    return x, g, b
