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


# the axial attention alone at the benchmarked shape, bf16 q/k/v ~ N(0, 1),
# scale 1/8, B = 4 chunks, T = 801 frames, F = 62 bands, 8 heads x 64.  The time axis is B*F
# sequences of T tokens, the band axis B*T sequences of F tokens.  The fixture
# (config3_ref.npz) holds the reference's outputs for a seeded sample of (sequence, head)
# pairs, stored as float16.
CONFIG3 = dict(B=4, T=801, F=62, H=8, D=64, scale=0.125, seeds={"time": 61, "band": 62},
               samples={"time": 8, "band": 64}, sample_seed=63)


def bf16_values(a: np.ndarray) -> np.ndarray:
    """fp32 array rounded to the nearest bf16 value (ties to even), kept in fp32."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)).astype(np.uint32)
    return r.view(np.float32)


def config3_inputs(axis: str):
    """q, k, v [S, H, N, D] fp32 holding bf16 values, S sequences of N tokens on `axis`."""
    c = CONFIG3
    S, N = (c["B"] * c["F"], c["T"]) if axis == "time" else (c["B"] * c["T"], c["F"])
    rng = np.random.default_rng(c["seeds"][axis])
    return tuple(bf16_values(rng.standard_normal((S, c["H"], N, c["D"]), dtype=np.float32)) for _ in range(3))


def config3_samples(axis: str):
    """The sampled (sequence, head) pairs of the fixture, sorted."""
    c = CONFIG3
    S = c["B"] * c["F"] if axis == "time" else c["B"] * c["T"]
    rng = np.random.default_rng(c["sample_seed"] + (0 if axis == "time" else 1))
    flat = np.sort(rng.choice(S * c["H"], c["samples"][axis], replace=False))
    return flat // c["H"], flat % c["H"]
