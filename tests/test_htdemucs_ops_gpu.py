"""GPU parity of the ops the reference shares with HTDemucs' transformer
(src/model_htdemucs.cu:542-659): msst_sdpa (ops::scaled_dot_product_attention,
head_dim 48 and cross-attention with Nq != Nk) and msst_layernorm (ops::layer_norm).

Checked against the reference engine's own outputs (tests/golden/ops_htdemucs.npz,
made by oracle/_ref on a B200 from the seeds in tests/golden/op_cases.py) and
against the fp32 CPU oracle on the same 16-bit-rounded inputs.

Tolerances (relative L2): attention output rounded to fp16 / bf16 with P also
16-bit: 3e-3 / 1.5e-2, the bars of the Roformer attention test; vs the reference's
TF32 path the input rounding adds to that.  LayerNorm fp32: 1e-6 (summation order
only); 16-bit outputs: one rounding, 1e-3 / 5e-3.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden, rel_l2
import op_cases

pytestmark = pytest.mark.gpu

ATTN_TOL = {"fp16": 3e-3, "bf16": 1.5e-2}
REF_TOL = {"fp16": 4e-3, "bf16": 2e-2}


def _dt(torch, prec):
    return torch.float16 if prec == "fp16" else torch.bfloat16


def _rounded(torch, a, prec):
    t = torch.from_numpy(a).to(_dt(torch, prec))
    return t, t.float().numpy()


@pytest.mark.parametrize("prec", ["fp16", "bf16"])
@pytest.mark.parametrize("name", list(op_cases.SDPA_CASES))
def test_sdpa_vs_reference(cuda, name, prec):
    torch = cuda
    import oracle
    from msst_b200 import ops

    z, _ = golden("ops_htdemucs.npz")
    q, k, v, scale = op_cases.sdpa_inputs(name)
    D = q.shape[-1]
    (tq, q16), (tk, k16), (tv, v16) = (_rounded(torch, a, prec) for a in (q, k, v))
    y = ops.scaled_dot_product_attention(tq.cuda(), tk.cuda(), tv.cuda(), scale)
    torch.cuda.synchronize()
    y = y.float().cpu().numpy()
    s = scale if scale != 0.0 else op_cases.default_scale(D)
    assert rel_l2(y, oracle.attention(q16, k16, v16, s)) < ATTN_TOL[prec]
    assert rel_l2(y, z[f"sdpa_{name}_fp32"]) < REF_TOL[prec]
    assert rel_l2(y, z[f"sdpa_{name}_fp16"]) < REF_TOL[prec]


# edge shapes: one query / one key, keys inside the first 32-column chunk, several
# K/V tiles with a ragged tail, query tiles without a pair partner, d = 8 and 64; the
# odd last tile of each (batch, head) runs paired with the next one's, or alone when
# their count is odd ((3, 1, 64, 33, 8), (1, 3, 300, 300, 64))
@pytest.mark.parametrize("B,H,Nq,Nk,D", [(1, 1, 1, 1, 64), (2, 3, 7, 5, 48), (1, 2, 300, 259, 64),
                                          (1, 1, 129, 385, 16), (3, 1, 64, 33, 8), (1, 8, 257, 128, 48),
                                          (2, 2, 128, 1, 32), (1, 3, 300, 300, 64)])
@pytest.mark.parametrize("prec", ["fp16", "bf16"])
def test_sdpa_shapes_vs_oracle(cuda, B, H, Nq, Nk, D, prec):
    torch = cuda
    import oracle
    from msst_b200 import ops

    rng = np.random.default_rng(B * 1000 + Nq * 7 + Nk + D)
    q = rng.standard_normal((B, H, Nq, D)).astype(np.float32)
    k = rng.standard_normal((B, H, Nk, D)).astype(np.float32)
    v = rng.standard_normal((B, H, Nk, D)).astype(np.float32)
    (tq, q16), (tk, k16), (tv, v16) = (_rounded(torch, a, prec) for a in (q, k, v))
    y = ops.scaled_dot_product_attention(tq.cuda(), tk.cuda(), tv.cuda(), 0.0)
    torch.cuda.synchronize()
    r = oracle.attention(q16, k16, v16, op_cases.default_scale(D))
    assert rel_l2(y.float().cpu().numpy(), r) < ATTN_TOL[prec]


def test_sdpa_large_logits_vs_oracle(cuda):
    """Score ranges far beyond the lazy-rescale threshold (2^8) in the second key
    tile: the exact two-pass path and the O rescale must keep the result exact."""
    torch = cuda
    import oracle
    from msst_b200 import ops

    rng = np.random.default_rng(77)
    B, H, Nq, Nk, D = 1, 2, 130, 300, 48
    q = rng.standard_normal((B, H, Nq, D)).astype(np.float32)
    k = rng.standard_normal((B, H, Nk, D)).astype(np.float32)
    k[:, :, 150:170] *= 6.0
    v = rng.standard_normal((B, H, Nk, D)).astype(np.float32)
    (tq, q16), (tk, k16), (tv, v16) = (_rounded(torch, a, "fp16") for a in (q, k, v))
    y = ops.scaled_dot_product_attention(tq.cuda(), tk.cuda(), tv.cuda(), 0.5)
    torch.cuda.synchronize()
    assert rel_l2(y.float().cpu().numpy(), oracle.attention(q16, k16, v16, 0.5)) < ATTN_TOL["fp16"]


def test_sdpa_rejects_bad_arguments(cuda):
    torch = cuda
    from msst_b200 import MsstError, ops

    q = torch.zeros(1, 1, 4, 72, dtype=torch.float16, device="cuda")
    with pytest.raises(MsstError):
        ops.scaled_dot_product_attention(q, q, q)  # head_dim 72 > 64
    q = torch.zeros(1, 1, 4, 20, dtype=torch.float16, device="cuda")
    with pytest.raises(MsstError):
        ops.scaled_dot_product_attention(q, q, q)  # head_dim not a multiple of 8
    q = torch.zeros(1, 2, 4, 64, dtype=torch.float16, device="cuda")
    k = torch.zeros(1, 1, 4, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError):
        ops.scaled_dot_product_attention(q, k, k)


@pytest.mark.parametrize("out", ["fp32", "fp16", "bf16"])
@pytest.mark.parametrize("name", list(op_cases.LN_CASES))
def test_layer_norm_vs_reference(cuda, name, out):
    torch = cuda
    import oracle
    from msst_b200 import ops

    z, _ = golden("ops_htdemucs.npz")
    x, g, b = op_cases.ln_inputs(name)
    dt = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}[out]
    y = ops.layer_norm(torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda(),
                       op_cases.LN_EPS, dtype=dt)
    torch.cuda.synchronize()
    y = y.float().cpu().numpy()
    tol = {"fp32": 1e-6, "fp16": 1e-3, "bf16": 5e-3}[out]
    assert rel_l2(y, z[f"ln_{name}"]) < tol
    assert rel_l2(y, oracle.layernorm(x, g, b, op_cases.LN_EPS)) < tol


@pytest.mark.parametrize("rows,D", [(1, 4), (5000, 1024), (3, 132), (70001, 384)])
def test_layer_norm_shapes_vs_oracle(cuda, rows, D):
    torch = cuda
    import oracle
    from msst_b200 import ops

    rng = np.random.default_rng(rows + D)
    x = (3.0 + rng.standard_normal((rows, D))).astype(np.float32)
    g = rng.standard_normal(D).astype(np.float32)
    b = rng.standard_normal(D).astype(np.float32)
    y = ops.layer_norm(torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda())
    torch.cuda.synchronize()
    assert rel_l2(y.cpu().numpy(), oracle.layernorm(x, g, b)) < 1e-6
