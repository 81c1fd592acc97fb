"""GPU parity of the op-level C ABI (msst_rmsnorm, msst_gemm, msst_gemm_qkv_rope,
msst_attention) against fp32 references computed from the same 16-bit inputs,
and against the reference engine's own SDPA outputs (tests/golden/ops.npz).

Tolerances: outputs stored in 16-bit carry one rounding (fp16 2^-11, bf16 2^-8
relative); accumulation is fp32 in both paths.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import golden, rel_l2

pytestmark = pytest.mark.gpu

TOL16 = {"fp16": 2e-3, "bf16": 1.2e-2}


def _dt(torch, name):
    return {"fp16": torch.float16, "bf16": torch.bfloat16}[name]


def oracle_mod():
    import oracle

    return oracle


@pytest.mark.parametrize("prec", ["fp16", "bf16"])
@pytest.mark.parametrize("rows,D", [(1000, 384), (20000, 384), (333, 512), (20001, 512), (1, 512), (8, 128), (1, 256)])
def test_rmsnorm_and_gates(cuda, prec, rows, D):
    torch = cuda
    from msst_b200 import ops

    g = torch.Generator().manual_seed(rows + D)
    x = torch.randn(rows, D, generator=g) * 3
    gamma = 1 + 0.1 * torch.randn(D, generator=g)
    wg = 0.05 * torch.randn(8, D, generator=g)
    bg = 0.02 * torch.randn(8, generator=g)
    scale = float(np.sqrt(np.float32(D)))
    y, gates = ops.rmsnorm(x.cuda(), gamma.cuda(), scale, _dt(torch, prec), wg.cuda(), bg.cuda())
    torch.cuda.synchronize()
    ref = oracle_mod().rmsnorm(x.numpy(), gamma.numpy(), scale)
    assert rel_l2(y.float().cpu().numpy(), ref) < TOL16[prec]
    ref_g = 1 / (1 + np.exp(-(ref.astype(np.float64) @ wg.numpy().T.astype(np.float64) + bg.numpy())))
    np.testing.assert_allclose(gates.cpu().numpy(), ref_g, rtol=0, atol=1e-4)


def test_rmsnorm_matches_reference_engine(cuda):
    torch = cuda
    from msst_b200 import ops

    z, _ = golden("ops.npz")
    x, gmm, ref = z["rms_x"], z["rms_g"], z["rms_out"]
    y, _ = ops.rmsnorm(torch.from_numpy(x).cuda(), torch.from_numpy(gmm).cuda(), float(np.sqrt(np.float32(x.shape[1]))),
                       torch.float16)
    torch.cuda.synchronize()
    assert rel_l2(y.float().cpu().numpy(), ref) < 1e-3


def _lin_ref(x16, w16, b):
    return x16.float() @ w16.float().t() + (b if b is not None else 0)


@pytest.mark.parametrize("prec", ["fp16", "bf16"])
@pytest.mark.parametrize("M,K,N", [(1000, 384, 1536), (300, 1536, 384), (129, 512, 512), (64, 64, 128), (77, 128, 200)])
@pytest.mark.parametrize("act", ["none", "gelu", "tanh", "sigmoid"])
def test_gemm_store16(cuda, prec, M, K, N, act):
    torch = cuda
    from msst_b200 import ops

    g = torch.Generator().manual_seed(M * 7 + N)
    dt = _dt(torch, prec)
    x = torch.randn(M, K, generator=g).to(dt).cuda()
    w = (0.05 * torch.randn(N, K, generator=g)).to(dt).cuda()
    b = (0.05 * torch.randn(N, generator=g)).cuda()
    y = ops.gemm(x, w, b, "store16", act)
    torch.cuda.synchronize()
    r = _lin_ref(x, w, b)
    r = {"none": r, "gelu": torch.nn.functional.gelu(r), "tanh": torch.tanh(r), "sigmoid": torch.sigmoid(r)}[act]
    assert rel_l2(y.float().cpu().numpy(), r.cpu().numpy()) < TOL16[prec]


@pytest.mark.parametrize("prec", ["fp16", "bf16"])
@pytest.mark.parametrize("M,K,N", [(1000, 512, 384), (130, 1536, 512), (5, 64, 96)])
def test_gemm_fp32_epilogues(cuda, prec, M, K, N):
    torch = cuda
    from msst_b200 import ops

    g = torch.Generator().manual_seed(M + K + N)
    dt = _dt(torch, prec)
    x = torch.randn(M, K, generator=g).to(dt).cuda()
    w = (0.05 * torch.randn(N, K, generator=g)).to(dt).cuda()
    b = (0.05 * torch.randn(N, generator=g)).cuda()
    r = _lin_ref(x, w, b)
    y = ops.gemm(x, w, b, "store32")
    torch.cuda.synchronize()
    assert rel_l2(y.cpu().numpy(), r.cpu().numpy()) < 1e-5
    base = torch.randn(M, N, generator=g).cuda()
    out = base.clone()
    ops.gemm(x, w, None, "resid32", out=out)
    torch.cuda.synchronize()
    assert rel_l2(out.cpu().numpy(), (base + _lin_ref(x, w, None)).cpu().numpy()) < 1e-5


@pytest.mark.parametrize("prec", ["fp16", "bf16"])
@pytest.mark.parametrize("N", [56, 1040, 256, 48])
def test_gemm_glu(cuda, prec, N):
    torch = cuda
    from msst_b200 import ops

    g = torch.Generator().manual_seed(N)
    dt = _dt(torch, prec)
    M, K = 301, 1536
    x = torch.randn(M, K, generator=g).to(dt).cuda()
    w = (0.05 * torch.randn(N, K, generator=g)).to(dt).cuda()
    b = (0.05 * torch.randn(N, generator=g)).cuda()
    y = ops.gemm(x, w, b, "glu32")
    torch.cuda.synchronize()
    r = _lin_ref(x, w, b)
    r = r[:, 0::2] * torch.sigmoid(r[:, 1::2])  # columns interleaved (value, gate)
    assert rel_l2(y.cpu().numpy(), r.cpu().numpy()) < 1e-5


# CTA-pair GEMM tiles (cta_group::2 MMAs): by default only the residual GEMMs
# with K >= 512 use them; MSST_GEMM_PAIR=2 (read once per process) routes every
# launch with at least 148 whole-column 256-row pair tiles through them, so the
# other epilogues are checked in a child process.  The sizes include a last pair
# tile whose second CTA's rows lie past M (zero-filled A rows, clipped stores).
PAIR_CASES = [("store16", 37003, 384, 1536), ("store32", 60000, 1536, 384), ("resid32", 60000, 1536, 384),
              ("glu32", 40000, 512, 1024), ("resid32", 48060, 512, 512), ("qkv", 48060, 384, 1536)]


def pair_case_error(epi, M, K, N, prec):
    """rel-L2 error of one pair-tile GEMM against an fp32 torch reference."""
    import torch
    from msst_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(M + N)
    dt = _dt(torch, prec)
    x = torch.randn(M, K, device="cuda", generator=g).to(dt)
    w = (0.05 * torch.randn(N, K, device="cuda", generator=g)).to(dt)
    b = 0.05 * torch.randn(N, device="cuda", generator=g)
    r = _lin_ref(x, w, b)
    if epi == "store16":
        y = ops.gemm(x, w, b, "store16", "gelu")
        r = torch.nn.functional.gelu(r)
    elif epi == "resid32":
        base = torch.randn(M, N, device="cuda", generator=g)
        y = base.clone()
        ops.gemm(x, w, b, "resid32", out=y)
        r = r + base
    elif epi == "glu32":
        y = ops.gemm(x, w, b, "glu32")
        r = r[:, 0::2] * torch.sigmoid(r[:, 1::2])
    elif epi == "qkv":
        T, F, H = 801, 60, 8
        inv = 10000.0 ** (-np.arange(0, 64, 2, dtype=np.float64) / 64)
        ang = np.arange(T, dtype=np.float64)[:, None] * inv[None, :]
        cs, sn = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
        y = ops.gemm_qkv_rope(x, w, H, torch.from_numpy(cs).cuda(), torch.from_numpy(sn).cuda(), F, T)
        r = _lin_ref(x, w, None).view(M, 3, H, 32, 2)
        pos = torch.from_numpy((np.arange(M) // F) % T).cuda()
        c = torch.from_numpy(cs).cuda()[pos][:, None, :]
        s_ = torch.from_numpy(sn).cuda()[pos][:, None, :]
        for part in (0, 1):
            x0, x1 = r[:, part, :, :, 0].clone(), r[:, part, :, :, 1].clone()
            r[:, part, :, :, 0] = x0 * c - x1 * s_
            r[:, part, :, :, 1] = x0 * s_ + x1 * c
        r = r.view(M, N)
    else:
        y = ops.gemm(x, w, b, "store32")
    torch.cuda.synchronize()
    return rel_l2(y.float().cpu().numpy(), r.cpu().numpy())


def _pair_tol(epi, prec):
    return TOL16[prec] if epi in ("store16", "qkv") else 1e-5


@pytest.mark.parametrize("prec", ["fp16", "bf16"])
def test_gemm_pair_tiles_default(cuda, prec):
    """The default policy's pair launches (residual, K >= 512)."""
    for epi, M, K, N in PAIR_CASES:
        if epi == "resid32":
            assert pair_case_error(epi, M, K, N, prec) < _pair_tol(epi, prec), (epi, M, K, N)


def test_gemm_pair_tiles_all_epilogues(cuda):
    import subprocess
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    code = ("import sys; sys.path.insert(0, %r); import conftest, test_kernels_gpu as t\n"
            "bad = []\n"
            "for prec in ('fp16', 'bf16'):\n"
            "    for epi, M, K, N in t.PAIR_CASES:\n"
            "        e = t.pair_case_error(epi, M, K, N, prec)\n"
            "        if not e < t._pair_tol(epi, prec): bad.append((epi, M, K, N, prec, e))\n"
            "print('BAD', bad) if bad else print('OK')\n") % here
    env = dict(os.environ, MSST_GEMM_PAIR="2")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout[-2000:] + r.stderr[-2000:]


@pytest.mark.parametrize("prec", ["fp16", "bf16"])
@pytest.mark.parametrize("axis,shape", [("time", (2, 131, 5, 2, 128)), ("band", (2, 131, 5, 2, 128)),
                                        ("time", (1, 801, 60, 8, 384))])
def test_qkv_rope(cuda, prec, axis, shape):
    torch = cuda
    from msst_b200 import ops

    oracle = oracle_mod()
    B, T, F, H, D = shape
    M = B * T * F
    g = torch.Generator().manual_seed(3)
    dt = _dt(torch, prec)
    x = torch.randn(M, D, generator=g).to(dt).cuda()
    w = (0.1 * torch.randn(3 * H * 64, D, generator=g)).to(dt).cuda()
    npos = T if axis == "time" else F
    cs, sn = oracle.rope_tables(npos, 64)
    pos_div, pos_mod = (F, T) if axis == "time" else (1, F)
    y = ops.gemm_qkv_rope(x, w, H, torch.from_numpy(cs).cuda(), torch.from_numpy(sn).cuda(), pos_div, pos_mod)
    torch.cuda.synchronize()
    r = _lin_ref(x, w, None).cpu().numpy().reshape(M, 3, H, 64)
    pos = (np.arange(M) // pos_div) % pos_mod
    for part in (0, 1):
        v = r[:, part].copy()  # [M, H, 64]
        c, s = cs[pos][:, None, :], sn[pos][:, None, :]
        x0, x1 = v[..., 0::2].copy(), v[..., 1::2].copy()
        v[..., 0::2] = x0 * c - x1 * s
        v[..., 1::2] = x0 * s + x1 * c
        r[:, part] = v
    assert rel_l2(y.float().cpu().numpy(), r.reshape(M, -1)) < TOL16[prec]


def _attn_ref(qkv, B, T, F, H, axis, scale, gates):
    """fp32 reference on the [B,T,F] token grid; qkv [M, 3*H*64]."""
    import torch

    q, k, v = qkv.float().view(B, T, F, 3, H, 64).unbind(3)
    if axis == "time":
        perm = lambda t: t.permute(0, 2, 3, 1, 4)  # [B,F,H,T,64]
    else:
        perm = lambda t: t.permute(0, 1, 3, 2, 4)  # [B,T,H,F,64]
    q, k, v = perm(q), perm(k), perm(v)
    p = torch.softmax((q @ k.transpose(-1, -2)) * scale, dim=-1)
    o = p @ v
    o = o.permute(0, 3, 1, 2, 4) if axis == "time" else o.permute(0, 1, 3, 2, 4)  # [B,T,F,H,64]
    if gates is not None:
        o = o * gates.view(B, T, F, H, 1)
    return o.reshape(B * T * F, H * 64)


@pytest.mark.parametrize("prec", ["fp16", "bf16"])
# time axis: (2, 801, 3, 2) pairs the 33-row tail tiles of 12 units; (1, 801, 3, 1) and (1, 300, 1, 3) leave an odd
# unit's tail alone; (1, 100, 2, 8) has only tail tiles
@pytest.mark.parametrize("axis,B,T,F,H", [("time", 2, 801, 3, 2), ("time", 1, 100, 2, 8), ("time", 1, 256, 1, 1),
                                           ("time", 1, 801, 3, 1), ("time", 1, 300, 1, 3),
                                           ("band", 2, 50, 60, 2), ("band", 1, 33, 62, 8), ("band", 3, 7, 5, 1),
                                           ("band", 1, 20, 100, 2), ("band", 2, 9, 32, 2), ("band", 1, 11, 33, 1),
                                           ("band", 1, 5, 128, 1), ("band", 1, 40, 1, 1)])
def test_attention(cuda, prec, axis, B, T, F, H):
    torch = cuda
    from msst_b200 import ops

    g = torch.Generator().manual_seed(B * T + F)
    dt = _dt(torch, prec)
    M = B * T * F
    qkv = torch.randn(M, 3 * H * 64, generator=g).to(dt).cuda()
    gates = torch.rand(M, H, generator=g).cuda()
    y = ops.attention(qkv, B, T, F, H, axis, 0.125, gates)
    torch.cuda.synchronize()
    r = _attn_ref(qkv, B, T, F, H, axis, 0.125, gates)
    tol = {"fp16": 3e-3, "bf16": 1.5e-2}[prec]
    assert rel_l2(y.float().cpu().numpy(), r.cpu().numpy()) < tol


@pytest.mark.parametrize("N", [129, 60])
def test_attention_matches_reference_engine(cuda, N):
    """Our attention vs the reference's live SDPA (TF32 QK^T) and its scalar flash kernel."""
    torch = cuda
    from msst_b200 import ops

    z, _ = golden("ops.npz")
    q, k, v = z[f"qkv_{N}"]
    B, H, _, D = q.shape
    # pack as a QKV buffer: time axis with F = 1 (N = T) or band axis with T = 1 (N = F)
    qkv = np.concatenate([t.transpose(0, 2, 1, 3).reshape(B, N, H * D) for t in (q, k, v)], axis=-1)
    qkv = torch.from_numpy(qkv.reshape(B * N, -1)).half().cuda()
    if N > 64:
        y = ops.attention(qkv, B, N, 1, H, "time", 0.125)
    else:
        y = ops.attention(qkv, B, 1, N, H, "band", 0.125)
    torch.cuda.synchronize()
    y = y.float().cpu().numpy().reshape(B, N, H, D).transpose(0, 2, 1, 3)
    assert rel_l2(y, z[f"sdpa_{N}_fp32"]) < 3e-3
    assert rel_l2(y, z[f"sdpa_{N}_fp16"]) < 3e-3
    assert rel_l2(y, z[f"flash_{N}"]) < 3e-3


def test_linear_matches_reference_engine(cuda):
    torch = cuda
    from msst_b200 import ops

    z, _ = golden("ops.npz")
    x = torch.from_numpy(z["rms_x"]).half().cuda()
    w = torch.from_numpy(z["lin_w"]).half().cuda()
    b = torch.from_numpy(z["lin_b"]).cuda()
    for act in ("none", "gelu", "sigmoid"):
        y = ops.gemm(x, w, b, "store16", act)
        torch.cuda.synchronize()
        assert rel_l2(y.float().cpu().numpy(), z[f"lin_{act}_fp16"]) < 2e-3
        assert rel_l2(y.float().cpu().numpy(), z[f"lin_{act}_fp32"]) < 3e-3


def test_kernel_timing_records_launches(cuda):
    """msst_kernel_timing brackets each launch with events and tags it with its algorithmic cost."""
    torch = cuda
    from msst_b200 import kernel_timing, kernel_timing_report, ops

    M, K, N = 4096, 384, 1536
    x = torch.randn(M, K, device="cuda").half()
    w = (0.02 * torch.randn(N, K, device="cuda")).half()
    kernel_timing(True)
    for _ in range(3):
        ops.gemm(x, w, None, "store16", "gelu")
    kernel_timing(False)
    ops.gemm(x, w, None, "store16", "gelu")  # not recorded
    rep = kernel_timing_report()
    assert set(rep) == {"gemm_store16_gelu"}
    k = rep["gemm_store16_gelu"]
    assert k["launches"] == 3
    assert k["flop"] == pytest.approx(3 * 2.0 * M * N * K)
    assert k["bytes"] == pytest.approx(3 * ((M * K + N * K) * 2.0 + M * N * 2.0))
    assert 0.0 < k["total_ms"] < 1000.0
    kernel_timing(True)  # restarting discards the records
    kernel_timing(False)
    assert kernel_timing_report() == {}
