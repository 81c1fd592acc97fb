"""GPU parity of the block- and op-level entry points on top of the kernels:
msst_grouped_gemm, msst_roformer_attn_block / msst_roformer_ffn_block,
msst_band_gather and msst_mask_apply (with msst_model_band_tables).

References: fp32 torch restatements of the same math on the same 16-bit inputs
(grouped GEMM), the fp32 CPU oracle (attention and feed-forward blocks, band
gather, mask merge), and the library's whole-transformer entry point (block
composition, bit-identical because it runs the same kernels in the same order).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu


def _groups():
    # packed x [300, 320], W [700, 256], out [400, 512]; disjoint output blocks.  The
    # third group's block ends at the last row and column of out, so its m (112)
    # and n (120) need not be multiples of 32.
    return [
        dict(m=96, a_row0=0, a_col0=0, k=128, n=96, b_row0=0, b_col0=64, out_row0=0, out_col0=0),
        dict(m=160, a_row0=120, a_col0=192, k=128, n=192, b_row0=100, b_col0=128, out_row0=96, out_col0=96),
        dict(m=112, a_row0=164, a_col0=64, k=64, n=120, b_row0=400, b_col0=0, out_row0=288, out_col0=392),
        dict(m=64, a_row0=200, a_col0=256, k=64, n=256, b_row0=300, b_col0=192, out_row0=288, out_col0=0),
    ]


def _ref_block(x, w, g, bias, act):
    import torch

    a = x[g["a_row0"]:g["a_row0"] + g["m"], g["a_col0"]:g["a_col0"] + g["k"]].float()
    b = w[g["b_row0"]:g["b_row0"] + g["n"], g["b_col0"]:g["b_col0"] + g["k"]].float()
    y = a @ b.T
    if bias is not None:
        y = y + bias
    if act == "gelu":
        y = torch.nn.functional.gelu(y)
    return y


@pytest.mark.parametrize("prec", ["fp16", "bf16"])
@pytest.mark.parametrize("epi,act", [("store16", "gelu"), ("store32", "none"), ("resid32", "none"), ("glu32", "none")])
def test_grouped_gemm(cuda, prec, epi, act):
    torch = cuda
    from msst_b200 import ops

    dt = torch.float16 if prec == "fp16" else torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(300, 320, device="cuda", generator=g).to(dt)
    w = (0.1 * torch.randn(700, 256, device="cuda", generator=g)).to(dt)
    groups = _groups()
    for q in groups:
        q["bias"] = 0.1 * torch.randn(q["n"], device="cuda", generator=g)
    odt = dt if epi == "store16" else torch.float32
    if epi == "resid32":
        out0 = torch.randn(400, 512, device="cuda", generator=g)
    else:
        out0 = torch.zeros(400, 512, device="cuda", dtype=odt)
    out = out0.clone()
    ops.grouped_gemm(x, w, groups, out, epi, act)
    torch.cuda.synchronize()
    exp = out0.float().clone()
    for q in groups:
        y = _ref_block(x, w, q, q["bias"], act)
        r0, c0 = q["out_row0"], q["out_col0"]
        if epi == "glu32":
            exp[r0:r0 + q["m"], c0:c0 + q["n"] // 2] = y[:, 0::2] * torch.sigmoid(y[:, 1::2])
        elif epi == "resid32":
            exp[r0:r0 + q["m"], c0:c0 + q["n"]] += y
        else:
            exp[r0:r0 + q["m"], c0:c0 + q["n"]] = y
    tol = (2e-3 if prec == "fp16" else 1.2e-2) if epi == "store16" else 1e-5
    # the whole matrix: blocks computed, everything else untouched
    assert rel_l2(out.float().cpu().numpy(), exp.cpu().numpy()) < tol


def test_grouped_gemm_rejects_bad_groups(cuda):
    torch = cuda
    from msst_b200 import MsstError, ops

    x = torch.zeros(64, 64, device="cuda", dtype=torch.float16)
    w = torch.zeros(64, 64, device="cuda", dtype=torch.float16)
    out = torch.zeros(64, 64, device="cuda", dtype=torch.float16)
    bad = [
        dict(m=65, n=64, k=64),                         # A rows outside x
        dict(m=64, n=64, k=64, b_col0=8),               # B columns outside W
        dict(m=32, n=32, k=64, out_col0=4),             # 16-bit output block not on 16 bytes
        dict(m=16, n=32, k=64),                         # partial 32-row box inside out
        dict(m=32, n=32, k=32),                         # k not a multiple of 64
    ]
    for q in bad:
        with pytest.raises(MsstError):
            ops.grouped_gemm(x, w, [q], out)
    torch.cuda.synchronize()


def _model(tmp_path_factory, kind, cfg_kw, seed):
    from msst_b200 import synth

    cfg = (synth.mbr_config if kind == "mbr" else synth.bsr_config)(**cfg_kw)
    path = str(tmp_path_factory.mktemp("blocks") / f"{kind}_{seed}.csm")
    sd = synth.make_weights(cfg, seed)
    synth.write_csm(path, cfg, sd)
    return path, cfg, sd


@pytest.mark.parametrize("dim,T", [(128, 40), (384, 801), (512, 801)])
@pytest.mark.parametrize("axis", ["time", "band"])
def test_blocks_compose_to_transformer(cuda, tmp_path_factory, axis, dim, T):
    """BS-Roformer (no per-transformer final norm): attention + feed-forward blocks
    over all layers are bit-identical to msst_model_transformer, also at T = 801
    (388 row tiles: several per CTA of the persistent kernels)."""
    torch = cuda
    from msst_b200 import Model

    kw = dict(depth=1, dim=dim, time_transformer_depth=2, freq_transformer_depth=2)
    path, cfg, _ = _model(tmp_path_factory, "bsr", kw, 3)
    m = Model(path, 0, "bf16")
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(1, T, m.info["num_bands"], m.info["dim"], device="cuda", generator=g)
    ref = m.transformer(0, axis, x.clone())
    y = x.clone()
    layers = cfg["time_transformer_depth"] if axis == "time" else cfg["freq_transformer_depth"]
    for layer in range(layers):
        m.attn_block(0, axis, layer, y)
        m.ffn_block(0, axis, layer, y)
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    m.close()


def test_attn_and_ffn_block_vs_oracle(cuda, tmp_path_factory):
    torch = cuda
    import oracle
    from msst_b200 import Model, MsstError

    path, cfg, sd = _model(tmp_path_factory, "mbr", dict(depth=1, dim=128), 11)
    om = oracle.Model(cfg, sd)
    m = Model(path, 0, "fp16")
    B, T, nb, D = 1, 40, m.info["num_bands"], m.info["dim"]
    rng = np.random.default_rng(4)
    x = rng.standard_normal((B, T, nb, D)).astype(np.float32)
    xt = torch.from_numpy(x.copy()).cuda()
    m.attn_block(0, "time", 0, xt)
    ya = xt.cpu().numpy()
    xr = np.ascontiguousarray(x.transpose(0, 2, 1, 3)).reshape(B * nb, T, D)
    ra = (xr + om.attention_block(xr, "layers.0.0.layers.0.0", T)).reshape(B, nb, T, D).transpose(0, 2, 1, 3)
    assert rel_l2(ya, ra) < 3e-3
    m.ffn_block(0, "time", 0, xt)
    yf = xt.cpu().numpy()
    ya_r = np.ascontiguousarray(ya.transpose(0, 2, 1, 3)).reshape(B * nb, T, D)
    rf = (ya_r + om.ff_block(ya_r, "layers.0.0.layers.0.1")).reshape(B, nb, T, D).transpose(0, 2, 1, 3)
    assert rel_l2(yf, rf) < 3e-3
    with pytest.raises(MsstError):
        m.attn_block(0, "time", 5, xt)
    m.close()


@pytest.mark.parametrize("dim", [128, 256, 384])
def test_ffn_block_large_vs_oracle(cuda, tmp_path_factory, dim):
    """Feed-forward block at M = 801 x 60 = 48060 rows (376 row tiles, several per CTA of
    the fused kernel at dims <= 384; the CTAs take equal runs of (tile, hidden chunk)
    units, so some tiles are split between two CTAs whose partial sums are added in a
    fixed order: two runs give the same bits)."""
    torch = cuda
    import oracle
    from msst_b200 import Model

    path, cfg, sd = _model(tmp_path_factory, "mbr", dict(depth=1, dim=dim), 17 + dim)
    om = oracle.Model(cfg, sd)
    m = Model(path, 0, "fp16")
    B, T, nb, D = 1, 801, m.info["num_bands"], m.info["dim"]
    rng = np.random.default_rng(dim)
    x = rng.standard_normal((B, T, nb, D)).astype(np.float32)
    xt = torch.from_numpy(x.copy()).cuda()
    m.ffn_block(0, "time", 0, xt)
    y = xt.cpu().numpy()
    xr = np.ascontiguousarray(x.transpose(0, 2, 1, 3)).reshape(B * nb, T, D)
    r = (xr + om.ff_block(xr, "layers.0.0.layers.0.1")).reshape(B, nb, T, D).transpose(0, 2, 1, 3)
    assert rel_l2(y, r) < 3e-3
    for _ in range(2):
        x2 = torch.from_numpy(x.copy()).cuda()
        m.ffn_block(0, "time", 0, x2)
        assert torch.equal(x2, xt)
    m.close()


def _spec_cufft(om, audio):
    """The oracle STFT in the library's cuFFT R2C layout: [B*C*T, nbins, 2]."""
    import oracle

    cfg = om.cfg
    B, C, L = audio.shape
    st = oracle.stft(audio.reshape(B * C, L), cfg["stft_n_fft"], cfg["stft_hop_length"], om.win)  # [BC, F, T, 2]
    return np.ascontiguousarray(st.transpose(0, 2, 1, 3)).reshape(-1, st.shape[1], 2)


@pytest.mark.parametrize("kind", ["mbr", "bsr"])
def test_band_gather_vs_oracle(cuda, tmp_path_factory, kind):
    torch = cuda
    import oracle
    from msst_b200 import Model, ops, synth

    path, cfg, sd = _model(tmp_path_factory, kind, dict(depth=1, dim=128), 5)
    om = oracle.Model(cfg, sd)
    m = Model(path, 0, "fp16")
    t = m.band_tables()
    audio = synth.make_audio(22050, 2, 3)[None]
    B, T = 1, 22050 // cfg["stft_hop_length"] + 1
    spec = torch.from_numpy(_spec_cufft(om, audio)).cuda()
    out = ops.band_gather(spec, B, T, t, torch.float16).float().cpu().numpy()
    xin = om.band_input(om.stft_repr(audio)).reshape(B * T, -1)
    col, off = 0, 0
    for b, d in enumerate(om.dims):
        ref = oracle.rmsnorm(xin[:, off:off + d], om._w(f"band_split.to_features.{b}.0.gamma"),
                             np.sqrt(np.float32(d)))
        assert rel_l2(out[:, col:col + d], ref) < 2e-3, b
        pad = ((d + 63) // 64) * 64
        assert not out[:, col + d:col + pad].any()  # zero K padding
        col += pad
        off += d
    assert col == t.sum_kpad
    m.close()


@pytest.mark.parametrize("kind", ["mbr", "bsr"])
def test_mask_apply_vs_oracle(cuda, tmp_path_factory, kind):
    torch = cuda
    import oracle
    from msst_b200 import Model, ops, synth

    path, cfg, sd = _model(tmp_path_factory, kind, dict(depth=1, dim=128), 6)
    om = oracle.Model(cfg, sd)
    m = Model(path, 0, "fp16")
    t = m.band_tables()
    audio = synth.make_audio(22050, 2, 4)[None]
    B, S, C = 1, m.info["num_stems"], 2
    T = 22050 // cfg["stft_hop_length"] + 1
    st = om.stft_repr(audio)  # [B, F*C, T, 2]
    spec = torch.from_numpy(_spec_cufft(om, audio)).cuda()
    rng = np.random.default_rng(8)
    masks = rng.standard_normal((B, S, T, t.sum_dims)).astype(np.float32)  # the model's masks layout
    mk = torch.from_numpy(np.ascontiguousarray(masks.transpose(1, 0, 2, 3)).reshape(S, B * T, -1)).cuda()
    out = ops.mask_apply(spec, mk, B, S, T, t).cpu().numpy()  # [B*S*C, T, F, 2]
    # the merge half of the oracle's apply_masks, restated
    FC = st.shape[1]
    F = FC // C
    if om.mel:
        nf = len(om.freq_indices)
        mm = masks.reshape(B, S, T, nf, 2).transpose(0, 1, 3, 2, 4)
        summed = np.zeros((B, S, FC, T, 2), np.float32)
        np.add.at(summed, (slice(None), slice(None), om.freq_indices), mm)
        mm = summed / np.maximum(om.nbpf, np.float32(1e-8))[None, None, :, None, None]
    else:
        mm = masks.reshape(B, S, T, FC, 2).transpose(0, 1, 3, 2, 4)
    a = st[:, None]
    ref = np.empty((B, S, FC, T, 2), np.float32)
    ref[..., 0] = a[..., 0] * mm[..., 0] - a[..., 1] * mm[..., 1]
    ref[..., 1] = a[..., 0] * mm[..., 1] + a[..., 1] * mm[..., 0]
    ref = ref.reshape(B, S, F, C, T, 2).transpose(0, 1, 3, 4, 2, 5).reshape(B * S * C, T, F, 2)
    if cfg.get("zero_dc", True):
        ref[:, :, 0] = 0.0
    assert rel_l2(out, ref) < 1e-5
    m.close()


# (kind, model kwargs, precision, T): band counts 60 / 62 (slot 64) and 32 (slot 32),
# widths 128 / 384 / 512 (the last with the 2-stage weight ring), an odd number of
# band sequences (a half-empty last tile) and T = 801 (many tiles per CTA)
BAND_CASES = [
    ("mbr", dict(depth=1, dim=128), "fp16", 41),
    ("bsr", dict(depth=1, dim=384), "fp16", 801),
    ("bsr", dict(depth=1, dim=512), "bf16", 57),
    ("mbr", dict(depth=1, dim=256, num_bands=32), "fp16", 33),
]


@pytest.mark.parametrize("kind,kw,prec,T", BAND_CASES)
def test_band_attention_block_vs_oracle(cuda, tmp_path_factory, kind, kw, prec, T):
    """The band-axis attention block (QKV projection, rotary, attention, gates and
    head merge in one kernel, band_attn.cu) against the fp32 oracle."""
    torch = cuda
    import oracle
    from msst_b200 import Model, device_error

    path, cfg, sd = _model(tmp_path_factory, kind, kw, 23 + kw["dim"])
    om = oracle.Model(cfg, sd)
    m = Model(path, 0, prec)
    B, nb, D = 1, m.info["num_bands"], m.info["dim"]
    rng = np.random.default_rng(T)
    x = rng.standard_normal((B, T, nb, D)).astype(np.float32)
    xt = torch.from_numpy(x.copy()).cuda()
    m.attn_block(0, "band", 0, xt)
    y = xt.cpu().numpy()
    xb = x.reshape(B * T, nb, D)
    r = (xb + om.attention_block(xb, "layers.0.1.layers.0.0", nb)).reshape(B, T, nb, D)
    assert device_error(True) == 0
    assert rel_l2(y, r) < {"fp16": 3e-3, "bf16": 1.5e-2}[prec]
    m.close()
