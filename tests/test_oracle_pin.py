"""CPU: the fp32 oracle against the reference engine's own outputs (tests/golden/).

These pin the oracle before it is trusted as the checker of the CUDA path.  The
reference's GEMMs run in TF32, so agreement is at the 1e-3 level for masks and
>= 60 dB for waveforms; its scalar flash kernel and RMSNorm are fp32 and agree
at ~1e-6.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden, rel_l2, snr_db


def oracle_mod():
    import oracle

    return oracle


def test_rmsnorm_pin():
    o = oracle_mod()
    z, _ = golden("ops.npz")
    y = o.rmsnorm(z["rms_x"], z["rms_g"], np.sqrt(np.float32(z["rms_x"].shape[1])))
    assert rel_l2(y, z["rms_out"]) < 1e-6


@pytest.mark.parametrize("act", ["none", "gelu", "sigmoid"])
def test_linear_pin(act):
    o = oracle_mod()
    z, _ = golden("ops.npz")
    y = o.linear(z["rms_x"], z["lin_w"], z["lin_b"], act)
    assert rel_l2(y, z[f"lin_{act}_fp32"]) < 2e-3  # reference GEMM is TF32


@pytest.mark.parametrize("N", [129, 60])
def test_attention_and_rope_pin(N):
    o = oracle_mod()
    z, _ = golden("ops.npz")
    q, k, v = z[f"qkv_{N}"]
    y = o.attention(q, k, v, 0.125)
    assert rel_l2(y, z[f"flash_{N}"]) < 1e-5   # reference scalar fp32 flash kernel
    assert rel_l2(y, z[f"sdpa_{N}_fp32"]) < 2e-3  # reference live path (TF32 QK^T)
    cs, sn = o.rope_tables(N, 64)
    np.testing.assert_allclose(o.rope(q, cs, sn), z[f"rope_q_{N}"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(o.rope(k, cs, sn), z[f"rope_k_{N}"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name", ["mbr_small", "bsr_small"])
def test_model_pin(name):
    o = oracle_mod()
    from msst_b200 import synth

    z, meta = golden(f"{name}_fp32.npz")
    spec = meta["spec"]
    cfg = (synth.mbr_config if spec["kind"] == "mbr" else synth.bsr_config)(**spec["cfg"])
    om = o.Model(cfg, synth.make_weights(cfg, spec["seed"]))
    audio = synth.make_audio(meta["n_samples"], 2, meta["audio_seed"])[None]
    masks, st = om.masks(audio)
    out = om.apply_masks(masks, st)
    assert rel_l2(masks, z["masks"]) < 1e-3
    assert snr_db(out, z["out"]) >= 60.0


def test_chunked_pin():
    o = oracle_mod()
    from msst_b200 import synth

    z, meta = golden("mbr_chunked_fp32.npz")
    cfg = synth.mbr_config(**meta["cfg"])
    om = o.Model(cfg, synth.make_weights(cfg, meta["weights_seed"]))
    track = synth.make_audio(meta["track_len"], 2, meta["track_seed"])
    step = o.resolve_step(meta["cfg"]["chunk_size"], meta["overlap"], 2)
    y = o.separate(lambda a: om.forward(a), track, meta["cfg"]["chunk_size"], step, meta["chunk_batch"])
    assert snr_db(y, z["out"]) >= 60.0


def test_tail_padding_semantics():
    """The reference's contiguous-source read only changes channels > 0 of the final short chunk."""
    o = oracle_mod()
    rng = np.random.default_rng(0)
    mix = rng.standard_normal((2, 1000)).astype(np.float32)
    a = o.tail_chunk(mix, 700, 400, ref_compat=True)
    b = o.tail_chunk(mix, 700, 400, ref_compat=False)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(b[1, :300], mix[1, 700:])
    assert not np.array_equal(a[1], b[1])
    # reflect padding when more than half a chunk remains, zeros otherwise
    np.testing.assert_array_equal(b[0, 300:302], mix[0, [998, 997]])
    c = o.tail_chunk(mix, 900, 400, ref_compat=False)
    assert np.all(c[:, 100:] == 0)


def test_chunk_plan_matches_reference_rules():
    o = oracle_mod()
    step = o.resolve_step(352800, 0.25, 2)
    assert step == 264600
    border, total, starts = o.chunk_plan(3020850, 352800, step)
    assert (border, total, len(starts)) == (88200, 3197250, 13)
    assert o.resolve_step(352800, 0.0, 2) == 176400      # default num_overlap = 2
    assert o.resolve_step(352800, 4.0, 2) == 88200       # overlap >= 1 is num_overlap


@pytest.mark.parametrize("name", ["self48", "cross48", "cross64", "self32"])
def test_sdpa_cross_length_pin(name):
    """ops::scaled_dot_product_attention at head_dim 48 / 32 and Nq != Nk (the shapes
    HTDemucs' transformer feeds it), default scale 1/sqrt(d)."""
    import op_cases

    o = oracle_mod()
    z, _ = golden("ops_htdemucs.npz")
    q, k, v, scale = op_cases.sdpa_inputs(name)
    s = scale if scale != 0.0 else op_cases.default_scale(q.shape[-1])
    assert rel_l2(o.attention(q, k, v, s), z[f"sdpa_{name}_fp32"]) < 2e-3  # reference QK^T is TF32


@pytest.mark.parametrize("name", ["ln384", "ln512", "ln200"])
def test_layernorm_pin(name):
    import op_cases

    o = oracle_mod()
    z, _ = golden("ops_htdemucs.npz")
    x, g, b = op_cases.ln_inputs(name)
    assert rel_l2(o.layernorm(x, g, b, op_cases.LN_EPS), z[f"ln_{name}"]) < 1e-6


@pytest.mark.parametrize("name", ["mbr_opts", "bsr_opts"])
def test_options_pin(name):
    """The oracle against the reference engine on models with its optional switches:
    band tables derived at load, skip connections, a normalised STFT and the output
    padded to the input length (including the reference's padding layout)."""
    import oracle
    from msst_b200 import synth

    z, meta = golden(f"{name}_fp32.npz")
    spec = meta["spec"]
    cfg = (synth.mbr_config if spec["kind"] == "mbr" else synth.bsr_config)(**spec["cfg"])
    sd = synth.make_weights(cfg, spec["seed"], precomputed_bands=spec.get("precomputed_bands", True))
    audio = synth.make_audio(meta["n_samples"], 2, meta["seed"])[None]
    om = oracle.Model(cfg, sd)
    masks, _ = om.masks(audio)
    assert rel_l2(masks, z["masks"]) < 2e-3
    assert snr_db(om.forward(audio), z["out"]) >= 60.0
