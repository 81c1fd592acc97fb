"""GPU parity at the benchmarked shapes against the reference engine run on a B200
(tests/golden/cfg{1,2}_ref.npz, written by tests/golden/make_golden.py
--only bench-shapes from oracle/_ref; they hold seeded windows of the output
waveforms and rows of the fp32 masks, the full arrays being hundreds of MB;
tests/golden/config3_ref.npz, written by --only config3, the reference attention's
output for sampled sequence-heads).

* MelBandRoformer D384 x 6, fp16, the bench's own weights and
  68.5 s track, separated exactly as bench.py times it (overlap 0.25, 4 chunks per
  forward); masks of the track's first forward batch.
  Reference graph: src/model_mel_band_roformer.cu:744-1062, chunking
  src/inference_app.cpp:100-324.
* BS-Roformer D512 x 12 with bf16 weights, bf16 operands, one
  forward of 8 chunks of 352800 samples.  Reference graph:
  src/model_bs_roformer.cu:420-609.

* the axial attention alone at B = 4 chunks, T = 801, F = 62,
  8 heads x 64, bf16 q/k/v ~ N(0, 1), both axes.  Reference op:
  src/ops_attention.cu:522-599.

Bars: output waveforms >= 45 dB SNR against the reference's fp32 and fp16 runs;
masks within the stated relative L2 of the reference's fp32 masks; attention
outputs within 1e-2 relative L2.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import golden, rel_l2, snr_db

pytestmark = pytest.mark.gpu

SNR_MIN = 45.0
MASK_TOL = {"fp16": 4e-3, "bf16": 2.5e-2}


def _model(tmp_path_factory, spec):
    from msst_b200 import synth

    cfg = (synth.mbr_config if spec["kind"] == "mbr" else synth.bsr_config)(**spec["cfg"])
    sd = synth.make_weights(cfg, spec["seed"], weight_dtype=spec["weight_dtype"])
    path = str(tmp_path_factory.mktemp("bench_shapes") / "m.csm")
    synth.write_csm(path, cfg, sd)
    return path, cfg


def _report(name, **kv):
    print(f"{name}: " + json.dumps({k: round(v, 6) for k, v in kv.items()}))


def test_config1_separation_vs_reference(cuda, tmp_path_factory):
    torch = cuda
    import oracle
    from msst_b200 import Model, synth

    z, meta = golden("cfg1_ref.npz")
    spec, W = meta["spec"], meta["window"]
    path, cfg = _model(tmp_path_factory, spec)
    n = int(round(spec["track_seconds"] * 44100))
    track = synth.make_audio(n, 2, spec["track_seed"])
    m = Model(path, 0, "fp16")
    y = m.separate(torch.from_numpy(track).cuda(), spec["overlap"], spec["chunk_batch"]).cpu().numpy()
    est = np.stack([y[:, w:w + W] for w in z["windows"]], axis=1)
    # masks of the first forward batch (the plan's first chunk_batch chunks)
    step = oracle.resolve_step(cfg["chunk_size"], spec["overlap"], cfg["num_overlap"])
    first = np.stack(oracle.chunk_inputs(track, cfg["chunk_size"], step)[: spec["chunk_batch"]])
    masks = m.masks(torch.from_numpy(first).cuda()).cpu().numpy()
    m.close()
    rows = masks.reshape(-1, masks.shape[-1])[z["mask_rows"]]
    s32, s16 = snr_db(est, z["out_fp32"]), snr_db(est, z["out_fp16"])
    e32 = rel_l2(rows, z["mask_rows_fp32"])
    _report("config1 fp16", out_snr_db_vs_ref_fp32=s32, out_snr_db_vs_ref_fp16=s16, mask_rel_l2_vs_ref_fp32=e32,
            ref_fp16_vs_ref_fp32_snr_db=snr_db(z["out_fp16"], z["out_fp32"]))
    assert s32 >= SNR_MIN and s16 >= SNR_MIN
    assert e32 < MASK_TOL["fp16"]


def test_config2_forward_vs_reference(cuda, tmp_path_factory):
    torch = cuda
    from msst_b200 import Model, synth

    z, meta = golden("cfg2_ref.npz")
    spec, W = meta["spec"], meta["window"]
    path, cfg = _model(tmp_path_factory, spec)
    B, cs = spec["chunks"], cfg["chunk_size"]
    audio = synth.make_audio(B * cs, 2, spec["audio_seed"])
    audio = np.ascontiguousarray(audio.reshape(2, B, cs).transpose(1, 0, 2))
    m = Model(path, 0, "bf16")
    x = torch.from_numpy(audio).cuda()
    y = m.forward(x).cpu().numpy()
    masks = m.masks(x).cpu().numpy()
    m.close()
    est = np.stack([y[:, :, w:w + W] for w in z["windows"]], axis=2)
    rows = masks.reshape(-1, masks.shape[-1])[z["mask_rows"]]
    s32, s16 = snr_db(est, z["out_fp32"]), snr_db(est, z["out_fp16"])
    e32 = rel_l2(rows, z["mask_rows_fp32"])
    _report("config2 bf16", out_snr_db_vs_ref_fp32=s32, out_snr_db_vs_ref_fp16=s16, mask_rel_l2_vs_ref_fp32=e32,
            ref_fp16_vs_ref_fp32_snr_db=snr_db(z["out_fp16"], z["out_fp32"]))
    assert s32 >= SNR_MIN and s16 >= SNR_MIN
    assert e32 < MASK_TOL["bf16"]


@pytest.mark.parametrize("axis", ["time", "band"])
def test_config3_attention_vs_reference(cuda, axis):
    """BASELINE config 3 at its own shape (B = 4 chunks, T = 801, F = 62, 8 heads x 64, bf16
    q/k/v ~ N(0, 1), scale 1/8): msst_attention against the reference's
    ops::scaled_dot_product_attention (src/ops_attention.cu:522-599) on the same seeded inputs,
    in its fp32 (TF32 QK^T) and fp16-value modes, on the fixture's sampled (sequence, head)
    pairs.  The bar, 1e-2 relative L2, is bf16's output rounding with margin (the reference's
    two modes differ by about 5e-4)."""
    torch = cuda
    import op_cases
    from msst_b200 import ops

    z, meta = golden("config3_ref.npz")
    c = op_cases.CONFIG3
    B, T, F, H, D = c["B"], c["T"], c["F"], c["H"], c["D"]
    q, k, v = op_cases.config3_inputs(axis)

    def token_major(a):
        # [S, H, N, D] -> [B*T*F, H*D] on the token grid (sequence s = b*F + f on the time axis,
        # b*T + t on the band axis)
        t = torch.from_numpy(a).cuda()
        if axis == "time":
            t = t.view(B, F, H, T, D).permute(0, 3, 1, 2, 4)
        else:
            t = t.view(B, T, H, F, D).permute(0, 1, 3, 2, 4)
        return t.reshape(B * T * F, H * D).to(torch.bfloat16)

    qkv = torch.cat([token_major(a) for a in (q, k, v)], dim=1).contiguous()
    del q, k, v
    y = ops.attention(qkv, B, T, F, H, axis, c["scale"]).float()
    torch.cuda.synchronize()
    seq, head = op_cases.config3_samples(axis)
    N = T if axis == "time" else F
    if axis == "time":
        y = y.view(B, T, F, H, D).permute(0, 2, 3, 1, 4).reshape(B * F, H, T, D)
    else:
        y = y.view(B, T, F, H, D).permute(0, 1, 3, 2, 4).reshape(B * T, H, F, D)
    ours = y[torch.from_numpy(seq).cuda(), torch.from_numpy(head).cuda()].cpu().numpy()
    assert ours.shape == (len(seq), N, D)
    e32 = rel_l2(ours, z[f"{axis}_fp32"].astype(np.float32))
    e16 = rel_l2(ours, z[f"{axis}_fp16"].astype(np.float32))
    _report(f"config3 {axis}", rel_l2_vs_ref_fp32=e32, rel_l2_vs_ref_fp16=e16)
    assert e32 < 1e-2 and e16 < 1e-2
