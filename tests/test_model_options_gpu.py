"""GPU parity of the reference drivers' optional config switches against the
reference engine's own outputs (tests/golden/{mbr,bsr}_opts_*.npz, written by
tests/golden/make_golden.py --only options from oracle/_ref on a B200):

* a MelBandRoformer .csm without __precomputed__ band tables (the band tables
  are then derived at load, src/model_mel_band_roformer.cu:214-313,377);
* skip_connection (src/model_mel_band_roformer.cu:846-852,898-901,
  src/model_bs_roformer.cu:478-531);
* stft_normalized (src/ops_stft.cu:358-365,380-389);
* match_input_audio_length with an input that is not a multiple of hop_length
  (src/model_mel_band_roformer.cu:764,1021, src/ops_stft.cu:484-493).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden, rel_l2, snr_db

pytestmark = pytest.mark.gpu

MASK_TOL = {"fp16": 4e-3, "bf16": 2.5e-2}


@pytest.fixture(scope="module")
def option_models(tmp_path_factory):
    from msst_b200 import synth

    out = {}
    for name in ("mbr_opts", "bsr_opts"):
        _, meta = golden(f"{name}_fp32.npz")
        spec = meta["spec"]
        cfg = (synth.mbr_config if spec["kind"] == "mbr" else synth.bsr_config)(**spec["cfg"])
        sd = synth.make_weights(cfg, spec["seed"], precomputed_bands=spec.get("precomputed_bands", True))
        path = str(tmp_path_factory.mktemp("opts") / f"{name}.csm")
        synth.write_csm(path, cfg, sd)
        out[name] = (path, cfg, meta)
    return out


@pytest.mark.parametrize("prec", ["fp16"])
@pytest.mark.parametrize("name", ["mbr_opts", "bsr_opts"])
def test_options_vs_reference(cuda, option_models, name, prec):
    torch = cuda
    from msst_b200 import Model, synth

    path, cfg, meta = option_models[name]
    audio = synth.make_audio(meta["n_samples"], 2, meta["seed"])[None]
    m = Model(path, 0, prec)
    info = m.info
    assert info["skip_connection"] == 1 and info["stft_normalized"] == 1 and info["match_input_audio_length"] == 1
    assert info["bands_from_file"] == (0 if name == "mbr_opts" else 1)
    x = torch.from_numpy(audio).cuda()
    masks = m.masks(x).cpu().numpy()
    y = m.forward(x).cpu().numpy()
    m.close()
    zf, _ = golden(f"{name}_fp32.npz")
    zh, _ = golden(f"{name}_fp16.npz")
    assert y.shape == zf["out"].shape and y.shape[-1] == meta["n_samples"]
    assert masks.shape == zf["masks"].shape
    err = rel_l2(masks, zf["masks"])
    s32, s16 = snr_db(y, zf["out"]), snr_db(y, zh["out"])
    print(f"{name} {prec}: masks rel-L2 {err:.2e} vs reference fp32; output {s32:.1f} dB vs fp32, {s16:.1f} dB vs fp16")
    assert err < MASK_TOL[prec]
    assert s32 >= 45.0 and s16 >= 45.0
    # the samples past the reconstructed (L // hop) * hop are the zero padding of ops::istft
    tail = (meta["n_samples"] // cfg["stft_hop_length"]) * cfg["stft_hop_length"]
    assert np.all(y[..., tail:] == 0.0)


@pytest.mark.parametrize("name", ["mbr_opts", "bsr_opts"])
def test_options_bf16_checkpoint_vs_oracle(cuda, option_models, name, tmp_path):
    """The same switches on bf16 operands, with a bf16 checkpoint (weights that are
    bf16 values: the reference fixtures' fp32 weights would be rounded by the bf16
    path itself), against the fp32 oracle on the same weights."""
    torch = cuda
    import oracle
    from msst_b200 import Model, synth

    _, cfg, meta = option_models[name]
    spec = meta["spec"]
    sd = synth.make_weights(cfg, spec["seed"], precomputed_bands=spec.get("precomputed_bands", True),
                            weight_dtype="bf16")
    path = str(tmp_path / f"{name}_bf16w.csm")
    synth.write_csm(path, cfg, sd)
    audio = synth.make_audio(meta["n_samples"], 2, meta["seed"])[None]
    m = Model(path, 0, "bf16")
    y = m.forward(torch.from_numpy(audio).cuda()).cpu().numpy()
    m.close()
    snr = snr_db(y, oracle.Model(cfg, sd).forward(audio))
    print(f"{name} bf16 checkpoint: output {snr:.1f} dB vs the fp32 oracle")
    assert snr >= 45.0


def _device_ints(ptr: int, n: int) -> np.ndarray:
    """Copy n int32 values from a device pointer (a model-owned table) to the host."""
    from cuda.bindings import runtime as rt

    out = np.zeros(n, np.int32)
    (err,) = rt.cudaMemcpy(out.ctypes.data, ptr, 4 * n, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == rt.cudaError_t.cudaSuccess, err
    return out


def test_computed_mel_bands_match_oracle(cuda, option_models):
    """The band tables derived at load equal the oracle's restatement of the reference's fallback."""
    import oracle
    from msst_b200 import Model

    path, cfg, _ = option_models["mbr_opts"]
    m = Model(path, 0, "fp16")
    t = m.band_tables()
    nfreq_ref, bins_ref, _ = oracle.mel_bands_htk(cfg["sample_rate"], cfg["stft_n_fft"], cfg["num_bands"])
    cuda.cuda.synchronize()
    assert t.num_bands == cfg["num_bands"]
    np.testing.assert_array_equal(_device_ints(t.nfreq, t.num_bands), nfreq_ref)
    np.testing.assert_array_equal(_device_ints(t.bin_list, int(nfreq_ref.sum())), bins_ref)
    m.close()


@pytest.mark.parametrize("name", ["mbr_opts", "bsr_opts"])
def test_fixed_length_padding_vs_oracle(cuda, option_models, name):
    """msst_model_separate on a short track (one whole-track forward) with
    MSST_SEPARATE_FIX_TAIL_PADDING pads every output row with its own samples; the
    oracle's ref_compat=False gives the same semantics."""
    torch = cuda
    import oracle
    from msst_b200 import Model, synth

    path, cfg, meta = option_models[name]
    audio = synth.make_audio(meta["n_samples"], 2, meta["seed"])
    m = Model(path, 0, "fp16")
    y = m.separate(torch.from_numpy(audio).cuda(), fix_tail_padding=True).cpu().numpy()
    m.close()
    sd = synth.make_weights(cfg, meta["spec"]["seed"], precomputed_bands=meta["spec"].get("precomputed_bands", True))
    ref = oracle.Model(cfg, sd).forward(audio[None], ref_compat=False)[0]
    assert y.shape == ref.shape
    assert snr_db(y, ref) >= 45.0
