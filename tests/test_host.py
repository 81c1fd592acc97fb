"""CPU: host-side logic — synthetic models, the .csm container, the C ABI exports."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def test_mel_band_tables():
    from msst_b200 import synth

    mb = synth.mel_bands(44100, 2048, 60, True)
    dims = mb.band_freq_dims(2)
    assert len(mb.freq_indices) == 3958
    assert sum(dims) == 7916 and min(dims) == 24 and max(dims) == 520
    assert mb.num_bands_per_freq.max() == 2 and mb.num_bands_per_freq.min() >= 1
    # stereo interleave: (f*2, f*2+1)
    fi = mb.freq_indices.reshape(-1, 2)
    assert np.all(fi[:, 1] == fi[:, 0] + 1) and np.all(fi[:, 0] % 2 == 0)


def test_bsr_bands():
    from msst_b200 import synth

    assert sum(synth.BSR_FREQS_PER_BANDS) == 1025 and len(synth.BSR_FREQS_PER_BANDS) == 62
    assert sum(synth.band_dims(synth.bsr_config())) == 4100


@pytest.mark.parametrize("half", [False, True])
def test_csm_roundtrip(tmp_path, half):
    from msst_b200 import synth

    cfg = synth.mbr_config(depth=1, dim=128)
    sd = synth.make_weights(cfg, 1)
    p = str(tmp_path / "m.csm")
    synth.write_csm(p, cfg, sd, half=half)
    cfg2, sd2 = synth.read_csm(p)
    assert cfg2 == cfg and set(sd2) == set(sd)
    for k, v in sd.items():
        if v.dtype == np.int64:
            np.testing.assert_array_equal(sd2[k], v)
        else:
            np.testing.assert_allclose(sd2[k].astype(np.float32), v, rtol=1e-3 if half else 0, atol=1e-4 if half else 0)


def test_weight_names_match_reference_loaders():
    """Every tensor the reference drivers bind (src/model_mel_band_roformer.cu:391-471) is present."""
    from msst_b200 import synth

    cfg = synth.mbr_config(depth=2, dim=128)
    sd = synth.make_weights(cfg, 0)
    for d in range(2):
        for t in range(2):
            tp = f"layers.{d}.{t}"
            for n in ("layers.0.0.norm.gamma", "layers.0.0.to_qkv.weight", "layers.0.0.to_gates.weight",
                      "layers.0.0.to_gates.bias", "layers.0.0.to_out.0.weight", "layers.0.1.net.0.gamma",
                      "layers.0.1.net.1.weight", "layers.0.1.net.1.bias", "layers.0.1.net.4.weight",
                      "layers.0.1.net.4.bias", "norm.gamma"):
                assert f"{tp}.{n}" in sd
    # MBR mask MLP has mask_estimator_depth + 1 = 3 linears; the last doubles the band's dims for the GLU
    assert sd["mask_estimators.0.to_freqs.0.0.4.weight"].shape[0] == 2 * synth.band_dims(cfg)[0]


def header_symbols():
    text = open(os.path.join(ROOT, "include", "msst_b200.h")).read()
    return sorted(set(re.findall(r"\b(msst_[a-z0-9_]+)\s*\(", text)))


def test_c_abi_exports_every_declared_symbol():
    from msst_b200 import EXPORTS, LIB_PATH, lib

    assert os.path.exists(LIB_PATH), "libmsst_b200.so not built"
    L = lib()
    declared = header_symbols()
    assert len(declared) >= 15
    for name in declared:
        assert hasattr(L, name), f"{name} declared in msst_b200.h but not exported"
    assert set(declared) == set(EXPORTS)


def test_c_abi_error_paths_without_gpu(tmp_path):
    from msst_b200 import MSST_ERR_IO, MsstError, lib

    L = lib()
    h = ctypes.c_void_p()
    rc = L.msst_model_load(str(tmp_path / "missing.csm").encode(), 0, 0, ctypes.byref(h))
    assert rc == MSST_ERR_IO and b"cannot open" in L.msst_last_error()
    bad = tmp_path / "bad.csm"
    bad.write_bytes(b"NOPE" + b"\0" * 16)
    assert L.msst_model_load(str(bad).encode(), 0, 0, ctypes.byref(h)) == MSST_ERR_IO
    assert b"magic" in L.msst_last_error()
    assert L.msst_version() >= 1
    with pytest.raises(MsstError):
        from msst_b200 import check

        check(MSST_ERR_IO)


def test_shared_op_argument_checks_without_gpu():
    """msst_sdpa / msst_layernorm reject bad shapes before touching a device."""
    from msst_b200 import BF16, F16, F32, MSST_ERR_INVALID, lib

    L = lib()
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    assert L.msst_sdpa(None, p, p, 1, 1, 4, 4, 64, 0.0, F16, p, None) == MSST_ERR_INVALID
    assert L.msst_sdpa(p, p, p, 1, 1, 4, 4, 72, 0.0, F16, p, None) == MSST_ERR_INVALID
    assert b"head_dim" in L.msst_last_error()
    assert L.msst_sdpa(p, p, p, 1, 1, 4, 4, 20, 0.0, BF16, p, None) == MSST_ERR_INVALID
    assert L.msst_sdpa(p, p, p, 1, 1, 0, 4, 64, 0.0, F16, p, None) == MSST_ERR_INVALID
    assert L.msst_sdpa(p, p, p, 1, 1, 4, 4, 64, 0.0, F32, p, None) == MSST_ERR_INVALID
    assert L.msst_layernorm(p, 4, 6, p, p, 1e-5, F32, p, None) == MSST_ERR_INVALID
    assert L.msst_layernorm(p, 4, 2048, p, p, 1e-5, F16, p, None) == MSST_ERR_INVALID
    assert L.msst_layernorm(p, 4, 384, p, p, 1e-5, 7, p, None) == MSST_ERR_INVALID
    assert L.msst_layernorm(None, 4, 384, p, p, 1e-5, F32, p, None) == MSST_ERR_INVALID


def test_library_has_no_cpu_fallback_symbols():
    """The product library links no oracle code."""
    out = os.popen(f"nm -D {os.path.join(ROOT, 'cuda-msst-infer_b200', 'msst_b200', 'lib', 'libmsst_b200.so')}").read()
    assert "msst_oracle" not in out and "refh_" not in out


def test_kernel_timing_api_without_gpu():
    """Timing on/off and an empty report need no device; the report is keyed by kernel name."""
    from msst_b200 import kernel_launches, kernel_timing, kernel_timing_report

    kernel_timing(True)
    kernel_timing(False)
    assert kernel_timing_report() == {}
    assert kernel_launches(reset=True) >= 0


def test_htk_band_sizes_match_oracle():
    """synth's band sizes for checkpoints without precomputed tables (used to shape
    their weights) equal the oracle's C restatement of the reference's fallback."""
    import oracle
    from msst_b200 import synth

    for nb in (32, 48, 60, 64):
        sizes = synth.htk_band_sizes(44100, 2048, nb)
        nfreq, bins, count = oracle.mel_bands_htk(44100, 2048, nb)
        np.testing.assert_array_equal(sizes, nfreq)
        assert count.min() >= 1 and bins.size == nfreq.sum()
