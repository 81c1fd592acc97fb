"""GPU: msst_model_transformer_noalloc against msst_model_transformer.

The no-alloc entry point exists for callers that must not allocate device
memory while they run (real-time audio hosts whose processing callback cannot
wait on cudaMalloc / cudaFree, applications that own all device memory).  It
runs the same kernels with every intermediate in the library's fixed device
array, so its output must match the allocating entry point's; it is called twice
in a row because all calls share (and leave behind) the same scratch contents.
This file is collected last so a failure here never hides other tests.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-5  # same kernels on the same inputs: identical up to launch-order effects


@pytest.fixture(scope="module")
def small_model(tmp_path_factory):
    from msst_b200 import Model, synth

    cfg = synth.mbr_config(depth=1, dim=128)
    path = str(tmp_path_factory.mktemp("noalloc") / "m.csm")
    synth.write_csm(path, cfg, synth.make_weights(cfg, 21))
    m = Model(path, 0, "fp16")
    yield m, cfg
    m.close()


def _noalloc(torch, m, d, axis, x):
    from msst_b200 import AXIS, check, lib

    check(lib().msst_model_transformer_noalloc(m._h, d, AXIS[axis], ctypes.c_void_p(x.data_ptr()), x.shape[0],
                                               x.shape[1], ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))


@pytest.mark.parametrize("axis", ["time", "band"])
def test_noalloc_matches_allocating_entry_point(cuda, small_model, axis):
    torch = cuda
    m, cfg = small_model
    B, T, nb, D = 2, 57, 60, cfg["dim"]
    g = torch.Generator(device="cuda").manual_seed(7)
    x0 = torch.randn(B, T, nb, D, device="cuda", generator=g)
    ref = x0.clone()
    m.transformer(0, axis, ref)
    torch.cuda.synchronize()
    for _ in range(2):  # second call reuses the scratch the first one left behind
        y = x0.clone()
        _noalloc(torch, m, 0, axis, y)
        torch.cuda.synchronize()
        assert rel_l2(y.cpu().numpy(), ref.cpu().numpy()) < TOL


def test_noalloc_rejects_oversize(cuda, small_model):
    torch = cuda
    from msst_b200 import MSST_ERR_INVALID, MsstError

    m, cfg = small_model
    x = torch.zeros(8, 801, 60, cfg["dim"], device="cuda")  # 384,480 tokens: far beyond the fixed scratch
    with pytest.raises(MsstError) as ei:
        _noalloc(torch, m, 0, "time", x)
    assert ei.value.code == MSST_ERR_INVALID and "scratch" in str(ei.value)
