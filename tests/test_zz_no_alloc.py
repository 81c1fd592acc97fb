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

# same kernels on the same inputs; only the rotary tables differ (computed on the
# device here, on the host by the allocating path: a few ulp)
TOL = 1e-5


# (dim, mlp_expansion_factor, batch, T): the GEMM column tiles differ across these
# widths (dim 128 / 384 / 640 -> out-projection tiles 128 / 192 / 256; mlp 1 -> a
# 128-wide feed-forward), and every case stays inside the fixed scratch array
CASES = [(128, 4, 2, 57), (384, 4, 1, 57), (640, 4, 1, 41), (128, 1, 2, 57)]


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    from msst_b200 import Model, synth

    out = {}
    d = tmp_path_factory.mktemp("noalloc")
    for dim, mlp, _, _ in CASES:
        cfg = synth.mbr_config(depth=1, dim=dim, mlp_expansion_factor=mlp)
        path = str(d / f"m{dim}_{mlp}.csm")
        synth.write_csm(path, cfg, synth.make_weights(cfg, 21))
        out[(dim, mlp)] = (Model(path, 0, "fp16"), cfg)
    yield out
    for m, _ in out.values():
        m.close()


@pytest.fixture(scope="module")
def small_model(models):
    return models[(128, 4)]


def _noalloc(torch, m, d, axis, x):
    from msst_b200 import AXIS, check, lib

    check(lib().msst_model_transformer_noalloc(m._h, d, AXIS[axis], ctypes.c_void_p(x.data_ptr()), x.shape[0],
                                               x.shape[1], ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))


@pytest.mark.parametrize("axis", ["time", "band"])
@pytest.mark.parametrize("dim,mlp,B,T", CASES)
def test_noalloc_matches_allocating_entry_point(cuda, models, axis, dim, mlp, B, T):
    torch = cuda
    m, cfg = models[(dim, mlp)]
    nb = cfg["num_bands"]
    g = torch.Generator(device="cuda").manual_seed(7)
    x0 = torch.randn(B, T, nb, dim, device="cuda", generator=g)
    ref = x0.clone()
    m.transformer(0, axis, ref)
    # one warm-up call: the first use on a device may load the library's module
    # (and with it the fixed array) under lazy loading
    warm = x0.clone()
    _noalloc(torch, m, 0, axis, warm)
    ys = [x0.clone() for _ in range(2)]
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for y in ys:  # the second call reuses the scratch the first one left behind
        _noalloc(torch, m, 0, axis, y)
        torch.cuda.synchronize()
        assert rel_l2(y.cpu().numpy(), ref.cpu().numpy()) < TOL
    assert torch.cuda.mem_get_info()[0] == free_before, "the no-alloc entry point allocated device memory"


def test_noalloc_rejects_oversize(cuda, small_model):
    torch = cuda
    from msst_b200 import MSST_ERR_INVALID, MsstError

    m, cfg = small_model
    x = torch.zeros(8, 801, 60, cfg["dim"], device="cuda")  # 384,480 tokens: far beyond the fixed scratch
    with pytest.raises(MsstError) as ei:
        _noalloc(torch, m, 0, "time", x)
    assert ei.value.code == MSST_ERR_INVALID and "scratch" in str(ei.value)
