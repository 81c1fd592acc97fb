"""CPU: the C++ shim that keeps the reference's cudasep::Tensor call sites
(cuda-msst-infer_b200/shim/msst_shim.h) compiles against the reference's own
headers (src/tensor.h, src/ops.h) and include/msst_b200.h.  Needs the reference
sources, present only where the fixtures are built; skipped elsewhere."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

from conftest import ROOT

REF_SRC = "/root/reference/src"

TU = r'''
#include "msst_shim.h"
// odr-use every wrapper so each one is type-checked against the reference's Tensor
using namespace cudasep;
void use_all(Tensor& x, Tensor& g, Tensor& b, Tensor& w16) {
  Tensor a = msst::rms_norm16(x, g, 19.6f);
  Tensor c = msst::linear_gelu16(a, w16, b);
  Tensor d = msst::layer_norm(x, g, b);
  Tensor e = msst::sdpa16(a, a, a);
  msst::Model m("model.csm", 0);
  Tensor f = m.forward(x);
  Tensor h = m.separate(x, 0.25f, 4);
  (void)c; (void)d; (void)e; (void)f; (void)h;
}
'''


def test_shim_compiles_against_reference_headers(tmp_path):
    if not os.path.isdir(REF_SRC):
        pytest.skip("reference sources not present")
    cxx = shutil.which("g++") or "/usr/bin/g++"
    src = tmp_path / "shim_tu.cpp"
    src.write_text(TU)
    cmd = [cxx, "-std=c++17", "-fsyntax-only", "-I/usr/local/cuda/include", "-I/usr/include/x86_64-linux-gnu",
           f"-I{REF_SRC}", f"-I{os.path.join(ROOT, 'include')}",
           f"-I{os.path.join(ROOT, 'cuda-msst-infer_b200', 'shim')}", str(src)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
