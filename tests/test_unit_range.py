"""Host check of UnitRange (csrc/common.cuh), the work split of the persistent
fused feed-forward and band-attention kernels: CTA c of G takes the contiguous
units [U*c/G, U*(c+1)/G) of U = tiles x J (tile, hidden chunk / head) units,
walked as one segment per tile.

The struct is compiled for the host from the same header the kernels use and
checked over many shapes: every unit is covered exactly once, each CTA's count
is its share, and with G <= tiles (the feed-forward's grid) a tile is split
between at most two neighbouring CTAs in the form the feed-forward's flag
protocol relies on: chunks [0, k) as CTA c's last segment, [k, J) as CTA c+1's
first.  No GPU is needed.
"""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "cuda-msst-infer_b200", "csrc")

PROGRAM = r"""
#include <cstdio>
#include <vector>
#include "common.cuh"
using msst::UnitRange;

static int check(int ntiles, int J, int G, bool ffn_grid) {
  const long long U = (long long)ntiles * J;
  std::vector<int> owner((size_t)U, -1);
  std::vector<std::vector<int>> segs(G);  // per CTA: flattened (t, j0, j1)
  for (int c = 0; c < G; ++c) {
    const UnitRange r(ntiles, J, c, G);
    long long n = 0;
    int prev_t = -1;
    for (int s = 0; s < r.nseg; ++s) {
      int t, j0, j1;
      r.seg(s, t, j0, j1);
      if (t < 0 || t >= ntiles || j0 < 0 || j1 > J || j0 >= j1) return 1;
      if (t <= prev_t) return 2;  // tiles in increasing order, one segment each
      prev_t = t;
      for (int j = j0; j < j1; ++j) {
        long long u = (long long)t * J + j;
        if (owner[(size_t)u] != -1) return 3;
        owner[(size_t)u] = c;
      }
      n += j1 - j0;
      segs[c].push_back(t), segs[c].push_back(j0), segs[c].push_back(j1);
    }
    if (n != r.count || n != U * (c + 1) / G - U * c / G) return 4;
  }
  for (long long u = 0; u < U; ++u)
    if (owner[(size_t)u] < 0) return 5;
  if (ffn_grid) {
    for (int c = 0; c < G; ++c) {
      const std::vector<int>& v = segs[c];
      const int ns = (int)v.size() / 3;
      for (int s = 0; s < ns; ++s) {
        const int t = v[3 * s], j0 = v[3 * s + 1], j1 = v[3 * s + 2];
        if (j0 > 0 && j1 < J) return 6;       // a run inside one tile: not with G <= tiles
        if (j0 > 0) {                          // tail part: the CTA's first segment,
          if (s != 0 || c == 0) return 7;      // the head part [0, j0) is CTA c-1's last
          const std::vector<int>& p = segs[c - 1];
          const int m = (int)p.size() / 3 - 1;
          if (p[3 * m] != t || p[3 * m + 1] != 0 || p[3 * m + 2] != j0) return 8;
        }
        if (j1 < J && (s != ns - 1 || c == G - 1)) return 9;  // head part: the CTA's last
      }
    }
  }
  return 0;
}

int main() {
  unsigned x = 12345u;
  auto rnd = [&](int lo, int hi) { x = x * 1664525u + 1013904223u; return lo + (int)((x >> 8) % (unsigned)(hi - lo + 1)); };
  const int Js[] = {1, 2, 3, 4, 6, 8, 12, 16, 24};
  int cases = 0;
  for (int i = 0; i < 4000; ++i) {
    const int ntiles = i < 300 ? 1 + i : rnd(1, 3000);
    const int J = Js[i % 9];
    const int sms = i % 3 == 0 ? 148 : rnd(1, 160);
    // the feed-forward's grid: min(tiles, SMs); the band kernel's: min(tiles * heads, SMs)
    const int Gf = ntiles < sms ? ntiles : sms;
    const long long U = (long long)ntiles * J;
    const int Gb = U < sms ? (int)U : sms;
    int e = check(ntiles, J, Gf, true);
    if (e) { std::printf("fail %d ffn ntiles=%d J=%d G=%d\n", e, ntiles, J, Gf); return 1; }
    e = check(ntiles, J, Gb, false);
    if (e) { std::printf("fail %d band ntiles=%d J=%d G=%d\n", e, ntiles, J, Gb); return 1; }
    cases += 2;
  }
  std::printf("ok %d\n", cases);
  return 0;
}
"""


def test_unit_range_covers_and_splits(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    src = tmp_path / "unit_range.cu"
    src.write_text(PROGRAM)
    exe = tmp_path / "unit_range"
    # the header's device helpers need the library's target; the check itself runs on the host
    subprocess.run([nvcc, "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=sm_100a", "-I", CSRC, str(src),
                    "-o", str(exe)], check=True, capture_output=True, timeout=300)
    out = subprocess.run([str(exe)], check=False, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.startswith("ok"), out.stdout + out.stderr
