// gemm.cu — persistent, warp-specialised tcgen05 GEMM for sm_100a with fused
// epilogues.  Replaces the cuBLAS GEMM + separate bias/activation/residual
// kernels of the reference (src/ops_linear.cu:150-427, src/ops_fused.cu:203-303,
// the residual add in src/tensor.cu:1439-1442 and the per-band loops of
// src/model_mel_band_roformer.cu:676-736).
//
// CTA = 320 threads (192 with the residual epilogue):
//   warp 0     TMA producer (one lane): A/B k-blocks of 64 into a smem ring
//   warp 1     MMA issuer (one lane): tcgen05.mma M=128 N=BN K=16, fp32 accumulators
//              in TMEM, double-buffered so the epilogue of tile i overlaps the
//              main loop of tile i+1; also owns the TMEM allocation
//   warps 2-9  epilogue (warps 2-5 for the residual epilogue): warp w reads
//              TMEM lane quarter w%4 and, with 8 epilogue warps, column half
//              (w-2)/4, 32 columns at a time; bias/activation/RoPE in fp32; the
//              32x32 result is staged in swizzled smem and leaves by TMA bulk
//              store (or bulk reduce-add into the fp32 residual stream).
// Tiles of all groups are walked in one static persistent schedule; the group
// table is read from the kernel's parameter space, so shared memory holds only
// the ring (4 stages at BN 256, 5 at BN 192 with the residual epilogue) and staging.
// Large launches run the CTA-pair variant (gemm_pair_kernel, below).
#include <cstdlib>

#include "common.cuh"
#include "gemm.cuh"

namespace msst {

namespace {

template <int EPI>
struct EpiTraits {
  static constexpr bool kTma = EPI != kEpiGlu32;
  static constexpr bool k16 = EPI == kEpiStore16 || EPI == kEpiQkvRope;
  // per-warp staging: 32 rows x 32 columns (64 B rows for 16-bit, 128 B for fp32)
  static constexpr uint32_t kStageBytes = k16 ? 2048 : 4096;
  // epilogue warps: two per TMEM lane quarter, each on half the tile's columns;
  // the residual reduce-add (long K, light epilogue) uses one, which halves its
  // staging and leaves room for a 5th ring stage
  static constexpr int kWarps = EPI == kEpiResid32 ? 4 : 8;
  static constexpr int kThreads = 64 + 32 * kWarps;
  // staging buffers per warp (a second one, letting a chunk be staged while the
  // previous chunk's bulk store still reads its buffer, measured no faster: the
  // stores are bound by the output's DRAM writes, not by the wait)
  static constexpr int kStgBufs = 1;
  static constexpr uint32_t kWarpStgBytes = kStageBytes * kStgBufs;
};

template <int BN, int EPI>
struct GemmCfg {
  static constexpr uint32_t kABytes = kGemmBM * kGemmBK * 2;
  static constexpr uint32_t kBBytes = BN * kGemmBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kEpiBytes = EpiTraits<EPI>::kWarps * EpiTraits<EPI>::kWarpStgBytes;
  static constexpr size_t kFixed = 1024 + kEpiBytes + 256;
  static constexpr int kStagesRaw = (int)((232448 - kFixed) / kStageBytes);
  static constexpr int kStages = kStagesRaw > 6 ? 6 : kStagesRaw;
  static constexpr uint32_t kTmemCols = (2 * BN <= 256) ? 256 : 512;
  static constexpr size_t kSmemBytes = kFixed + (size_t)kStages * kStageBytes;
  static_assert(kStages >= 2, "not enough shared memory for a 2-stage ring");
};

__device__ __forceinline__ int find_group(const GemmGroup* g, int n, int t) {
  int i = 0;
  while (i + 1 < n && g[i + 1].tile_begin <= t) ++i;
  return i;
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 abs2(float2 v) { return make_float2(fabsf(v.x), fabsf(v.y)); }

// The epilogue activations on pairs of columns: the FMA-pipe arithmetic runs as
// packed f32x2 operations (half the issue slots), the MUFU work (ex2, rcp) per
// element.
//
// GELU, erf form (reference src/ops_fused.cu:21-24): 0.5 x (1 + erf(x / sqrt 2)),
// erf by Abramowitz & Stegun, Handbook of Mathematical Functions, formula 7.1.26
// (after Hastings): erf(a) = 1 - t(a1 + t(a2 + t(a3 + t(a4 + t a5)))) e^{-a^2},
// t = 1/(1 + p a), |error| <= 1.5e-7 for a >= 0, odd extension for a < 0 -- two
// MUFU operations and a handful of FMAs, well below the 16-bit output rounding.
// The polynomial's signs are folded so that 1 - t poly(t) e^{-a^2} is one FMA.
__device__ __forceinline__ float2 gelu2(float2 x) {
  const float2 z = __fmul2_rn(x, f2(0.70710678118654752f));
  const float2 a = abs2(z);
  const float2 d = __ffma2_rn(a, f2(0.3275911f), f2(1.0f));
  const float2 t = make_float2(rcp_approx(d.x), rcp_approx(d.y));
  float2 q = __ffma2_rn(t, f2(-1.061405429f), f2(1.453152027f));
  q = __ffma2_rn(t, q, f2(-1.421413741f));
  q = __ffma2_rn(t, q, f2(0.284496736f));
  q = __ffma2_rn(t, q, f2(-0.254829592f));
  const float2 np = __fmul2_rn(t, q);                       // -t*poly(t)
  const float2 s = __fmul2_rn(__fmul2_rn(a, f2(-1.4426950408889634f)), a);  // -a^2 log2(e)
  const float2 e = make_float2(fast_exp2(s.x), fast_exp2(s.y));
  const float2 r = __ffma2_rn(np, e, f2(1.0f));             // erf(|z|)
  const float2 erf = make_float2(copysignf(r.x, z.x), copysignf(r.y, z.y));
  const float2 h = __fmul2_rn(x, f2(0.5f));
  return __ffma2_rn(h, erf, h);
}
// tanh(x) = 1 - 2 / (1 + 2^(2x log2 e)); saturates exactly to +-1 at both ends
__device__ __forceinline__ float2 tanh2(float2 x) {
  const float2 s = __fmul2_rn(x, f2(2.8853900817779268f));
  const float2 d = __fadd2_rn(make_float2(fast_exp2(s.x), fast_exp2(s.y)), f2(1.0f));
  return __ffma2_rn(make_float2(rcp_approx(d.x), rcp_approx(d.y)), f2(-2.0f), f2(1.0f));
}
// logistic sigmoid, 1 / (1 + 2^(-x log2 e)) with an approximate reciprocal (the
// reference's --use_fast_math build also makes this division approximate)
__device__ __forceinline__ float2 sigmoid2(float2 x) {
  const float2 s = __fmul2_rn(x, f2(-1.4426950408889634f));
  const float2 d = __fadd2_rn(make_float2(fast_exp2(s.x), fast_exp2(s.y)), f2(1.0f));
  return make_float2(rcp_approx(d.x), rcp_approx(d.y));
}

// RoPE table entries of one chunk (cos[4] then sin[4]), fetched before the
// accumulator wait / TMEM load so the global loads overlap them.  (Fetching the
// bias the same way measured slower for the GELU epilogue, which needs the
// registers; the bias is read at use.)
struct ChunkOps {
  float4 a[8];
};

template <int EPI>
__device__ __forceinline__ void chunk_prefetch(const GemmParams& p, const GemmGroup& g, int row, int col,
                                               ChunkOps& o) {
  if constexpr (EPI == kEpiQkvRope) {
    if (col < p.rope_cols) {
      const int half = p.head_dim >> 1;
      const int pos = (row / p.pos_div) % p.pos_mod;
      const int i0 = (col % p.head_dim) >> 1;
      const float4* cs = reinterpret_cast<const float4*>(p.rope_cos + (size_t)pos * half + i0);
      const float4* sn = reinterpret_cast<const float4*>(p.rope_sin + (size_t)pos * half + i0);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        o.a[u] = __ldg(cs + u);
        o.a[4 + u] = __ldg(sn + u);
      }
    }
  }
}

// bias, activation and RoPE on one 32-column chunk of one row (fp32 registers)
template <int EPI>
__device__ __forceinline__ void chunk_math(const GemmParams& p, const GemmGroup& g, int row, int col, float (&v)[32],
                                           const ChunkOps& o) {
  if constexpr (EPI != kEpiQkvRope) {
    if (g.bias != nullptr && g.n - col >= 32 && ((reinterpret_cast<uintptr_t>(g.bias + col) & 15) == 0)) {
      const float4* b4 = reinterpret_cast<const float4*>(g.bias + col);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 b = __ldg(b4 + q);
        const float2 lo = __fadd2_rn(make_float2(v[4 * q], v[4 * q + 1]), make_float2(b.x, b.y));
        const float2 hi = __fadd2_rn(make_float2(v[4 * q + 2], v[4 * q + 3]), make_float2(b.z, b.w));
        v[4 * q] = lo.x;
        v[4 * q + 1] = lo.y;
        v[4 * q + 2] = hi.x;
        v[4 * q + 3] = hi.y;
      }
    } else if (g.bias != nullptr) {
      const int nvalid = min(32, g.n - col);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nvalid) v[j] += __ldg(g.bias + col + j);
    }
  }
  if constexpr (EPI == kEpiStore16) {
    if (p.act == kActGelu) {
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float2 y = gelu2(make_float2(v[j], v[j + 1]));
        v[j] = y.x;
        v[j + 1] = y.y;
      }
    } else if (p.act == kActTanh) {
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float2 y = tanh2(make_float2(v[j], v[j + 1]));
        v[j] = y.x;
        v[j + 1] = y.y;
      }
    } else if (p.act == kActSigmoid) {
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float2 y = sigmoid2(make_float2(v[j], v[j + 1]));
        v[j] = y.x;
        v[j + 1] = y.y;
      }
    }
  } else if constexpr (EPI == kEpiQkvRope) {
    if (col < p.rope_cols) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 c4 = o.a[u], s4 = o.a[4 + u];
        const float c[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = 4 * u + k;
          const float x0 = v[2 * j], x1 = v[2 * j + 1];
          v[2 * j] = x0 * c[k] - x1 * sn[k];
          v[2 * j + 1] = x0 * sn[k] + x1 * c[k];
        }
      }
    }
  }
}

// GLU epilogue with direct stores (value/gate columns interleaved by the weight packing)
__device__ __forceinline__ void glu_store(const GemmGroup& g, int row, int col, const float (&v)[32]) {
  const int nvalid = min(32, g.n - col);
  const long long orow = (long long)row * g.out_row_mul + g.out_row_add;
  float* o = reinterpret_cast<float*>(g.out) + orow * g.ldo + g.out_col0 + (col >> 1);
  float w[16];
#pragma unroll
  for (int j = 0; j < 16; j += 2) {
    const float2 gt = sigmoid2(make_float2(v[2 * j + 1], v[2 * j + 3]));
    const float2 y = __fmul2_rn(make_float2(v[2 * j], v[2 * j + 2]), gt);
    w[j] = y.x;
    w[j + 1] = y.y;
  }
  const int nout = nvalid >> 1;
  if (nout == 16 && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
    float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
    for (int q = 0; q < 4; ++q) o4[q] = make_float4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < nout) o[j] = w[j];
  }
}

// Write this lane's row of a 32x32 chunk into the warp's staging tile using the
// swizzle the output tensor map expects (SW64 for 16-bit rows of 64 B, SW128 for
// fp32 rows of 128 B); 8 consecutive rows cover all 32 banks.
template <typename T, bool k16>
__device__ __forceinline__ void stage_row(uint8_t* stg, int r, const float (&v)[32]) {
  if constexpr (k16) {
    uint8_t* rowp = stg + r * 64;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 w = make_uint4(pack2<T>(v[8 * c], v[8 * c + 1]), pack2<T>(v[8 * c + 2], v[8 * c + 3]),
                                 pack2<T>(v[8 * c + 4], v[8 * c + 5]), pack2<T>(v[8 * c + 6], v[8 * c + 7]));
      *reinterpret_cast<uint4*>(rowp + ((c ^ ((r >> 1) & 3)) << 4)) = w;
    }
  } else {
    uint8_t* rowp = stg + r * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4*>(rowp + ((c ^ (r & 7)) << 4)) =
          make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  }
}

// Epilogue of one accumulator tile by epilogue warp `warp` (absolute index >= 2):
// the warp owns TMEM lane quarter warp % 4 (rows row_base + 32 * (warp % 4) + lane
// of the group) and, with 8 epilogue warps, one half of the tile's columns,
// 32 at a time.  acc = TMEM address of the tile's column 0.  wait_acc() waits for
// the accumulator (false: gave up); the first chunk's operands (bias, RoPE
// tables) are fetched before it.
template <int BN, int EPI, typename T, typename WaitAcc>
__device__ __forceinline__ bool epilogue_tile(const GemmParams& p, const GemmGroup& g, const CUtensorMap* map_o,
                                              uint32_t acc, int row_base, int tn, int warp, int lane, uint8_t* stg,
                                              WaitAcc&& wait_acc) {
  using Epi = EpiTraits<EPI>;
  const int q = warp & 3;
  const int half = (warp - 2) >> 2;
  const int row = row_base + q * 32 + lane;
  const int n_eff = min(BN, g.n - tn * BN);
  constexpr int kSplit = Epi::kWarps / 4;  // warps per TMEM lane quarter
  const int c_begin = half * (BN / kSplit);
  const int c_end = min(c_begin + BN / kSplit, n_eff);
  ChunkOps ops;
  if (c_begin < c_end) chunk_prefetch<EPI>(p, g, row, tn * BN + c_begin, ops);
  if (!wait_acc()) return false;
  tc_fence_after();
  int i = 0;
  for (int c0 = c_begin; c0 < c_end; c0 += 32, ++i) {
    const int col = tn * BN + c0;
    if (c0 != c_begin) chunk_prefetch<EPI>(p, g, row, col, ops);
    uint32_t r[32];
    tmem_ld32(acc + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, r);
    tmem_ld_wait();
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    chunk_math<EPI>(p, g, row, col, v, ops);
    if constexpr (Epi::kTma) {
      uint8_t* buf = stg + (Epi::kStgBufs == 2 ? (i & 1) : 0) * Epi::kStageBytes;
      if (lane == 0) {
        if constexpr (Epi::kStgBufs == 2)
          bulk_wait_read1();
        else
          bulk_wait_read0();
      }
      __syncwarp();
      stage_row<T, Epi::k16>(buf, lane, v);
      fence_proxy_async_smem();
      __syncwarp();
      // boxes starting past the group's last row stay unwritten (they would hold
      // products of the next group's A rows)
      const int row0 = row_base + q * 32;
      if (lane == 0 && row0 < g.m) {
        const int x = g.out_col0 + col, y = g.oy0 + g.oy_row * row0, z = g.oz0 + g.oz_row * row0;
        if constexpr (EPI == kEpiResid32)
          tma_reduce_add_3d(map_o, buf, x, y, z);
        else
          tma_store_3d(map_o, buf, x, y, z);
      }
      if (lane == 0) bulk_commit();
    } else {
      if (row < g.m) glu_store(g, row, col, v);
    }
  }
  return true;
}

template <int BN, int EPI, typename T>
__global__ void __launch_bounds__(EpiTraits<EPI>::kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_o, const __grid_constant__ GemmParams p) {
  using Cfg = GemmCfg<BN, EPI>;
  using Epi = EpiTraits<EPI>;
  constexpr int kStages = Cfg::kStages;
  constexpr uint32_t kIsBf16 = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * Cfg::kABytes;
  uint8_t* sEpi = sB + kStages * Cfg::kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + Cfg::kEpiBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const GemmGroup* groups = p.groups;  // read from the kernel's parameter space

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], Epi::kWarps);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    if constexpr (Epi::kTma) tma_prefetch_desc(&map_o);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x) {
        const GemmGroup& g = groups[find_group(groups, p.num_groups, t)];
        const int lt = t - g.tile_begin;
        const int tm = lt / g.tiles_n, tn = lt - tm * g.tiles_n;
        const int kblocks = g.k / kGemmBK;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], ph ^ 1u, kErrTimeoutSmemEmpty, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          tma_load_2d(sA + stage * Cfg::kABytes, &map_a, &full[stage], g.a_col0 + kb * kGemmBK,
                      g.a_row0 + tm * kGemmBM);
          // B in two boxes of BN/2 rows (the tensor map's box is shared with the pair kernel)
          tma_load_2d(sB + stage * Cfg::kBBytes, &map_b, &full[stage], g.b_col0 + kb * kGemmBK, g.b_row0 + tn * BN);
          tma_load_2d(sB + stage * Cfg::kBBytes + Cfg::kBBytes / 2, &map_b, &full[stage], g.b_col0 + kb * kGemmBK,
                      g.b_row0 + tn * BN + BN / 2);
          if (++stage == kStages) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      int abuf = 0;
      uint32_t aph = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x) {
        const GemmGroup& g = groups[find_group(groups, p.num_groups, t)];
        const int lt = t - g.tile_begin;
        const int tn = lt % g.tiles_n;
        const int n_eff = min(BN, g.n - tn * BN);
        const uint32_t n_mma = (uint32_t)((n_eff + 15) & ~15);
        const uint32_t idesc = umma_idesc_f16(kIsBf16, n_mma);
        const int kblocks = g.k / kGemmBK;
        if (!mbar_wait(&tempty[abuf], aph ^ 1u, kErrTimeoutTmemEmpty, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(abuf * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], ph, kErrTimeoutTmaFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * Cfg::kABytes);
          const uint32_t b0 = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
          for (int kk = 0; kk < kGemmBK / 16; ++kk) {
            umma_f16_ss(d_tmem, sw128_desc(a0 + kk * 32, 16, 1024), sw128_desc(b0 + kk * 32, 16, 1024), idesc,
                        (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[abuf]);
        abuf ^= 1;
        if (abuf == 0) aph ^= 1u;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (8 warps)
    uint8_t* stg = sEpi + (warp - 2) * Epi::kWarpStgBytes;
    int abuf = 0;
    uint32_t aph = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
      const GemmGroup& g = groups[find_group(groups, p.num_groups, t)];
      const int lt = t - g.tile_begin;
      const int tm = lt / g.tiles_n, tn = lt - tm * g.tiles_n;
      if (!epilogue_tile<BN, EPI, T>(p, g, &map_o, tmem_base + (uint32_t)(abuf * BN), tm * kGemmBM, tn, warp, lane,
                                     stg, [&] { return mbar_wait(&tfull[abuf], aph, kErrTimeoutTmemFull, abort_flag); }))
        break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[abuf]);
      abuf ^= 1;
      if (abuf == 0) aph ^= 1u;
    }
    if constexpr (Epi::kTma) {
      if (lane == 0) bulk_wait0();
      __syncwarp();
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs computes 256 x BN output tiles with
// M = 256 tcgen05 MMAs (cta_group::2) issued by rank 0.  Each CTA streams its own
// 128 A rows and BN/2 B rows per k-block, so a CTA moves (128 + BN/2) x 64
// operand elements per k-block for a 128 x BN slice of the product instead of
// (128 + BN) x 64 -- a third less shared-memory traffic per FLOP at BN = 256,
// and a 32 KB stage instead of 48 KB, so more k-blocks are in flight.
//   full[s]   (rank 0 only) one arrival (rank 0's expect_tx of both CTAs' bytes);
//             both CTAs' TMA loads complete on it
//   empty[s]  (each CTA) the pair MMA's commit, multicast to both CTAs
//   tfull[b]  (each CTA) accumulator b ready, multicast commit
//   tempty[b] (rank 0 only) both CTAs' epilogue warps arrive (2 x kWarps)
// Every role falls through to the final cluster barrier, including after a
// bounded wait gave up, so neither CTA leaves while the other may still touch
// its shared memory; then both free the pair's TMEM.
template <int BN, int EPI>
struct PairCfg {
  static constexpr uint32_t kABytes = kGemmBM * kGemmBK * 2;
  static constexpr uint32_t kBBytes = (BN / 2) * kGemmBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kEpiBytes = EpiTraits<EPI>::kWarps * EpiTraits<EPI>::kWarpStgBytes;
  static constexpr size_t kFixed = 1024 + kEpiBytes + 256;
  static constexpr int kStagesRaw = (int)((232448 - kFixed) / kStageBytes);
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr uint32_t kTmemCols = (2 * BN <= 256) ? 256 : 512;
  static constexpr size_t kSmemBytes = kFixed + (size_t)kStages * kStageBytes;
  static_assert(kStages >= 2, "not enough shared memory for a 2-stage ring");
};

template <int BN, int EPI, typename T>
__global__ void __launch_bounds__(EpiTraits<EPI>::kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_o, const __grid_constant__ GemmParams p) {
  using Cfg = PairCfg<BN, EPI>;
  using Epi = EpiTraits<EPI>;
  constexpr int kStages = Cfg::kStages;
  constexpr uint32_t kIsBf16 = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr int kPairM = 2 * kGemmBM;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * Cfg::kABytes;
  uint8_t* sEpi = sB + kStages * Cfg::kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + Cfg::kEpiBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const GemmGroup* groups = p.groups;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = (int)(blockIdx.x >> 1), num_pairs = (int)(gridDim.x >> 1);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * Epi::kWarps);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    if constexpr (Epi::kTma) tma_prefetch_desc(&map_o);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tc_fence_before();
  }
  // barriers initialised in both CTAs before either signals the other's
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = pair; ok && t < p.total_tiles; t += num_pairs) {
        const GemmGroup& g = groups[find_group(groups, p.num_groups, t)];
        const int lt = t - g.tile_begin;
        const int tm = lt / g.tiles_n, tn = lt - tm * g.tiles_n;
        const int kblocks = g.k / kGemmBK;
        const int a_row = g.a_row0 + tm * kPairM + (int)rank * kGemmBM;
        const int b_row = g.b_row0 + tn * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], ph ^ 1u, kErrTimeoutSmemEmpty, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
          tma_load_2d_pair(sA + stage * Cfg::kABytes, &map_a, bar, g.a_col0 + kb * kGemmBK, a_row);
          tma_load_2d_pair(sB + stage * Cfg::kBBytes, &map_b, bar, g.b_col0 + kb * kGemmBK, b_row);
          if (++stage == kStages) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (rank 0)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t ph = 0;
      int abuf = 0;
      uint32_t aph = 0;
      bool ok = true;
      const uint32_t idesc = umma_idesc_f16(kIsBf16, (uint32_t)BN, 0, (uint32_t)kPairM);
      for (int t = pair; ok && t < p.total_tiles; t += num_pairs) {
        const GemmGroup& g = groups[find_group(groups, p.num_groups, t)];
        const int kblocks = g.k / kGemmBK;
        if (!mbar_wait(&tempty[abuf], aph ^ 1u, kErrTimeoutTmemEmpty, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(abuf * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], ph, kErrTimeoutTmaFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * Cfg::kABytes);
          const uint32_t b0 = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
          for (int kk = 0; kk < kGemmBK / 16; ++kk) {
            umma_f16_ss_pair(d_tmem, sw128_desc(a0 + kk * 32, 16, 1024), sw128_desc(b0 + kk * 32, 16, 1024), idesc,
                             (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == kStages) {
            stage = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[abuf], 0x3);
        abuf ^= 1;
        if (abuf == 0) aph ^= 1u;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    uint8_t* stg = sEpi + (warp - 2) * Epi::kWarpStgBytes;
    int abuf = 0;
    uint32_t aph = 0;
    for (int t = pair; t < p.total_tiles; t += num_pairs) {
      const GemmGroup& g = groups[find_group(groups, p.num_groups, t)];
      const int lt = t - g.tile_begin;
      const int tm = lt / g.tiles_n, tn = lt - tm * g.tiles_n;
      if (!epilogue_tile<BN, EPI, T>(p, g, &map_o, tmem_base + (uint32_t)(abuf * BN), tm * kPairM + (int)rank * kGemmBM,
                                     tn, warp, lane, stg,
                                     [&] { return mbar_wait(&tfull[abuf], aph, kErrTimeoutTmemFull, abort_flag); }))
        break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[abuf]), 0));
      abuf ^= 1;
      if (abuf == 0) aph ^= 1u;
    }
    if constexpr (Epi::kTma) {
      if (lane == 0) bulk_wait0();
      __syncwarp();
    }
  }

  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

// Algorithmic cost of one launch: 2*m*n*k FLOPs per group; bytes = A and B read
// once, the output written once (the residual epilogue also reads it).
struct GemmCost {
  const char* name;
  double flop, bytes;
};

GemmCost gemm_cost(const GemmParams& p, int epi, int esize) {
  static const char* const kStore16[4] = {"gemm_store16", "gemm_store16_gelu", "gemm_store16_tanh",
                                          "gemm_store16_sigmoid"};  // indexed by kAct*
  GemmCost c{nullptr, 0.0, 0.0};
  switch (epi) {
    case kEpiStore16: c.name = kStore16[(p.act >= 0 && p.act < 4) ? p.act : 0]; break;
    case kEpiResid32: c.name = "gemm_resid32"; break;
    case kEpiStore32: c.name = "gemm_store32"; break;
    case kEpiGlu32: c.name = "gemm_glu32"; break;
    default: c.name = "gemm_qkv_rope"; break;
  }
  const double out_bytes = epi == kEpiStore16 || epi == kEpiQkvRope ? 2.0 : epi == kEpiResid32 ? 8.0
                           : epi == kEpiGlu32                      ? 2.0  // n/2 fp32 columns
                                                                   : 4.0;
  for (int i = 0; i < p.num_groups; ++i) {
    const GemmGroup& g = p.groups[i];
    c.flop += 2.0 * g.m * (double)g.n * g.k;
    c.bytes += ((double)g.m * g.k + (double)g.n * g.k) * esize + (double)g.m * g.n * out_bytes;
  }
  return c;
}

template <int BN, int EPI, typename T>
cudaError_t launch_one(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, const GemmParams& p,
                       int num_sms, cudaStream_t stream) {
  using Cfg = GemmCfg<BN, EPI>;
  auto kern = gemm_kernel<BN, EPI, T>;
  static std::atomic<unsigned long long> configured{0};
  cudaError_t e = ensure_smem_limit(kern, (int)Cfg::kSmemBytes, configured);
  if (e != cudaSuccess) return e;
  const int grid = p.total_tiles < num_sms ? p.total_tiles : num_sms;
  if (grid <= 0) return cudaSuccess;
  const GemmCost cost = gemm_cost(p, EPI, (int)sizeof(T));
  LaunchScope scope(cost.name, cost.flop, cost.bytes, stream);
  kern<<<grid, EpiTraits<EPI>::kThreads, Cfg::kSmemBytes, stream>>>(ma, mb, mo, p);
  return cudaGetLastError();
}

// The pair kernel as a cluster launch of 2 x (co-resident clusters) CTAs at most;
// `pp` holds the group table re-tiled for 256-row pair tiles.
template <int BN, int EPI, typename T>
cudaError_t launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, const GemmParams& pp,
                        cudaStream_t stream) {
  using Cfg = PairCfg<BN, EPI>;
  auto kern = gemm_pair_kernel<BN, EPI, T>;
  // co-resident pairs: the same for every B200 of the process, so cached once
  static std::atomic<int> max_pairs{0};
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(EpiTraits<EPI>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static std::atomic<unsigned long long> configured{0};
  cudaError_t e = ensure_smem_limit(kern, (int)Cfg::kSmemBytes, configured);
  if (e != cudaSuccess) return e;
  if (max_pairs.load() == 0) {
    cfg.gridDim = dim3(2 * 148, 1, 1);
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess) return e;
    if (n < 1) return cudaErrorInvalidConfiguration;
    max_pairs.store(n);
  }
  const int mp = max_pairs.load();
  const int pairs = pp.total_tiles < mp ? pp.total_tiles : mp;
  if (pairs <= 0) return cudaSuccess;
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  const GemmCost cost = gemm_cost(pp, EPI, (int)sizeof(T));
  LaunchScope scope(cost.name, cost.flop, cost.bytes, stream);
  return cudaLaunchKernelEx(&cfg, kern, ma, mb, mo, pp);
}

// Pair tiles for the residual reduce-add when every group's columns are whole BN
// tiles, K >= 512 and there are at least two pair tiles per co-resident pair.
// Measured: the residual GEMMs gain 4-10 % (their operand stream dominates);
// the 16-bit-output GEMMs at K = 384 are bound by their output writes and lose
// 3-5 % to the pair coupling, so they stay on single CTAs.  MSST_GEMM_PAIR=0
// turns pairs off, MSST_GEMM_PAIR=2 uses them for every eligible launch.
bool use_pair(const GemmParams& p, int bn, int epi) {
  static const int env = [] {
    const char* e = getenv("MSST_GEMM_PAIR");
    return e ? atoi(e) : 1;
  }();
  if (env == 0) return false;
  // by default: the residual GEMMs at K >= 512 and the 16-bit / GLU outputs at K >= 1024
  // (the mask estimator's hidden layers, where the main loop outweighs the output
  // writes; at K = 384 those are write-bound and the pair's coupled hand-off costs)
  const bool wide_out = epi == kEpiStore16 || epi == kEpiGlu32;
  if (env == 1 && epi != kEpiResid32 && !wide_out) return false;
  long long pair_tiles = 0;
  for (int i = 0; i < p.num_groups; ++i) {
    const GemmGroup& g = p.groups[i];
    if (g.n % bn != 0) return false;
    if (env == 1 && g.k < (wide_out ? 1024 : 512)) return false;
    pair_tiles += (long long)((g.m + 2 * kGemmBM - 1) / (2 * kGemmBM)) * (g.n / bn);
  }
  return pair_tiles >= 2 * 74;
}

template <int BN, typename T>
cudaError_t dispatch_epi(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, const GemmParams& p,
                         int epi, int num_sms, cudaStream_t s) {
  if (use_pair(p, BN, epi)) {
    GemmParams pp = p;
    int tiles = 0;
    for (int i = 0; i < pp.num_groups; ++i) {
      GemmGroup& g = pp.groups[i];
      g.tiles_n = g.n / BN;
      g.tile_begin = tiles;
      tiles += ((g.m + 2 * kGemmBM - 1) / (2 * kGemmBM)) * g.tiles_n;
    }
    pp.total_tiles = tiles;
    switch (epi) {
      case kEpiStore16: return launch_pair<BN, kEpiStore16, T>(ma, mb, mo, pp, s);
      case kEpiResid32: return launch_pair<BN, kEpiResid32, T>(ma, mb, mo, pp, s);
      case kEpiStore32: return launch_pair<BN, kEpiStore32, T>(ma, mb, mo, pp, s);
      case kEpiGlu32: return launch_pair<BN, kEpiGlu32, T>(ma, mb, mo, pp, s);
      case kEpiQkvRope: return launch_pair<BN, kEpiQkvRope, T>(ma, mb, mo, pp, s);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (epi) {
    case kEpiStore16: return launch_one<BN, kEpiStore16, T>(ma, mb, mo, p, num_sms, s);
    case kEpiResid32: return launch_one<BN, kEpiResid32, T>(ma, mb, mo, p, num_sms, s);
    case kEpiStore32: return launch_one<BN, kEpiStore32, T>(ma, mb, mo, p, num_sms, s);
    case kEpiGlu32: return launch_one<BN, kEpiGlu32, T>(ma, mb, mo, p, num_sms, s);
    case kEpiQkvRope: return launch_one<BN, kEpiQkvRope, T>(ma, mb, mo, p, num_sms, s);
    default: return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------------------
// Fused feed-forward block (see gemm.cuh).  CTA = 320 threads, persistent over a
// contiguous range of the launch's (128-row tile, 128-wide hidden chunk) units
// (UnitRange), so every CTA gets the same number of chunks (give or take one)
// instead of whole tiles in rounds of the grid size.  A tile whose chunks are split
// between CTA c (chunks [0, k), the last segment of its range) and CTA c + 1
// (chunks [k, J), its first segment) gets two partial reduce-adds into x, ordered
// by a flag: c + 1 adds its partial O (no b2) and then releases the flag of each
// epilogue warp; the matching warp of c acquires it (long since released: c + 1 did
// that part first) before adding O + b2, so the result does not depend on timing.
// Roles:
//   warp 0     TMA: the tile's xn (D/64 swizzled 128x64 atoms, resident for the
//              tile), then W1 / W2 128x64 blocks through a 16 KB ring in the order
//              the MMAs consume them
//   warp 1     MMA issuer: S = xn . W1_j^T (TMEM columns [0, 128)) and
//              O += P_j . W2_j^T (columns [128, 128 + D)), issued as
//              S_0, S_1, O_0, S_2, O_1, ..., O_{J-1} so that the GELU of chunk j
//              overlaps S_{j+1}
//   warps 2-9  per chunk: S -> registers (64 columns each), bias + GELU, 16-bit P
//              rows into the K-major swizzled P tile; per tile: O + b2 staged (in
//              the P tile's shared memory) and bulk-reduce-added into x
// TMEM holds one S chunk and O, so D + 128 <= 512.
namespace ffn {
constexpr int kBM = 128, kBH = 128, kBK = 64;
constexpr uint32_t kBlock = kBM * kBK * 2;  // one 128x64 16-bit block (16 KB)
constexpr uint32_t kStage = 2 * kBlock;      // ring stage: two blocks, 8 MMAs per wait and commit
constexpr int kStages = 3;
constexpr int kMaxD = 384;
constexpr uint32_t kStgBytes = 4096;  // per epilogue warp: 32 x 32 fp32, inside the P tile
constexpr size_t kSmem = 1024 + (kMaxD / kBK) * kBlock + 2 * kBlock + kStages * kStage + 256;
}  // namespace ffn

template <typename T>
__global__ void __launch_bounds__(320, 1)
    ffn_fused_kernel(const __grid_constant__ CUtensorMap map_xn, const __grid_constant__ CUtensorMap map_w1,
                     const __grid_constant__ CUtensorMap map_w2, const __grid_constant__ CUtensorMap map_x,
                     const __grid_constant__ FfnParams p) {
  using namespace ffn;
  constexpr uint32_t kIsBf16 = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sX = smem;                              // D/64 blocks
  uint8_t* sP = sX + (kMaxD / kBK) * kBlock;       // 2 blocks (128 rows x 128 hidden)
  uint8_t* sW = sP + 2 * kBlock;                   // ring
  // The O epilogue stages through the P tile: it runs after the tile's last O MMAs
  // (which read the last P) completed and before the same warps write the next P.
  uint8_t* sEpi = sP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sW + kStages * kStage);
  uint64_t* x_full = bars;
  uint64_t* x_empty = bars + 1;
  uint64_t* w_full = bars + 2;
  uint64_t* w_empty = w_full + kStages;
  uint64_t* s_full = w_empty + kStages;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_full = s_free + 1;
  uint64_t* p_free = p_full + 1;
  uint64_t* o_full = p_free + 1;
  uint64_t* o_free = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = p.D / kBK;      // k-blocks of S
  const int J = p.H / kBH;        // hidden chunks
  const int ntiles = (p.m + kBM - 1) / kBM;
  // this CTA's (tile, hidden chunk) units; the grid is at most ntiles CTAs, so every
  // range holds at least J units and a tile is split between at most two CTAs
  const UnitRange range(ntiles, J, (int)blockIdx.x, (int)gridDim.x);
  if (threadIdx.x == 0) {
    mbar_init(x_full, 1);
    mbar_init(x_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 8);
    mbar_init(p_full, 8);
    mbar_init(p_free, 1);
    mbar_init(o_full, 1);
    mbar_init(o_free, 8);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_xn);
    tma_prefetch_desc(&map_w1);
    tma_prefetch_desc(&map_w2);
    tma_prefetch_desc(&map_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      // one stage = two 128x64 boxes: (x, y) and (x + dx, y + dy)
      auto load_w = [&](const CUtensorMap* map, int x, int y, int dx, int dy) -> bool {
        if (!mbar_wait(&w_empty[st], ph ^ 1u, kErrTimeoutSmemEmpty, abort_flag)) return false;
        mbar_arrive_expect_tx(&w_full[st], kStage);
        tma_load_2d(sW + st * kStage, map, &w_full[st], x, y);
        tma_load_2d(sW + st * kStage + kBlock, map, &w_full[st], x + dx, y + dy);
        if (++st == kStages) {
          st = 0;
          ph ^= 1u;
        }
        return true;
      };
      for (int lt = 0; ok && lt < range.nseg; ++lt) {
        int t, j0, j1;
        range.seg(lt, t, j0, j1);
        if (!mbar_wait(x_empty, (lt & 1) ^ 1u, kErrTimeoutSmemEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(x_full, nkb * kBlock);
        for (int kb = 0; kb < nkb; ++kb) tma_load_2d(sX + kb * kBlock, &map_xn, x_full, kb * kBK, t * kBM);
        // consumption order: S_j0, then (S_{j+1}, O_j) for j = j0..j1-1; an S stage holds
        // k-blocks kb, kb+1 of W1_j, an O stage the chunk's two 64-column halves of W2
        // rows n3*128..
        for (int kb = 0; ok && kb < nkb; kb += 2) ok = load_w(&map_w1, kb * kBK, j0 * kBH, kBK, 0);
        for (int j = j0; ok && j < j1; ++j) {
          if (j + 1 < j1)
            for (int kb = 0; ok && kb < nkb; kb += 2) ok = load_w(&map_w1, kb * kBK, (j + 1) * kBH, kBK, 0);
          // O stages: each 256-row piece of W2 per 64-column hidden half (two 128-row
          // boxes), then a last 128-row piece with both hidden halves
          for (int r = 0; ok && r < p.D / 256; ++r)
            for (int kb2 = 0; ok && kb2 < kBH / kBK; ++kb2) ok = load_w(&map_w2, j * kBH + kb2 * kBK, r * 256, 0, kBM);
          if (ok && p.D % 256 != 0) ok = load_w(&map_w2, j * kBH, (p.D / 256) * 256, kBK, 0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(kIsBf16, 128, 0);
      const uint32_t idesc256 = umma_idesc_f16(kIsBf16, 256, 0);
      const uint32_t tS = tmem, tO = tmem + 128;
      int st = 0;
      uint32_t ph = 0;
      uint32_t sc = 0, pc = 0;  // S chunks issued, P chunks consumed
      bool ok = true;
      auto issue_s = [&]() -> bool {
        if (!mbar_wait(s_free, (sc & 1) ^ 1u, kErrTimeoutFfnS, abort_flag)) return false;
        tc_fence_after();
        for (int kb = 0; kb < nkb; kb += 2) {
          if (!mbar_wait(&w_full[st], ph, kErrTimeoutTmaFull, abort_flag)) return false;
          tc_fence_after();
          // descriptors of the stage's first k-step; each further 16-element k-step is
          // +32 bytes (+2 in the start-address field), the second block +16 KB
          const uint64_t da = sw128_desc(smem_u32(sX + kb * kBlock), 16, 1024);
          const uint64_t db = sw128_desc(smem_u32(sW + st * kStage), 16, 1024);
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              const uint64_t off = (uint64_t)(h * (kBlock >> 4) + kk * 2);
              umma_f16_ss(tS, da + off, db + off, idesc, (kb | h | kk) != 0 ? 1u : 0u);
            }
          umma_commit(&w_empty[st]);
          if (++st == kStages) {
            st = 0;
            ph ^= 1u;
          }
        }
        umma_commit(s_full);
        ++sc;
        return true;
      };
      auto issue_o = [&](bool first) -> bool {
        if (!mbar_wait(p_full, pc & 1, kErrTimeoutFfnP, abort_flag)) return false;
        tc_fence_after();
        const uint64_t da = sw128_desc(smem_u32(sP), 16, 1024);
        // 256-row pieces: N = 256 MMAs over one hidden half per stage
        for (int r = 0; r < p.D / 256; ++r) {
          for (int kb2 = 0; kb2 < kBH / kBK; ++kb2) {
            if (!mbar_wait(&w_full[st], ph, kErrTimeoutTmaFull, abort_flag)) return false;
            tc_fence_after();
            const uint64_t db = sw128_desc(smem_u32(sW + st * kStage), 16, 1024);
            const uint32_t dO = tO + (uint32_t)(r * 256);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_f16_ss(dO, da + (uint64_t)(kb2 * (kBlock >> 4) + kk * 2), db + (uint64_t)(kk * 2), idesc256,
                          (first && kb2 == 0 && kk == 0) ? 0u : 1u);
            umma_commit(&w_empty[st]);
            if (++st == kStages) {
              st = 0;
              ph ^= 1u;
            }
          }
        }
        // last 128-row piece: N = 128 over both hidden halves in one stage
        if (p.D % 256 != 0) {
          if (!mbar_wait(&w_full[st], ph, kErrTimeoutTmaFull, abort_flag)) return false;
          tc_fence_after();
          const uint64_t db = sw128_desc(smem_u32(sW + st * kStage), 16, 1024);
          const uint32_t dO = tO + (uint32_t)((p.D / 256) * 256);
#pragma unroll
          for (int kb2 = 0; kb2 < kBH / kBK; ++kb2)
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              const uint64_t off = (uint64_t)(kb2 * (kBlock >> 4) + kk * 2);
              umma_f16_ss(dO, da + off, db + off, idesc, (first && kb2 == 0 && kk == 0) ? 0u : 1u);
            }
          umma_commit(&w_empty[st]);
          if (++st == kStages) {
            st = 0;
            ph ^= 1u;
          }
        }
        umma_commit(p_free);
        ++pc;
        return true;
      };
      for (int lt = 0; ok && lt < range.nseg; ++lt) {
        int t, j0, j1;
        range.seg(lt, t, j0, j1);
        if (!mbar_wait(x_full, lt & 1, kErrTimeoutTmaFull, abort_flag)) break;
        tc_fence_after();
        ok = issue_s();
        for (int j = j0; ok && j < j1; ++j) {
          if (j + 1 < j1) {
            ok = issue_s();
            if (ok && j + 2 == j1) umma_commit(x_empty);  // the segment's last S reads xn
          } else if (j1 - j0 == 1) {
            umma_commit(x_empty);
          }
          if (!ok) break;
          if (j == j0) {
            // O of the previous tile drained by the epilogue
            if (!mbar_wait(o_free, (lt & 1) ^ 1u, kErrTimeoutFfnO, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          ok = issue_o(j == j0);
        }
        if (!ok) break;
        umma_commit(o_full);
      }
    }
  } else {
    // ------------------------------------------------------------ GELU + O epilogue (8 warps)
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = q * 32 + lane;  // row within the tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    // staging = the 4 KB of the P tile this warp writes (rows q*32.. of block `half`),
    // so waiting for its own bulk reads is enough before it writes P again
    uint8_t* stg = sEpi + (half * 4 + q) * kStgBytes;
    uint32_t sc = 0, pc = 0;
    bool ok = true;
    for (int lt = 0; ok && lt < range.nseg; ++lt) {
      int t, j0, j1;
      range.seg(lt, t, j0, j1);
      for (int j = j0; j < j1; ++j) {
        if (!mbar_wait(s_full, sc & 1, kErrTimeoutFfnS, abort_flag)) {
          ok = false;
          break;
        }
        ++sc;
        tc_fence_after();
        uint32_t ra[32], rb[32];
        tmem_ld32(tmem + lane_off + (uint32_t)(half * 64), ra);
        tmem_ld32(tmem + lane_off + (uint32_t)(half * 64 + 32), rb);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free);
        // bias + GELU, packed to 16-bit pairs: pk[0..15] columns half*64 + [0, 32), pk[16..31] + [32, 64)
        uint32_t pk[32];
        const float* b1 = p.b1 + j * kBH + half * 64;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const uint32_t(&rr)[32] = u == 0 ? ra : rb;
          const float4* b4 = reinterpret_cast<const float4*>(b1 + 32 * u);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 b = __ldg(b4 + q4);
            const float2 lo = gelu2(__fadd2_rn(make_float2(__uint_as_float(rr[4 * q4]), __uint_as_float(rr[4 * q4 + 1])),
                                               make_float2(b.x, b.y)));
            const float2 hi = gelu2(__fadd2_rn(
                make_float2(__uint_as_float(rr[4 * q4 + 2]), __uint_as_float(rr[4 * q4 + 3])), make_float2(b.z, b.w)));
            pk[16 * u + 2 * q4] = pack2<T>(lo.x, lo.y);
            pk[16 * u + 2 * q4 + 1] = pack2<T>(hi.x, hi.y);
          }
        }
        // P_{j-1} consumed by its O MMAs
        if (!mbar_wait(p_free, (pc & 1) ^ 1u, kErrTimeoutFfnP, abort_flag)) {
          ok = false;
          break;
        }
        // the previous tile's O reduce-adds have read this warp's staging (= its P rows)
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
        // row r of the K-major 128B-swizzled P block `half` (64 hidden columns)
        uint8_t* prow = sP + half * kBlock + r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        ++pc;
      }
      if (!ok) break;
      // O epilogue: columns [half * D/2, (half + 1) * D/2) of rows t*128 + r
      if (!mbar_wait(o_full, lt & 1, kErrTimeoutFfnO, abort_flag)) break;
      tc_fence_after();
      // a split tile: the later chunks' part (tail part, j0 > 0, this CTA's first
      // segment) adds its partial first; the part holding chunk 0 (head part, the
      // range's last segment) adds O + b2 once the matching warp of the next CTA has
      // released its flag
      const bool tail_part = j0 > 0, head_part = j1 < J;
      unsigned* my_flag = p.flags + (size_t)blockIdx.x * 8 + (warp - 2);
      if (head_part) {
        if (lane == 0) ok = flag_wait(my_flag + 8, p.epoch, kErrTimeoutFfnFlag, abort_flag);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
      const int row0 = t * kBM + q * 32;
      for (int c0 = half * (p.D / 2); c0 < (half + 1) * (p.D / 2); c0 += 32) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_off + 128u + (uint32_t)c0, rr);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(rr[i]);
        if (p.b2 != nullptr && !tail_part) {
          const float4* b4 = reinterpret_cast<const float4*>(p.b2 + c0);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 b = __ldg(b4 + q4);
            v[4 * q4] += b.x;
            v[4 * q4 + 1] += b.y;
            v[4 * q4 + 2] += b.z;
            v[4 * q4 + 3] += b.w;
          }
        }
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
        stage_row<float, false>(stg, lane, v);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && row0 < p.m) {
          tma_reduce_add_3d(&map_x, stg, c0, row0, 0);
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
      if (tail_part) {
        // the partial's reduce-adds have been performed before the flag is released
        if (lane == 0) {
          bulk_wait0();
          flag_release(my_flag, p.epoch);
        }
        __syncwarp();
      }
    }
    if (lane == 0) bulk_wait0();
    __syncwarp();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

cudaError_t launch_gemm(const CUtensorMap& map_a, const CUtensorMap& map_b, const CUtensorMap& map_out,
                        const GemmParams& p, int epilogue, int bn, int bf16, int num_sms, cudaStream_t stream) {
  if (p.num_groups < 1 || p.num_groups > kGemmMaxGroups) return cudaErrorInvalidValue;
  for (int i = 0; i < p.num_groups; ++i) {
    const GemmGroup& g = p.groups[i];
    if (g.k <= 0 || (g.k % kGemmBK) != 0 || g.m < 0 || g.n <= 0) return cudaErrorInvalidValue;
    if (epilogue == kEpiGlu32 && (g.n % 2) != 0) return cudaErrorInvalidValue;
  }
  if (epilogue == kEpiQkvRope && (p.rope_cols % 32 != 0 || p.head_dim % 32 != 0)) return cudaErrorInvalidValue;
  if (bn == 256)
    return bf16 ? dispatch_epi<256, __nv_bfloat16>(map_a, map_b, map_out, p, epilogue, num_sms, stream)
                : dispatch_epi<256, __half>(map_a, map_b, map_out, p, epilogue, num_sms, stream);
  if (bn == 128)
    return bf16 ? dispatch_epi<128, __nv_bfloat16>(map_a, map_b, map_out, p, epilogue, num_sms, stream)
                : dispatch_epi<128, __half>(map_a, map_b, map_out, p, epilogue, num_sms, stream);
  if (bn == 192)
    return bf16 ? dispatch_epi<192, __nv_bfloat16>(map_a, map_b, map_out, p, epilogue, num_sms, stream)
                : dispatch_epi<192, __half>(map_a, map_b, map_out, p, epilogue, num_sms, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_ffn_fused(const CUtensorMap& map_xn, const CUtensorMap& map_w1, const CUtensorMap& map_w2,
                             const CUtensorMap& map_x, const FfnParams& p, int bf16, int num_sms, cudaStream_t stream) {
  if (p.m < 0 || p.D % ffn::kBM != 0 || p.D > ffn::kMaxD || p.H % ffn::kBH != 0 || p.H <= 0 || p.b1 == nullptr ||
      p.flags == nullptr)
    return cudaErrorInvalidValue;
  if (p.m == 0) return cudaSuccess;
  auto kern = bf16 ? ffn_fused_kernel<__nv_bfloat16> : ffn_fused_kernel<__half>;
  static std::atomic<unsigned long long> configured[2];
  cudaError_t e = ensure_smem_limit(kern, (int)ffn::kSmem, configured[bf16 ? 1 : 0]);
  if (e != cudaSuccess) return e;
  const int ntiles = (p.m + ffn::kBM - 1) / ffn::kBM;
  const int grid = ntiles < num_sms ? ntiles : num_sms;
  // algorithmic cost: both GEMMs; bytes = xn, W1, W2 read once, x read and written once
  const double flop = 4.0 * p.m * (double)p.D * p.H;
  const double bytes = (double)p.m * p.D * (2.0 + 8.0) + 2.0 * p.D * (double)p.H * (bf16 ? 2.0 : 2.0);
  LaunchScope scope("ffn_fused", flop, bytes, stream);
  kern<<<grid, 320, ffn::kSmem, stream>>>(map_xn, map_w1, map_w2, map_x, p);
  return cudaGetLastError();
}

MSST_DEFINE_ERROR_ACCESSOR(gemm_device_error)

}  // namespace msst
