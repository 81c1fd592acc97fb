// gemm.cuh — host-visible description of the grouped tcgen05 GEMM.
//
//   out_g = epilogue( A_g[m_g, k_g] . B_g[n_g, k_g]^T (+ bias_g) )   for each group g
//
// A and B are 16-bit (fp16 or bf16), K-contiguous ("K-major"), read by TMA
// from 2-D tensor maps with 128B swizzle.  Groups let one launch cover the
// per-band MLPs of the Roformer band-split and mask estimator (reference
// src/model_mel_band_roformer.cu:676-685,712-736), which the reference runs as
// 60-62 separate cuBLAS calls each.
//
// Outputs leave through TMA: each epilogue warp stages a 32x32 sub-tile in
// swizzled shared memory and issues a bulk tensor store (16-bit or fp32), or a
// bulk tensor reduce-add for the fp32 residual stream (the addition happens in
// L2; no thread reads the residual).  The output tensor map is 3-D
// {cols, Y, Z}; a group's output element (row, col) goes to coordinates
//   (out_col0 + col, oy0 + oy_row * row, oz0 + oz_row * row)
// so plain row-major outputs, band-strided rows and per-group row clipping are
// all one map.  The GLU epilogue (half-width, group-interleaved columns) uses
// direct stores instead.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace msst {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmMaxGroups = 64;

enum GemmEpilogue : int {
  kEpiStore16 = 0,   // out16 = act(acc + bias)                      (TMA store)
  kEpiResid32 = 1,   // out32 += acc + bias   residual stream update  (TMA reduce-add)
  kEpiStore32 = 2,   // out32  = acc + bias                           (TMA store)
  kEpiGlu32 = 3,     // out32[j] = (acc[2j]+b[2j]) * sigmoid(acc[2j+1]+b[2j+1])  (direct stores)
  kEpiQkvRope = 4,   // out16 = acc with interleaved-pair rotary on the first rope_cols columns (TMA store)
};

enum GemmAct : int { kActNone = 0, kActGelu = 1, kActTanh = 2, kActSigmoid = 3 };

struct GemmGroup {
  int m, n, k;            // output rows, output columns (before GLU halving), reduction length (k % 64 == 0)
  int a_row0, a_col0;     // A coordinates of this group's (0, 0)
  int b_row0, b_col0;     // B coordinates of this group's (0, 0)
  int tiles_n;            // ceil(n / BN)
  int tile_begin;         // first tile index of this group in the launch
  int out_col0;           // first output column (GLU: in halved units)
  int oy0, oy_row;        // TMA output Y coordinate = oy0 + oy_row * row
  int oz0, oz_row;        // TMA output Z coordinate = oz0 + oz_row * row
  long long ldo;          // direct stores: output row stride (elements)
  long long out_row_mul;  // direct stores: output row = row * out_row_mul + out_row_add
  long long out_row_add;
  void* out;              // direct stores: output base
  const float* bias;      // [n] or nullptr
};

struct GemmParams {
  int num_groups;
  int total_tiles;
  int act;
  // kEpiQkvRope: position = (row / pos_div) % pos_mod; cos/sin tables [pos_mod, head_dim/2]
  int pos_div, pos_mod, rope_cols, head_dim;
  const float* rope_cos;
  const float* rope_sin;
  GemmGroup groups[kGemmMaxGroups];
};

// Launches the GEMM.  `map_a` / `map_b` are 2-D tensor maps (inner dim = K) with
// box {64, 128} for A and {64, bn/2} for B (map_gemm_b), 128B swizzle.  Launches
// whose groups all have whole bn-column tiles and enough rows run as CTA pairs
// (256-row tiles, cta_group::2 MMAs; MSST_GEMM_PAIR=0 disables them).  `map_out` is the 3-D
// output map (box {32, 32, 1}; 64B swizzle for 16-bit outputs, 128B swizzle for
// fp32), ignored by kEpiGlu32.  bf16 != 0 selects bf16 operands (else fp16).
// bn in {128, 192, 256}.  Returns a cudaError_t.
cudaError_t launch_gemm(const CUtensorMap& map_a, const CUtensorMap& map_b, const CUtensorMap& map_out,
                        const GemmParams& p, int epilogue, int bn, int bf16, int num_sms, cudaStream_t stream);

// Fused feed-forward block (dim D <= 384, D and H multiples of 128):
//   x[m, D] += GELU(xn . W1^T + b1) . W2^T + b2
// xn [m, D] 16-bit (map box {64, 128}), W1 [H, D] (box {64, 128}), W2 [D, H]
// (box {64, 128}), x fp32 through the residual output map (box {32, 32, 1}).
// The hidden activation never leaves the SM: per 128-row tile the kernel loops
// over H/128 hidden chunks, S = xn . W1_j^T into TMEM, bias + GELU into a 16-bit
// P tile in shared memory, O += P . W2_j^T into TMEM (D columns), then adds O + b2
// to x by bulk tensor reduce-add.
struct FfnParams {
  int m, D, H;
  const float* b1;  // [H]
  const float* b2;  // [D] or nullptr
  // Eight words per CTA (>= 8 x the device's SM count, zero-initialised once) and a
  // value that differs from every earlier launch on the same words: orders the two
  // partial reduce-adds of a 128-row tile whose hidden chunks are split between two
  // neighbouring CTAs.
  unsigned* flags;
  unsigned epoch;
};
cudaError_t launch_ffn_fused(const CUtensorMap& map_xn, const CUtensorMap& map_w1, const CUtensorMap& map_w2,
                             const CUtensorMap& map_x, const FfnParams& p, int bf16, int num_sms, cudaStream_t stream);

}  // namespace msst
