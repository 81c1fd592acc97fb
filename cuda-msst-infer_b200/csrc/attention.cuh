// attention.cuh — host-visible description of the axial attention kernel.
//
// Non-causal softmax(scale * Q K^T) V over the heads of a fused QKV buffer
// [tokens, 3 * heads * 64] (RoPE already applied to Q and K by the QKV GEMM),
// followed by the per-head sigmoid gate and the head merge: the output is written
// as [tokens, heads * 64].  Replaces the reference's split_qkv_heads ->
// apply_rotary_emb -> cuBLAS QK^T -> softmax -> cuBLAS PV -> gate/merge chain
// (src/model_mel_band_roformer.cu:519-591, src/ops_attention.cu:96-181,390-599).
//
// Token layout is the Roformer's [B, T, F] order (token = (b*T + t)*F + f):
//   time axis  (mode 0): sequence (b, f) runs over t with stride F tokens
//   band axis  (mode 1): sequence (b, t) is F consecutive tokens; sequences
//                        shorter than 64 are packed 128/F per 128-row tile with a
//                        block-diagonal mask.
// Mode 2 is the plain op (ops::scaled_dot_product_attention, src/ops_attention.cu:522):
// separate q [B*H, Nq, d] and k, v [B*H, Nk, d] with d <= 64 (the tensor maps
// zero-fill columns d..63), no gates, out [B*H, Nq, d].  It runs the time-axis
// schedule with F = 1 and heads = 1 (B counts the B*H sequences).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace msst {

struct AttnParams {
  int mode;           // 0 time axis, 1 band axis (packed), 2 separate q / k / v
  int B, T, F;        // token grid
  int heads;          // H (head_dim fixed at 64)
  int seq_len;        // T (modes 0, 2) or F (mode 1): query rows per sequence
  int q_tiles;        // modes 0, 2: ceil(T/128); mode 1: number of 128-row packed tiles
  int seqs_per_tile;  // mode 1: 128 / attn_band_slot(F)
  int total_items;    // set by the launchers: work items (pairs of query tiles)
  int units;          // set by the launchers, modes 0 and 2: (sequence, head) units
  int num_tokens;     // B*T*F
  int kv_len;         // key rows per sequence (= seq_len except in mode 2)
  int kv_tiles;       // modes 0, 2: ceil(kv_len/128)
  int k_col, v_col;   // first column of K and V in their tensor maps (head 0)
  long long out_ld;   // output row stride in elements
  int d_out;          // output columns per head (64, or d in mode 2; a multiple of 8)
  float scale_log2;   // softmax scale * log2(e)
  const float* gates; // [tokens, heads] (sigmoid already applied) or nullptr
  void* out;          // [tokens, heads*64] (modes 0, 1) or [B*H*Nq, d] (mode 2), 16-bit
};

// Band axis (mode 1): each sequence of F <= 128 tokens occupies an aligned slot of
// 32, 64 or 128 rows of a 128-row tile (seqs_per_tile = 128 / slot), so every
// softmax warp's 32 rows belong to one sequence and its keys span at most
// slot / 32 column chunks.
inline int attn_band_slot(int F) { return F <= 32 ? 32 : (F <= 64 ? 64 : 128); }

// `qkv_map` is a 4-D tensor map over the QKV buffer (inner dim = 3*H*64 columns)
// with box {64, 1, 128, 1} (mode 0: dims {C, F, T, B}) or {64, slot, 1, 1}
// (mode 1: dims {C, tokens, 1, 1}, slot = attn_band_slot(F)), 128B swizzle; K and
// V are read through the same map at columns k_col / v_col.
cudaError_t launch_attention(const CUtensorMap& qkv_map, const AttnParams& p, int bf16, int num_sms,
                             cudaStream_t stream);

// Mode 2: q_map, k_map, v_map over q [B*H, Nq, d], k / v [B*H, Nk, d], each with
// dims {d, 1, N, B*H} and box {64, 1, 128, 1}, 128B swizzle.
cudaError_t launch_sdpa(const CUtensorMap& q_map, const CUtensorMap& k_map, const CUtensorMap& v_map,
                        const AttnParams& p, int bf16, int num_sms, cudaStream_t stream);

// Band-axis attention block fused with its QKV projection (band_attn.cu):
//   out[token, h*64 .. +64) = gate[token, h] * softmax_F(Q_h K_h^T / 8) V_h
// with [Q_h K_h V_h] = xn . [Wq_h; Wk_h; Wv_h]^T and rotary (interleaved pairs,
// position = the token's band index) on Q_h and K_h, for sequences of F <= 64
// consecutive tokens (one per frame).  map_xn: xn [tokens, D] 16-bit, box {64,
// attn_band_slot(F)}; map_w: W_qkv [3*inner, D] 16-bit, box {64, 64}; both 128B
// swizzle.  D % 64 == 0, D <= 512, head_dim 64.
struct BandAttnParams {
  int num_seqs;            // B*T sequences
  int F;                   // tokens per sequence (num_bands)
  int slot;                // attn_band_slot(F)
  int D;                   // model width (K of the projection)
  int heads;               // H; inner = H*64
  int inner;
  float scale_log2;        // softmax scale * log2(e)
  const float* rope_cos;   // [F, 32]
  const float* rope_sin;   // [F, 32]
  const float* gates;      // [tokens, H] (sigmoid applied) or nullptr
  void* out;               // [tokens, out_ld] 16-bit
  long long out_ld;
};
cudaError_t launch_band_attention_fused(const CUtensorMap& map_xn, const CUtensorMap& map_w, const BandAttnParams& p,
                                        int bf16, int num_sms, cudaStream_t stream);

}  // namespace msst
