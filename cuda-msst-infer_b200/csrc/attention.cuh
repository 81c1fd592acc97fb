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
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace msst {

struct AttnParams {
  int mode;           // 0 time axis, 1 band axis (packed)
  int B, T, F;        // token grid
  int heads;          // H (head_dim fixed at 64)
  int seq_len;        // T (mode 0) or F (mode 1)
  int q_tiles;        // mode 0: ceil(T/128); mode 1: number of 128-row packed tiles
  int seqs_per_tile;  // mode 1: 128 / attn_band_slot(F)
  int total_items;    // set by launch_attention: pairs of q-tiles x heads (x sequences on the time axis)
  int num_tokens;     // B*T*F
  float scale_log2;   // softmax scale * log2(e)
  const float* gates; // [tokens, heads] (sigmoid already applied) or nullptr
  void* out;          // [tokens, heads*64], 16-bit
};

// Band axis (mode 1): each sequence of F <= 128 tokens occupies an aligned slot of
// 32, 64 or 128 rows of a 128-row tile (seqs_per_tile = 128 / slot), so every
// softmax warp's 32 rows belong to one sequence and its keys span at most
// slot / 32 column chunks.
inline int attn_band_slot(int F) { return F <= 32 ? 32 : (F <= 64 ? 64 : 128); }

// `qkv_map` is a 4-D tensor map over the QKV buffer (inner dim = 3*H*64 columns)
// with box {64, 1, 128, 1} (mode 0: dims {C, F, T, B}) or {64, slot, 1, 1}
// (mode 1: dims {C, tokens, 1, 1}, slot = attn_band_slot(F)), 128B swizzle.
cudaError_t launch_attention(const CUtensorMap& qkv_map, const AttnParams& p, int bf16, int num_sms,
                             cudaStream_t stream);

}  // namespace msst
