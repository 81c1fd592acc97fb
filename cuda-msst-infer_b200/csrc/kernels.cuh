// kernels.cuh — launchers for the memory-bound kernels of the Roformer path.
#pragma once

#include <cuda_runtime.h>
#include <cufft.h>
#include <stdint.h>

namespace msst {

// RMSNorm as the reference defines it (src/ops_norm.cu:85-111):
//   y = x * rsqrt(sum(x^2) + 1e-12) * gamma * scale
// One warp per row, D % 128 == 0, D <= 1024.  Optional stages, in order:
//   gamma_pre: x <- RMSNorm(x; gamma_pre, scale_pre) written back to x (fp32)
//              (the MelBandRoformer per-transformer final norm, fused into the
//              next transformer's first pre-norm)
//   gamma:     y  = RMSNorm(x; gamma, scale) -> out16 (fp16/bf16), row r written at
//              out row  (r % F) * (rows / F) + r / F  when band_major, else r
//   wg/bg:     gates[r, h] = sigmoid(y . wg[h] + bg[h])  (the attention gate
//              projection, src/model_mel_band_roformer.cu:575)
struct RmsNormArgs {
  float* x;
  long long rows;
  int D;
  const float* gamma_pre;
  float scale_pre;
  const float* gamma;
  float scale;
  void* out16;
  int band_major;
  int F;
  const float* wg;
  const float* bg;
  float* gates;
  int heads;
};
cudaError_t launch_rmsnorm(const RmsNormArgs& a, int bf16, cudaStream_t s);

// LayerNorm over the last dimension (ops::layer_norm, src/ops_norm.cu:150-182,496-533):
// y = (x - mean) * rsqrt(var + eps) * gamma + beta, var the biased variance,
// x fp32 [rows, D] (D % 4 == 0, D <= 1024) -> out [rows, D] as fp32 (out_kind 0),
// fp16 (1) or bf16 (2).  One warp per row, the row held in registers.
struct LayerNormArgs {
  const float* x;
  long long rows;
  int D;
  const float* gamma;
  const float* beta;
  float eps;
  void* out;
  int out_kind;
};
cudaError_t launch_layernorm(const LayerNormArgs& a, cudaStream_t s);

// Band gather + per-band RMSNorm + 16-bit cast + zero K-padding: builds the A
// operand of the grouped band-split GEMM from the STFT (cuFFT R2C layout
// [Bc*C*T, nbins] complex).  Row bt = b*T + t; band j occupies columns
// [kcol[j], kcol[j] + kpad[j]) with dims[j] = 2*C*nfreq[j] real values ordered
// (bin, channel, re/im) as the reference folds them
// (src/model_mel_band_roformer.cu:808-829, src/model_bs_roformer.cu:465-473).
struct BandInArgs {
  const float2* spec;
  int Bc, C, T, nbins;
  int num_bands;
  const int* bin_start;   // [num_bands] into bin_list
  const int* nfreq;       // [num_bands]
  const int* bin_list;    // mono bin indices, band-concatenated
  const int* kcol;        // [num_bands]
  const int* kpad;        // [num_bands]
  const int* gcol;        // [num_bands] offset into gamma
  const float* gamma;     // concatenated band gammas
  void* out;              // [Bc*T, ld] 16-bit
  long long ld;
  const int* run_first;   // optional [num_bands]: the band's first bin when its bins are an
                          // ascending run (first, first+1, ...), else -1; nullptr: checked here
  float spec_scale;       // the STFT values are multiplied by this first (1, or
                          // 1/sqrt(n_fft) for stft_normalized models, src/ops_stft.cu:358-365)
};
cudaError_t launch_band_input(const BandInArgs& a, int bf16, cudaStream_t s);

// Mask merge + apply (src/model_mel_band_roformer.cu:926-1015,
// src/model_bs_roformer.cu:552-590): for every (b, stem, t, bin) the complex mask
// is the sum of the contributing bands' GLU outputs divided by
// max(count, 1e-8), multiplied into the STFT, DC zeroed when zero_dc; written in
// the cuFFT C2R input layout [(b*S + stem)*C + c][t][bin].
struct MaskApplyArgs {
  const float2* spec;      // [Bc*C*T, nbins]
  const float* mask;       // [S][Bc*T][mask_ld]
  long long mask_stem_stride;
  int mask_ld;
  const int* contrib_off;  // [nbins + 1]
  const int* contrib_col;  // mask column of (bin, channel 0, re) per contribution
  const float* denom;      // [nbins] clamp(count, 1e-8)
  float2* out;             // [Bc*S*C*T, nbins]
  int Bc, S, C, T, nbins;
  int zero_dc;
  float spec_scale;        // out = ((spec * spec_scale) x mask) * out_scale: the normalized
  float out_scale;         // STFT of stft_normalized models and the iSTFT's undoing of it
                           // (src/ops_stft.cu:358-365,380-389); 1 and 1 otherwise
  // optional [nbins] per-bin summary of the tables above, for bins with at most
  // two contributions: {col0, col1 or -1, 0, denom bits}; x = -2 marks a bin that
  // takes the general path.  nullptr: the general path everywhere.
  const int4* bin_pack;
};
cudaError_t launch_mask_apply(const MaskApplyArgs& a, cudaStream_t s);

// STFT framing (torch.stft center=True, reflect pad; src/ops_stft.cu:286-331):
// frames[(bc*T + t)*n_fft + n] = audio[bc, reflect(t*hop + n - n_fft/2)] * win[n].
cudaError_t launch_stft_frames(const float* audio, long long L, int BC, int T, int n_fft, int hop,
                               const float* win, float* frames, cudaStream_t s);

// iSTFT tail (src/ops_stft.cu:411-482): frames are the raw C2R outputs; each
// output sample gathers its <= ceil(n_fft/hop) windowed frames, scales by
// 1/n_fft, divides by the summed squared window where > 1e-8 and drops n_fft/2
// samples of centre padding.  out [BSC, out_len]: the (T-1)*hop reconstructed
// samples, zero-padded to out_len >= (T-1)*hop (the `length` argument of
// ops::istft, src/ops_stft.cu:484-493; out_len = (T-1)*hop is the default).
// ref_compat (only meaningful when out_len > (T-1)*hop): reproduce the
// reference's zero padding of the centre-trimmed slice, whose kernel reads its
// strided source as if it were contiguous (src/tensor.cu:1184-1216 on the view
// of src/ops_stft.cu:476-480): output row r, sample i < (T-1)*hop is the full
// reconstruction (n_fft + (T-1)*hop samples per row) at flat position
// n_fft/2 + r*(T-1)*hop + i.  Row 0 is unaffected; later rows are shifted.
cudaError_t launch_istft_ola(const float* frames, int BSC, int T, int n_fft, int hop, const float* win,
                             const float* wsum, float* out, long long out_len, int ref_compat, cudaStream_t s);

// Skip connections of the Roformer depth loop (src/model_mel_band_roformer.cu:846-852):
// x += skips[0] + skips[1] + ... + skips[count-1], added one at a time in that order
// (the same fp32 sums as the reference's sequence of tensor adds); skips[j] lives
// at skips + j * n.  x and skips 16-byte aligned, n % 4 == 0.
cudaError_t launch_skip_add(float* x, const float* skips, int count, long long n, cudaStream_t s);

// Chunked inference helpers (src/inference_app.cpp:100-324).
// Chunks k of the reflect-padded track: chunk k is padded samples [k*step, k*step +
// chunk).  The padded track is never materialised: padded index p maps to track
// index reflect(p - border).  The final, short chunk is padded to `chunk` samples;
// ref_compat reproduces the reference's contiguous-source indexing of that
// strided slice.
struct ChunkArgs {
  const float* track;      // [C, L] on device
  int C;
  long long L;
  long long border;        // reflect-pad size (0 when not padded)
  long long total;         // padded length
  int chunk;
  int step;
  int ref_compat;
};

// STFT framing of chunks first, first + stride, ... (count of them) straight from
// the track: launch_stft_frames over the batch [count, C, chunk] of those chunks,
// without building it (frames [count*C*T, n_fft]).
cudaError_t launch_stft_frames_chunks(const ChunkArgs& a, int first, int stride, int count, int T, int n_fft,
                                      int hop, const float* win, float* frames, cudaStream_t s);

// Windowed overlap-add stitch of chunk outputs, as a gather over the output
// (src/inference_app.cpp:252-306, src/ops_fused.cu:138-188): for every output
// row r < rows and track sample p in [begin, end), with q = p + border,
//   acc  = sum over the chunks k covering q, in increasing k, of y_k[r, q - k*step] * w_k
//   wsum = sum of the same w_k,   out[r, p] = wsum > 1e-8 ? acc / wsum : acc
// where w_k is the linear fade of chunk/10 samples (dropped at the track's first
// and last chunk).  The sums run in chunk order from zero, as the reference's
// accumulation buffer does, so the result does not depend on how the output is
// split into ranges.  Chunk k's output [rows, chunk] sits at y + slot(k)*rows*chunk,
// slot(k) = (k % slot_ranks) * slot_cap + k / slot_ranks (chunk order when
// slot_ranks = 1; round-robin shards gathered rank after rank otherwise).
struct StitchArgs {
  const float* y;
  int rows;
  int chunk, step, num_chunks;
  long long border, total, L;
  int slot_ranks, slot_cap;
  float* out;              // [rows, L]
  long long begin, end;
};
cudaError_t launch_stitch(const StitchArgs& a, cudaStream_t s);

}  // namespace msst
