// model.h — the Roformer model driver of libmsst_b200 (host side, C++17).
//
// Mirrors the reference drivers' public surface (load / forward, reference
// src/model_mel_band_roformer.h:36-46, src/model_bs_roformer.h) and the app
// layer's chunked inference (src/inference_app.cpp:100-324), re-pointed at the
// sm_100a kernels of this library.
#pragma once

#include <cufft.h>

#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "gemm.cuh"
#include "kernels.cuh"
#include "runtime.h"

namespace msst {

struct LayerWeights {
  DeviceBuffer g_attn, wqkv, wg, bg, wout;   // attention (norm gamma, W_qkv, gate W/b, W_out)
  DeviceBuffer g_ff, w1, b1, w2, b2;         // feed-forward
  CUtensorMap m_wqkv, m_wout, m_w1, m_w2;
  // GEMM column tile each B map above was encoded for (its box holds bn/2 rows):
  // every launch that reads a map must pass the same bn
  int bn_qkv = 0, bn_out = 0, bn_w1 = 0, bn_w2 = 0;
  CUtensorMap m_w1_f, m_w2_f;                // 128-row boxes for the fused feed-forward kernel
  CUtensorMap m_wqkv64;                      // 64-row boxes: one head's Q, K or V rows (band_attn.cu)
};

struct TransformerWeights {
  std::vector<LayerWeights> layers;
  DeviceBuffer g_final;  // MelBandRoformer only (norm_output)
};

struct StemWeights {
  std::vector<DeviceBuffer> w, b;  // per MLP layer, all bands concatenated along rows
  std::vector<CUtensorMap> m;
};

// The forward's input: audio [B, C, L], or (chunks != nullptr) chunks first,
// first + stride, ... of a track read in place (L = chunk size).
struct ChunkSource {
  const ChunkArgs* chunks = nullptr;
  int first = 0, stride = 1;
};

class Model {
 public:
  void load(const std::string& path, int device, int precision);
  const msst_model_info& info() const { return info_; }
  int device() const { return device_; }

  void forward(const float* audio, int B, int C, long long L, float* out, cudaStream_t s);
  // Samples per channel that forward() writes for an input of L samples.
  long long out_length(long long L) const;
  void masks(const float* audio, int B, int C, long long L, float* masks_out, cudaStream_t s);
  void transformer(int depth_index, int axis, float* x, int B, int T, cudaStream_t s);
  // One layer's attention block (RMSNorm + gates, QKV + RoPE, attention, out
  // projection, residual) or feed-forward block (RMSNorm, GELU MLP, residual),
  // in place on x [B*T*num_bands, dim] fp32.
  void attn_block(int depth_index, int axis, int layer, float* x, int B, int T, cudaStream_t s);
  void ffn_block(int depth_index, int axis, int layer, float* x, int B, int T, cudaStream_t s);
  // Device tables of the band gather and mask merge (read-only, owned by the model).
  void band_tables(msst_band_tables* t) const;
  // Same as transformer(), with every intermediate in the library's fixed device
  // array (noalloc.cu); allocates nothing.
  void transformer_noalloc(int depth_index, int axis, float* x, int B, int T, cudaStream_t s);
  void separate(const float* track, int C, long long L, float overlap, int chunk_batch, int flags, float* out,
                cudaStream_t s);
  // Host buffers in and out (staged through model-owned device buffers; pinned
  // host memory makes the copies asynchronous DMA).
  void separate_host(const float* track_host, int C, long long L, float overlap, int chunk_batch, int flags,
                     float* out_host);
  // The stream separate_host() runs on (created on first use, on the current device).
  cudaStream_t host_stream();
  void chunk_plan(long long L, float overlap, int* chunk, int* step, long long* border, long long* total,
                  int* num_chunks) const;
  // Sharded separation: forward chunks [first, first + count) of the track's plan
  // into out [count, stems*C, chunk], and stitch all chunk outputs of a track.
  // Chunks first, first + stride, ... (count of them), chunk_batch per forward.
  void forward_chunks(const float* track, int C, long long L, float overlap, int first, int stride, int count,
                      int chunk_batch, int flags, float* out, cudaStream_t s);
  void stitch(const float* chunks, int C, long long L, float overlap, float* out, cudaStream_t s);
  // Stitch output samples [begin, end) from chunk outputs laid out in slots
  // (k % slot_ranks) * slot_cap + k / slot_ranks (StitchArgs).
  void stitch_range(const float* chunks, int slot_ranks, int slot_cap, int C, long long L, float overlap,
                    long long begin, long long end, float* out, cudaStream_t s);
  void chunk_span(long long L, float overlap, int k, int flags, long long* in, long long* out_lo,
                  long long* out_hi) const;

 private:
  struct Work;  // per-(B, T) workspace
  Work& work(int B, int T);
  void run_trunk(int B, int T, cudaStream_t s, Work& w);
  void forward_impl(const float* audio, int B, int C, long long L, float* out, bool fix_padding, cudaStream_t s,
                    const ChunkSource& src = ChunkSource());
  void mel_bands_from_filterbank(std::vector<float>& denom);
  void run_front(const float* audio, const ChunkSource& src, int B, long long L, int T, cudaStream_t s, Work& w);
  void run_masks(int B, int T, cudaStream_t s, Work& w, float* masks_out);
  void run_transformer(int d, int axis, float* x, int B, int T, const float* pending_gamma, cudaStream_t s, Work& w);
  void run_attn_block(int d, int axis, int l, float* x, int B, int T, const float* pending_gamma, cudaStream_t s,
                      Work& w);
  bool ffn_fused_ok() const;
  bool band_fused_ok() const;
  void run_ffn_block(int d, int axis, int l, float* x, int B, int T, cudaStream_t s, Work& w);
  void gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, GemmParams& p, int epi, int bn,
            cudaStream_t s);
  const float* rope_table(int n, bool sine);
  const float* istft_wsum(int T);
  cufftHandle fft_plan(cufftType type, int batch, cudaStream_t s);
  void separate_pipeline(const float* track, const float* track_host, int C, long long L, float overlap,
                         int chunk_batch, int flags, float* out, float* out_host, cudaStream_t s);
  cudaEvent_t pipeline_event(size_t i);
  cudaStream_t copy_stream(int which);

  msst_model_info info_{};
  int device_ = 0;
  int bf16_ = 0;
  bool mel_ = true;
  int C_ = 2, nbins_ = 1025, hid_ = 1536, n_lin_ = 3, inner_ = 512, ff_ = 1536;
  bool zero_dc_ = true;
  bool stft_norm_ = false, skip_ = false, match_len_ = false;
  int num_sms_ = 148;

  std::vector<int> nfreq_, bin_start_, bin_list_, dims_, kpad_, kcol_, dim_off_, out3_off_;
  int ktot_ = 0, sum_dims_ = 0, sum_out3_ = 0;
  DeviceBuffer d_nfreq_, d_bin_start_, d_bin_list_, d_kpad_, d_kcol_, d_gcol_, d_run_first_;
  DeviceBuffer d_contrib_off_, d_contrib_col_, d_denom_, d_bin_pack_;

  DeviceBuffer w_bs_, b_bs_, g_bs_;
  CUtensorMap m_wbs_;
  std::vector<std::pair<TransformerWeights, TransformerWeights>> blocks_;  // (time, band) per depth
  DeviceBuffer final_norm_;                                                  // BSRoformer
  std::vector<StemWeights> stems_;
  DeviceBuffer window_;

  std::map<int, DeviceBuffer> rope_cos_, rope_sin_, wsum_;
  std::map<std::pair<int, int>, cufftHandle> plans_;
  std::map<std::pair<int, int>, std::unique_ptr<Work>> work_;
  DeviceBuffer sep_chunks_;              // chunk outputs of separate(), grown on demand
  DeviceBuffer host_in_, host_out_;      // staging of separate_host()
  cudaStream_t host_stream_ = nullptr;   // stream of separate_host()
  cudaStream_t copy_streams_[2] = {nullptr, nullptr};  // separate_host(): track up, stems down
  std::vector<cudaEvent_t> events_;      // separate_host() pipeline events, grown on demand

 public:
  Model();
  ~Model();
};

}  // namespace msst
