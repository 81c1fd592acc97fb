// Test-only harness over the REFERENCE engine (HuanLinOTO/CUDA-MSST-Infer),
// compiled from the reference's own sources by oracle/build_ref.sh into
// oracle/_ref/libcudasep_ref.so.  Nothing in the product links or loads this;
// only tests/ (golden-vector generation, GPU parity) and bench.py's informative
// "ref_gpu" leg call it.
//
// It exposes plain C entry points over the reference's public API
// (app::load_model / app::run_inference, inference_app.cpp:363,443), its model
// forward (model_mel_band_roformer.cu:744, model_bs_roformer.cu:420) and, by
// opening the drivers' private section, the sub-steps forward() is made of, so
// tests can compare the fp32 masks that come out of the mask estimator.
#define private public
#include "model_mel_band_roformer.h"
#include "model_bs_roformer.h"
#undef private
#include "inference_app.h"
#include "ops.h"
#include "flash_attention.cuh"

#include <cmath>
#include <cstring>
#include <string>
#include <vector>

using namespace cudasep;

namespace {

thread_local std::string g_err;

int fail(const std::exception& e) {
  g_err = e.what();
  return -1;
}

int copy_out(const Tensor& t, float* out, long long cap, long long* n_out) {
  Tensor c = t.contiguous();
  std::vector<float> host = c.to_cpu_f32();
  if (n_out) *n_out = (long long)host.size();
  if ((long long)host.size() > cap) {
    g_err = "output buffer too small: need " + std::to_string(host.size());
    return -2;
  }
  std::memcpy(out, host.data(), host.size() * sizeof(float));
  return 0;
}

// Rotary tables for one sequence length, cached the way the drivers cache them
// (model_mel_band_roformer.cu:859-864).
template <class M>
std::pair<Tensor, Tensor>& rope_tables(M& m, int n) {
  auto& c = m.rotary_cache_[n];
  if (c.first.numel() == 0) {
    Tensor rot = m.compute_rotary_cos_sin(n, m.cfg_.dim_head);
    c.first = rot.slice(0, 0, 1).squeeze(0).contiguous();
    c.second = rot.slice(0, 1, 2).squeeze(0).contiguous();
  }
  return c;
}

// Steps 1-9 of the forward pass (STFT .. mask estimator), returning the stacked
// fp32 masks [B, stems, T, sum(band_freq_dims)].  Follows
// model_mel_band_roformer.cu:775-926 and model_bs_roformer.cu:438-552.
template <class M>
Tensor masks_of(M& m, const Tensor& audio, bool mel) {
  auto& cfg = m.cfg_;
  const int64_t batch = audio.size(0), ch = audio.size(1), len = audio.size(2);
  Tensor st = ops::stft(audio.reshape({batch * ch, len}), cfg.stft_n_fft, cfg.stft_hop_length,
                        cfg.stft_win_length, m.stft_window_, true, cfg.stft_normalized);
  const int64_t F = st.size(1), T = st.size(2);
  st = st.reshape({batch, ch, F, T, 2});
  if (ch > 1) st = st.permute({0, 2, 1, 3, 4}).contiguous().reshape({batch, F * ch, T, 2});
  Tensor x;
  if constexpr (std::is_same_v<M, MelBandRoformer>) {
    x = st.index_select(1, m.freq_indices_gpu_);
  } else {
    x = st;
  }
  const int64_t nf = x.size(1);
  x = x.permute({0, 2, 1, 3}).contiguous().reshape({batch, T, nf * 2});
  x = m.apply_band_split(x);
  const int64_t nb = cfg.num_bands, dim = cfg.dim;
  std::vector<Tensor> skips;
  for (int d = 0; d < cfg.depth; ++d) {
    if (cfg.skip_connection)
      for (int j = 0; j < d; ++j) x = x + skips[j];
    x = x.permute({0, 2, 1, 3}).contiguous().reshape({batch * nb, T, dim});
    auto& tt = rope_tables(m, (int)T);
    x = m.apply_transformer(x, m.depth_blocks_[d].time_transformer, tt.first, tt.second);
    x = x.reshape({batch, nb, T, dim}).permute({0, 2, 1, 3}).contiguous();
    x = x.reshape({batch * T, nb, dim});
    auto& ft = rope_tables(m, (int)nb);
    x = m.apply_transformer(x, m.depth_blocks_[d].freq_transformer, ft.first, ft.second);
    x = x.reshape({batch, T, nb, dim});
    if (cfg.skip_connection) skips.push_back(x);
  }
  if constexpr (std::is_same_v<M, BSRoformer>) {
    x = ops::rms_norm(x, m.final_norm_gamma_, std::sqrt((float)dim));
  }
  (void)mel;
  std::vector<Tensor> stems;
  for (int s = 0; s < cfg.num_stems; ++s) stems.push_back(m.apply_mask_estimator(x, m.mask_estimators_[s]));
  return Tensor::stack(stems, 1);
}

}  // namespace

extern "C" {

const char* refh_last_error() { return g_err.c_str(); }

void* refh_load(const char* path, int device, int fp16) {
  try {
    auto* m = new app::LoadedModel(app::load_model(path, device, fp16 != 0));
    return m;
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

void refh_free(void* h) { delete static_cast<app::LoadedModel*>(h); }

// model_type: 1 = MelBandRoformer, 2 = BSRoformer (app::ModelType order).
int refh_info(void* h, int* model_type, int* num_stems, int* sample_rate, int* chunk_size,
              int* num_overlap) {
  auto* m = static_cast<app::LoadedModel*>(h);
  *model_type = (int)m->type;
  *num_stems = m->num_sources;
  *sample_rate = m->sample_rate;
  *chunk_size = m->chunk_size;
  *num_overlap = m->num_overlap;
  return 0;
}

// model.forward on [batch, channels, len] host audio; output copied to host.
int refh_forward(void* h, const float* audio, int batch, int channels, long long len, float* out,
                 long long cap, long long* n_out) {
  try {
    auto* m = static_cast<app::LoadedModel*>(h);
    Tensor in = Tensor::from_cpu_f32(audio, {batch, channels, len});
    Tensor o = m->forward(in);
    cudaDeviceSynchronize();
    return copy_out(o, out, cap, n_out);
  } catch (const std::exception& e) {
    return fail(e);
  }
}

int refh_masks(void* h, const float* audio, int batch, int channels, long long len, float* out,
               long long cap, long long* n_out) {
  try {
    auto* m = static_cast<app::LoadedModel*>(h);
    Tensor in = Tensor::from_cpu_f32(audio, {batch, channels, len});
    Tensor masks;
    if (m->type == app::ModelType::MelBandRoformer)
      masks = masks_of(m->mbr, in, true);
    else if (m->type == app::ModelType::BSRoformer)
      masks = masks_of(m->bsr, in, false);
    else
      throw std::runtime_error("refh_masks: not a Roformer model");
    cudaDeviceSynchronize();
    return copy_out(masks, out, cap, n_out);
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// app::run_inference on one [channels, len] track (chunked overlap-add path).
int refh_separate(void* h, const float* audio, int channels, long long len, float overlap,
                  int chunk_batch, float* out, long long cap, long long* n_out, double* infer_ms) {
  try {
    auto* m = static_cast<app::LoadedModel*>(h);
    if (chunk_batch > 0) m->chunk_batch_size = chunk_batch;
    AudioData a;
    a.samples = Tensor::from_cpu_f32(audio, {channels, len});
    a.sample_rate = m->sample_rate;
    a.channels = channels;
    a.num_samples = len;
    app::InferenceResult r = app::run_inference(*m, a, overlap, nullptr);
    if (infer_ms) *infer_ms = r.infer_ms;
    return copy_out(r.output, out, cap, n_out);
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// ops::scaled_dot_product_attention (ops_attention.cu:522) on host q,k,v [B,H,N,D].
// fp16 != 0 selects the FP16 value-GEMM path (g_quantize_fp16, ops_attention.cu:538).
int refh_sdpa(const float* q, const float* k, const float* v, int B, int H, int N, int D,
              float scale, int fp16, float* out) {
  try {
    bool saved = g_quantize_fp16;
    g_quantize_fp16 = fp16 != 0;
    Tensor tq = Tensor::from_cpu_f32(q, {B, H, N, D});
    Tensor tk = Tensor::from_cpu_f32(k, {B, H, N, D});
    Tensor tv = Tensor::from_cpu_f32(v, {B, H, N, D});
    Tensor o = ops::scaled_dot_product_attention(tq, tk, tv, scale);
    cudaDeviceSynchronize();
    g_quantize_fp16 = saved;
    return copy_out(o, out, (long long)B * H * N * D, nullptr);
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// ops::scaled_dot_product_attention with its own query and key lengths, q [B,H,N,D],
// k,v [B,H,Nk,D] (the cross-attention form of model_htdemucs.cu:640-650); scale 0
// selects the op's default 1/sqrt(D) (ops_attention.cu:541-543).
int refh_sdpa2(const float* q, const float* k, const float* v, int B, int H, int N, int Nk, int D, float scale,
               int fp16, float* out) {
  try {
    bool saved = g_quantize_fp16;
    g_quantize_fp16 = fp16 != 0;
    Tensor tq = Tensor::from_cpu_f32(q, {B, H, N, D});
    Tensor tk = Tensor::from_cpu_f32(k, {B, H, Nk, D});
    Tensor tv = Tensor::from_cpu_f32(v, {B, H, Nk, D});
    Tensor o = ops::scaled_dot_product_attention(tq, tk, tv, scale);
    cudaDeviceSynchronize();
    g_quantize_fp16 = saved;
    return copy_out(o, out, (long long)B * H * N * D, nullptr);
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// ops::layer_norm (ops_norm.cu:496) on host x [rows, D].
int refh_layer_norm(const float* x, const float* gamma, const float* beta, int rows, int D, float eps, float* out) {
  try {
    Tensor tx = Tensor::from_cpu_f32(x, {rows, D});
    Tensor tg = Tensor::from_cpu_f32(gamma, {D});
    Tensor tb = Tensor::from_cpu_f32(beta, {D});
    Tensor o = ops::layer_norm(tx, tg, tb, eps);
    cudaDeviceSynchronize();
    return copy_out(o, out, (long long)rows * D, nullptr);
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// Device time of ops::scaled_dot_product_attention (ops_attention.cu:522) on q,k,v
// [B,H,N,D] uploaded once: `warmup` untimed calls, then `iters` calls bracketed by
// CUDA events on the default stream; *ms_per_call gets the mean.
int refh_sdpa_bench(const float* q, const float* k, const float* v, int B, int H, int N, int D, float scale,
                    int fp16, int warmup, int iters, float* ms_per_call) {
  try {
    bool saved = g_quantize_fp16;
    g_quantize_fp16 = fp16 != 0;
    Tensor tq = Tensor::from_cpu_f32(q, {B, H, N, D});
    Tensor tk = Tensor::from_cpu_f32(k, {B, H, N, D});
    Tensor tv = Tensor::from_cpu_f32(v, {B, H, N, D});
    for (int i = 0; i < warmup; ++i) ops::scaled_dot_product_attention(tq, tk, tv, scale);
    CUDA_CHECK(cudaDeviceSynchronize());
    cudaEvent_t e0, e1;
    CUDA_CHECK(cudaEventCreate(&e0));
    CUDA_CHECK(cudaEventCreate(&e1));
    CUDA_CHECK(cudaEventRecord(e0, 0));
    for (int i = 0; i < iters; ++i) ops::scaled_dot_product_attention(tq, tk, tv, scale);
    CUDA_CHECK(cudaEventRecord(e1, 0));
    CUDA_CHECK(cudaEventSynchronize(e1));
    float ms = 0.f;
    CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    CUDA_CHECK(cudaDeviceSynchronize());
    g_quantize_fp16 = saved;
    *ms_per_call = ms / (float)(iters > 0 ? iters : 1);
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// As refh_sdpa_bench with its own key length Nk (k, v [B,H,Nk,D]).
int refh_sdpa2_bench(const float* q, const float* k, const float* v, int B, int H, int N, int Nk, int D, float scale,
                    int fp16, int warmup, int iters, float* ms_per_call) {
  try {
    bool saved = g_quantize_fp16;
    g_quantize_fp16 = fp16 != 0;
    Tensor tq = Tensor::from_cpu_f32(q, {B, H, N, D});
    Tensor tk = Tensor::from_cpu_f32(k, {B, H, Nk, D});
    Tensor tv = Tensor::from_cpu_f32(v, {B, H, Nk, D});
    for (int i = 0; i < warmup; ++i) ops::scaled_dot_product_attention(tq, tk, tv, scale);
    CUDA_CHECK(cudaDeviceSynchronize());
    cudaEvent_t e0, e1;
    CUDA_CHECK(cudaEventCreate(&e0));
    CUDA_CHECK(cudaEventCreate(&e1));
    CUDA_CHECK(cudaEventRecord(e0, 0));
    for (int i = 0; i < iters; ++i) ops::scaled_dot_product_attention(tq, tk, tv, scale);
    CUDA_CHECK(cudaEventRecord(e1, 0));
    CUDA_CHECK(cudaEventSynchronize(e1));
    float ms = 0.f;
    CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    CUDA_CHECK(cudaDeviceSynchronize());
    g_quantize_fp16 = saved;
    *ms_per_call = ms / (float)(iters > 0 ? iters : 1);
    return 0;
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// The reference's (unused by its own dispatch) scalar flash kernel,
// flash_attention.cuh:260, on host q,k,v [B,H,N,D] fp32.
int refh_flash(const float* q, const float* k, const float* v, int B, int H, int N, int D,
               float scale, float* out) {
  try {
    Tensor tq = Tensor::from_cpu_f32(q, {B, H, N, D});
    Tensor tk = Tensor::from_cpu_f32(k, {B, H, N, D});
    Tensor tv = Tensor::from_cpu_f32(v, {B, H, N, D});
    Tensor o = Tensor::empty({B, H, N, D});
    launch_flash_attention(tq.data_f32(), tk.data_f32(), tv.data_f32(), o.data_f32(), B * H, N, N, D,
                           scale);
    CUDA_CHECK(cudaDeviceSynchronize());
    return copy_out(o, out, (long long)B * H * N * D, nullptr);
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// ops::apply_rotary_emb (ops_misc.cu:73) on host q,k [B,H,N,D], cos/sin [N,D/2]; in place.
int refh_rope(float* q, float* k, const float* cosv, const float* sinv, int B, int H, int N, int D) {
  try {
    Tensor tq = Tensor::from_cpu_f32(q, {B, H, N, D});
    Tensor tk = Tensor::from_cpu_f32(k, {B, H, N, D});
    Tensor tc = Tensor::from_cpu_f32(cosv, {N, D / 2});
    Tensor ts = Tensor::from_cpu_f32(sinv, {N, D / 2});
    ops::apply_rotary_emb(tq, tk, tc, ts);
    cudaDeviceSynchronize();
    long long n = (long long)B * H * N * D;
    int rc = copy_out(tq, q, n, nullptr);
    return rc ? rc : copy_out(tk, k, n, nullptr);
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// ops::rms_norm (ops_norm.cu:455) on host x [rows, D].
int refh_rmsnorm(const float* x, const float* gamma, int rows, int D, float scale, float* out) {
  try {
    Tensor tx = Tensor::from_cpu_f32(x, {rows, D});
    Tensor tg = Tensor::from_cpu_f32(gamma, {D});
    Tensor o = ops::rms_norm(tx, tg, scale);
    cudaDeviceSynchronize();
    return copy_out(o, out, (long long)rows * D, nullptr);
  } catch (const std::exception& e) {
    return fail(e);
  }
}

// ops::linear / linear_gelu / linear_sigmoid (ops_linear.cu:150, ops_fused.cu:264,285).
// act: 0 = none, 1 = gelu, 2 = sigmoid.  fp16 != 0 converts W to fp16 first, as
// ModelWeights::convert_linear_weights_to_fp16 does (weights.cu:510).
int refh_linear(const float* x, const float* w, const float* b, int rows, int in_f, int out_f, int act,
                int fp16, float* out) {
  try {
    Tensor tx = Tensor::from_cpu_f32(x, {rows, in_f});
    Tensor tw = Tensor::from_cpu_f32(w, {out_f, in_f});
    if (fp16) tw = tw.to_f16();
    Tensor tb = Tensor::from_cpu_f32(b, {out_f});
    Tensor o = act == 1 ? ops::linear_gelu(tx, tw, tb)
               : act == 2 ? ops::linear_sigmoid(tx, tw, tb)
                          : ops::linear(tx, tw, tb);
    cudaDeviceSynchronize();
    return copy_out(o, out, (long long)rows * out_f, nullptr);
  } catch (const std::exception& e) {
    return fail(e);
  }
}

}  // extern "C"
