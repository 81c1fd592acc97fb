// msst_shim.h — keeps the reference's cudasep::Tensor call sites and its
// exception convention on top of the libmsst_b200 C ABI.  A maintainer adds this
// header to the reference's source tree (it includes the reference's tensor.h and
// ops.h) and re-points the Roformer drivers' ops at these functions; the model
// level (msst_model_*) replaces the drivers' load() / forward() and
// app::run_inference.  Every wrapper throws std::runtime_error with
// msst_last_error() on a non-zero status, as the reference's CUDA_CHECK does
// (src/tensor.h:28-34).
#pragma once

#include <stdexcept>
#include <string>
#include <vector>

#include "msst_b200.h"
#include "ops.h"
#include "tensor.h"

namespace cudasep {
namespace msst {

inline void check(int rc) {
  if (rc != MSST_OK) throw std::runtime_error(std::string("msst_b200: ") + msst_last_error());
}

// the reference's cuBLAS stream (ops.h CudaContext); its custom kernels use the legacy stream
inline void* stream() { return (void*)CudaContext::instance().stream(); }

inline int64_t last_dim(const Tensor& t) { return t.shape().back(); }

// ops::rms_norm(x, gamma, scale) (src/ops_norm.cu:455-491) with a 16-bit (fp16) result,
// the form the following GEMM reads
inline Tensor rms_norm16(const Tensor& x, const Tensor& gamma, float scale) {
  Tensor xf = x.contiguous();
  const int64_t D = last_dim(xf), rows = xf.numel() / D;
  Tensor out = Tensor::empty(xf.shape(), DType::Float16);
  check(msst_rmsnorm(xf.data_f32(), rows, (int)D, gamma.data_f32(), scale, MSST_F16, out.data_ptr(), nullptr,
                     nullptr, 0, nullptr, stream()));
  return out;
}

// ops::linear_gelu(x, W, b) (src/ops_fused.cu:264-282) with x and W already fp16 (the
// reference converts 2-D weights to fp16 at load in --fp16 mode, src/weights.cu:510-524)
inline Tensor linear_gelu16(const Tensor& x16, const Tensor& w16, const Tensor& b) {
  const int64_t K = last_dim(x16), rows = x16.numel() / K, N = w16.shape()[0];
  std::vector<int64_t> shape = x16.shape();
  shape.back() = N;
  Tensor out = Tensor::empty(shape, DType::Float16);
  check(msst_gemm(x16.data_ptr(), rows, (int)K, K, w16.data_ptr(), (int)N, b.data_f32(), MSST_EPI_STORE16,
                  MSST_ACT_GELU, MSST_F16, out.data_ptr(), N, stream()));
  return out;
}

// ops::layer_norm(x, gamma, beta, eps) (src/ops_norm.cu:496-533), fp32 out as the reference returns
inline Tensor layer_norm(const Tensor& x, const Tensor& gamma, const Tensor& beta, float eps = 1e-5f) {
  Tensor xf = x.contiguous();
  const int64_t D = last_dim(xf), rows = xf.numel() / D;
  Tensor out = Tensor::empty(xf.shape(), DType::Float32);
  check(msst_layernorm(xf.data_f32(), rows, (int)D, gamma.data_f32(), beta.data_f32(), eps, MSST_F32,
                       out.data_ptr(), stream()));
  return out;
}

// ops::scaled_dot_product_attention(q, k, v, scale) (src/ops_attention.cu:522-599) on fp16
// q [B,H,N,d], k / v [B,H,Nk,d], d <= 64; scale 0 = 1/sqrt(d)
inline Tensor sdpa16(const Tensor& q16, const Tensor& k16, const Tensor& v16, float scale = 0.0f) {
  const std::vector<int64_t>& qs = q16.shape();
  const int64_t B = qs[0], H = qs[1], N = qs[2], d = qs[3], Nk = k16.shape()[2];
  Tensor q = q16.contiguous(), k = k16.contiguous(), v = v16.contiguous();
  Tensor out = Tensor::empty({B, H, N, d}, DType::Float16);
  check(msst_sdpa(q.data_ptr(), k.data_ptr(), v.data_ptr(), (int)B, (int)H, (int)N, (int)Nk, (int)d, scale,
                  MSST_F16, out.data_ptr(), stream()));
  return out;
}

// A Roformer model behind the drivers' load() / forward() (src/model_mel_band_roformer.h:36-46)
// and app::run_inference (src/inference_app.cpp:443-497).
class Model {
 public:
  Model(const std::string& path, int device, int precision = MSST_F16) {
    check(msst_model_load(path.c_str(), device, precision, &m_));
    check(msst_model_get_info(m_, &info_));
  }
  ~Model() { msst_model_free(m_); }
  Model(const Model&) = delete;
  Model& operator=(const Model&) = delete;
  const msst_model_info& info() const { return info_; }

  // forward(): input [B, C, L] fp32 -> [B, C, L'] (one stem) or [B, S, C, L']
  Tensor forward(const Tensor& input) {
    Tensor in = input.contiguous();
    const std::vector<int64_t>& s = in.shape();
    const int64_t B = s[0], C = s[1], L = s[2];
    const int64_t Lo = info_.match_input_audio_length ? L : (L / info_.hop_length) * info_.hop_length;
    Tensor out = info_.num_stems == 1 ? Tensor::empty({B, C, Lo}) : Tensor::empty({B, info_.num_stems, C, Lo});
    check(msst_model_forward(m_, in.data_f32(), (int)B, (int)C, L, out.data_f32(), stream()));
    return out;
  }

  // run_inference(): chunked separation of a [C, L] track -> [S, C, L] (S dropped for one stem);
  // flags 0 reproduces the reference's output, including its final-chunk padding
  Tensor separate(const Tensor& track, float overlap, int chunk_batch, int flags = 0) {
    Tensor in = track.contiguous();
    const int64_t C = in.shape()[0], L = in.shape()[1];
    Tensor out = info_.num_stems == 1 ? Tensor::empty({C, L}) : Tensor::empty({info_.num_stems, C, L});
    check(msst_model_separate(m_, in.data_f32(), (int)C, L, overlap, chunk_batch, flags, out.data_f32(), stream()));
    return out;
  }

 private:
  msst_model* m_ = nullptr;
  msst_model_info info_{};
};

}  // namespace msst
}  // namespace cudasep
