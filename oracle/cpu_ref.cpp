// oracle/cpu_ref.cpp — TEST INFRASTRUCTURE, not product code.
//
// A plain fp32 CPU restatement of the arithmetic on the Roformer hot path of
// HuanLinOTO/CUDA-MSST-Infer.  Only tests/, __graft_entry__.smoke() and
// bench.py's CPU-baseline / reference legs load it, and only as the checker or
// as the timed CPU baseline; the product library never links or calls it.
//
// Parity pinning: the reference ships no tests or golden vectors, so this file
// is pinned against outputs of the reference engine itself, built from its own
// sources by oracle/build_ref.sh and run on a B200 (fixtures in tests/golden/,
// generator tests/golden/make_golden.py).
//
// Every function cites the reference code it restates (paths relative to the
// reference project).  Built by oracle/Makefile into oracle/_build/libmsst_oracle.so.
#include <algorithm>
#include <cmath>
#include <complex>
#include <cstdint>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ---------------------------------------------------------------------------
// C[M,N] = A[M,K] . W[N,K]^T (+ bias[N]); rows of A and W are K-contiguous, as
// in nn.Linear / the reference's cuBLAS column-major trick (src/ops_linear.cu:305-315).
// 4x4 register blocking over (rows of A, rows of W), K innermost so the
// compiler vectorises the dot products.
// ---------------------------------------------------------------------------
void gemm_abt(const float* A, const float* W, const float* bias, float* C, int64_t M, int64_t N,
              int64_t K, int64_t lda, int64_t ldw, int64_t ldc) {
  const int64_t MB = (M + 3) / 4, NB = (N + 3) / 4;
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
  for (int64_t ib = 0; ib < MB; ++ib) {
    for (int64_t jb = 0; jb < NB; ++jb) {
      const int64_t i0 = ib * 4, j0 = jb * 4;
      const int64_t ni = std::min<int64_t>(4, M - i0), nj = std::min<int64_t>(4, N - j0);
      const float* a[4];
      const float* w[4];
      for (int r = 0; r < 4; ++r) a[r] = A + (i0 + std::min<int64_t>(r, ni - 1)) * lda;
      for (int r = 0; r < 4; ++r) w[r] = W + (j0 + std::min<int64_t>(r, nj - 1)) * ldw;
      float acc[4][4] = {};
      // fixed-width lanes keep the inner loop vectorisable and the summation
      // order independent of the thread count
      constexpr int L = 16;
      float part[4][4][L] = {};
      int64_t k = 0;
      for (; k + L <= K; k += L) {
        for (int r = 0; r < 4; ++r)
          for (int c = 0; c < 4; ++c)
            for (int l = 0; l < L; ++l) part[r][c][l] += a[r][k + l] * w[c][k + l];
      }
      for (int r = 0; r < 4; ++r)
        for (int c = 0; c < 4; ++c) {
          float s = 0.f;
          for (int l = 0; l < L; ++l) s += part[r][c][l];
          for (int64_t kk = k; kk < K; ++kk) s += a[r][kk] * w[c][kk];
          acc[r][c] = s;
        }
      for (int r = 0; r < ni; ++r)
        for (int c = 0; c < nj; ++c)
          C[(i0 + r) * ldc + j0 + c] = acc[r][c] + (bias ? bias[j0 + c] : 0.f);
    }
  }
}

// In-place iterative radix-2 complex FFT (sign = -1 forward, +1 inverse, no scaling).
void fft_inplace(std::complex<double>* x, int n, int sign) {
  for (int i = 1, j = 0; i < n; ++i) {
    int bit = n >> 1;
    for (; j & bit; bit >>= 1) j ^= bit;
    j ^= bit;
    if (i < j) std::swap(x[i], x[j]);
  }
  for (int len = 2; len <= n; len <<= 1) {
    const double ang = sign * 2.0 * M_PI / len;
    const std::complex<double> wl(std::cos(ang), std::sin(ang));
    for (int i = 0; i < n; i += len) {
      std::complex<double> w(1.0, 0.0);
      for (int j = 0; j < len / 2; ++j) {
        std::complex<double> u = x[i + j], v = x[i + j + len / 2] * w;
        x[i + j] = u + v;
        x[i + j + len / 2] = u - v;
        w *= wl;
      }
    }
  }
}

inline int64_t reflect_index(int64_t i, int64_t n) {
  // one reflection without edge repeat, then a clamp (src/tensor.cu:394-403)
  if (i < 0)
    i = -i;
  else if (i >= n)
    i = 2 * (n - 1) - i;
  return std::min<int64_t>(std::max<int64_t>(i, 0), n - 1);
}

}  // namespace

extern "C" {

int msst_oracle_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void msst_oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

// RMSNorm as the reference computes it: x * rsqrt(sum(x^2) + 1e-12) * gamma * scale
// (src/ops_norm.cu:85-111; scale = sqrt(D) at every call site, e.g.
// src/model_mel_band_roformer.cu:526,533).  Rows may be strided (ldx, ldo).
void msst_oracle_rmsnorm(const float* x, const float* gamma, float* out, int64_t rows, int64_t D,
                         float scale, int64_t ldx, int64_t ldo) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * ldx;
    double ss = 0.0;
    for (int64_t j = 0; j < D; ++j) ss += (double)xr[j] * xr[j];
    const float inv = 1.0f / std::sqrt((float)ss + 1e-12f);
    float* o = out + r * ldo;
    for (int64_t j = 0; j < D; ++j) o[j] = xr[j] * inv * gamma[j] * scale;
  }
}

// nn.Linear with optional activation (src/ops_linear.cu:150-343,
// src/ops_fused.cu:264-303, src/ops_elementwise.cu:84-88):
// act 0 none, 1 GELU (erf form, src/ops_fused.cu:21-24), 2 sigmoid, 3 tanh.
void msst_oracle_linear(const float* x, const float* w, const float* b, float* out, int64_t rows,
                        int64_t in_f, int64_t out_f, int act) {
  gemm_abt(x, w, b, out, rows, out_f, in_f, in_f, in_f, out_f);
  if (act == 0) return;
  const int64_t n = rows * out_f;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float v = out[i];
    if (act == 1)
      out[i] = 0.5f * v * (1.0f + std::erf(v * 0.70710678118654752f));
    else if (act == 2)
      out[i] = 1.0f / (1.0f + std::exp(-v));
    else
      out[i] = std::tanh(v);
  }
}

// GLU over the last dim: first half * sigmoid(second half) (src/ops_elementwise.cu:321-343).
void msst_oracle_glu(const float* x, float* out, int64_t rows, int64_t half) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t j = 0; j < half; ++j) {
      const float a = x[r * 2 * half + j], g = x[r * 2 * half + half + j];
      out[r * half + j] = a * (1.0f / (1.0f + std::exp(-g)));
    }
}

// Rotary tables exactly as the drivers build them on the host
// (src/model_mel_band_roformer.cu:487-513): angle = n * 10000^(-2i/dim), fp32.
void msst_oracle_rope_tables(int n, int dim, float* cosv, float* sinv) {
  const int half = dim / 2;
  for (int p = 0; p < n; ++p)
    for (int i = 0; i < half; ++i) {
      const float freq = 1.0f / std::pow(10000.0f, (float)(2 * i) / (float)dim);
      const float ang = (float)p * freq;
      cosv[p * half + i] = std::cos(ang);
      sinv[p * half + i] = std::sin(ang);
    }
}

// Interleaved-pair rotation of x [B,H,N,D] in place (src/ops_misc.cu:39-69).
void msst_oracle_rope(float* x, const float* cosv, const float* sinv, int64_t B, int64_t H, int64_t N,
                      int64_t D) {
  const int64_t half = D / 2;
#pragma omp parallel for schedule(static)
  for (int64_t bh = 0; bh < B * H; ++bh)
    for (int64_t n = 0; n < N; ++n) {
      float* r = x + (bh * N + n) * D;
      for (int64_t i = 0; i < half; ++i) {
        const float c = cosv[n * half + i], s = sinv[n * half + i];
        const float x0 = r[2 * i], x1 = r[2 * i + 1];
        r[2 * i] = x0 * c - x1 * s;
        r[2 * i + 1] = x0 * s + x1 * c;
      }
    }
}

// Non-causal softmax(scale * Q K^T) V over q,k,v [B,H,N,D] (src/ops_attention.cu:522-599,
// softmax src/ops_attention.cu:390-452).
void msst_oracle_attention(const float* q, const float* k, const float* v, float* out, int64_t B,
                           int64_t H, int64_t N, int64_t Nk, int64_t D, float scale) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t bh = 0; bh < B * H; ++bh) {
    const float* Q = q + bh * N * D;
    const float* K = k + bh * Nk * D;
    const float* V = v + bh * Nk * D;
    float* O = out + bh * N * D;
    std::vector<float> s(Nk);
    std::vector<double> acc(D);
    for (int64_t i = 0; i < N; ++i) {
      float mx = -INFINITY;
      for (int64_t j = 0; j < Nk; ++j) {
        float d = 0.f;
        for (int64_t c = 0; c < D; ++c) d += Q[i * D + c] * K[j * D + c];
        s[j] = d * scale;
        mx = std::max(mx, s[j]);
      }
      double sum = 0.0;
      for (int64_t j = 0; j < Nk; ++j) {
        s[j] = std::exp(s[j] - mx);
        sum += s[j];
      }
      std::fill(acc.begin(), acc.end(), 0.0);
      for (int64_t j = 0; j < Nk; ++j)
        for (int64_t c = 0; c < D; ++c) acc[c] += (double)s[j] * V[j * D + c];
      for (int64_t c = 0; c < D; ++c) O[i * D + c] = (float)(acc[c] / sum);
    }
  }
}

// LayerNorm over the last dimension as src/ops_norm.cu:150-182 computes it: mean,
// then the biased variance of (x - mean), y = (x - mean) * rsqrt(var + eps) * gamma + beta
// (double accumulation here; the reference sums in fp32).
void msst_oracle_layernorm(const float* x, const float* gamma, const float* beta, float* out, int64_t rows,
                           int64_t D, float eps) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * D;
    double s = 0.0;
    for (int64_t j = 0; j < D; ++j) s += xr[j];
    const double mean = s / (double)D;
    double ss = 0.0;
    for (int64_t j = 0; j < D; ++j) ss += (xr[j] - mean) * (xr[j] - mean);
    const double inv = 1.0 / std::sqrt(ss / (double)D + (double)eps);
    float* o = out + r * D;
    for (int64_t j = 0; j < D; ++j) o[j] = (float)((xr[j] - mean) * inv * gamma[j] + beta[j]);
  }
}

// Periodic Hann window, torch.hann_window default (src/ops_stft.cu:253-259).
void msst_oracle_hann(int n, float* w) {
  for (int i = 0; i < n; ++i) w[i] = 0.5f * (1.0f - std::cos(2.0f * (float)M_PI * (float)i / (float)n));
}

// torch.stft(center=True, reflect pad, onesided) as src/ops_stft.cu:286-365:
// signal [B, L] -> out [B, n_fft/2+1, T, 2], T = L / hop + 1.  n_fft must be a power of two.
void msst_oracle_stft(const float* sig, int64_t B, int64_t L, int n_fft, int hop, const float* win,
                      float* out) {
  const int64_t pad = n_fft / 2, Lp = L + 2 * pad;
  const int64_t T = (Lp - n_fft) / hop + 1, F = n_fft / 2 + 1;
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
  for (int64_t b = 0; b < B; ++b)
    for (int64_t t = 0; t < T; ++t) {
      std::vector<std::complex<double>> buf(n_fft);
      for (int n = 0; n < n_fft; ++n) {
        const int64_t src = reflect_index(t * hop + n - pad, L);
        buf[n] = std::complex<double>((double)sig[b * L + src] * win[n], 0.0);
      }
      fft_inplace(buf.data(), n_fft, -1);
      for (int64_t f = 0; f < F; ++f) {
        float* o = out + ((b * F + f) * T + t) * 2;
        o[0] = (float)buf[f].real();
        o[1] = (float)buf[f].imag();
      }
    }
}

// torch.istft(center=True) as src/ops_stft.cu:371-489: C2R inverse (imaginary parts of
// the DC and Nyquist bins ignored, as cuFFT's C2R does), 1/n_fft, window, overlap-add,
// divide by the summed squared window where it exceeds 1e-8, trim n_fft/2 each side.
// spec [B, F, T, 2] -> out [B, (T-1)*hop] (length = n_fft + (T-1)*hop - n_fft); with
// trim = 0 the whole n_fft + (T-1)*hop samples per row.
void msst_oracle_istft(const float* spec, int64_t B, int64_t T, int n_fft, int hop, const float* win,
                       float* out, int trim) {
  const int64_t F = n_fft / 2 + 1;
  const int64_t full = n_fft + (T - 1) * hop, pad = trim ? n_fft / 2 : 0, Lout = full - 2 * pad;
  std::vector<float> wsum(full, 0.f);
  for (int64_t t = 0; t < T; ++t)
    for (int n = 0; n < n_fft; ++n) wsum[t * hop + n] += win[n] * win[n];
  std::vector<float> frames((size_t)B * T * n_fft);
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
  for (int64_t b = 0; b < B; ++b)
    for (int64_t t = 0; t < T; ++t) {
      std::vector<std::complex<double>> buf(n_fft);
      for (int64_t f = 0; f < F; ++f) {
        const float* s = spec + ((b * F + f) * T + t) * 2;
        double im = (f == 0 || f == F - 1) ? 0.0 : (double)s[1];
        buf[f] = std::complex<double>((double)s[0], im);
      }
      for (int64_t f = 1; f < n_fft / 2; ++f) buf[n_fft - f] = std::conj(buf[f]);
      fft_inplace(buf.data(), n_fft, +1);
      float* fr = frames.data() + (b * T + t) * n_fft;
      for (int n = 0; n < n_fft; ++n) fr[n] = (float)(buf[n].real() / n_fft) * win[n];
    }
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < B; ++b) {
    std::vector<double> acc(full, 0.0);
    for (int64_t t = 0; t < T; ++t)
      for (int n = 0; n < n_fft; ++n) acc[t * hop + n] += frames[(b * T + t) * n_fft + n];
    for (int64_t i = 0; i < Lout; ++i) {
      const int64_t p = i + pad;
      const float ws = wsum[p];
      out[b * Lout + i] = ws > 1e-8f ? (float)(acc[p] / ws) : (float)acc[p];
    }
  }
}

// MelBandRoformer band tables when a .csm carries no __precomputed__ tensors:
// the reference derives them from its HTK-scale triangular filterbank
// (ops::mel_filterbank, src/ops_misc.cu:469-525, thresholded at > 0 with the
// first and last corners forced to 1 in compute_mel_bands,
// src/model_mel_band_roformer.cu:214-240).  fp32 arithmetic in the reference's
// order, contraction into FMAs off (membership is decided by exact comparisons).
// Writes nfreq[num_bands], the bins of every band in order into bins
// (capacity num_bands * (n_fft/2+1)) and the number of bands per bin into count;
// returns the total number of (band, bin) pairs, or -1 if a band is empty.
__attribute__((optimize("fp-contract=off"))) int msst_oracle_mel_bands_htk(int sr, int n_fft, int num_bands,
                                                                         int* nfreq, int* bins, int* count) {
  const int nbins = n_fft / 2 + 1;
  auto mel = [](float f) { return 2595.0f * std::log10(1.0f + f / 700.0f); };
  auto hz = [](float m) { return 700.0f * (std::pow(10.0f, m / 2595.0f) - 1.0f); };
  const float m0 = mel(0.0f), m1 = mel((float)sr / 2.0f);
  std::vector<float> pt(num_bands + 2);
  for (int i = 0; i <= num_bands + 1; ++i) pt[i] = hz(m0 + (m1 - m0) * (float)i / (float)(num_bands + 1));
  for (int f = 0; f < nbins; ++f) count[f] = 0;
  int total = 0;
  for (int b = 0; b < num_bands; ++b) {
    int n = 0;
    for (int f = 0; f < nbins; ++f) {
      const float fr = (float)sr * (float)f / (float)n_fft;
      const float l = pt[b], c = pt[b + 1], r = pt[b + 2];
      float v = 0.0f;
      if (fr >= l && fr <= c) {
        if (c - l > 0.0f) v = (fr - l) / (c - l);
      } else if (fr > c && fr <= r) {
        if (r - c > 0.0f) v = (r - fr) / (r - c);
      }
      if ((b == 0 && f == 0) || (b == num_bands - 1 && f == nbins - 1)) v = 1.0f;
      if (v > 0.0f) {
        bins[total++] = f;
        ++count[f];
        ++n;
      }
    }
    if (n == 0) return -1;
    nfreq[b] = n;
  }
  return total;
}

}  // extern "C"
