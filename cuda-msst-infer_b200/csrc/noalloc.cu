// noalloc.cu — msst_model_transformer_noalloc: one axial transformer applied in
// place, with every intermediate in a fixed device array compiled into the
// library instead of memory obtained from cudaMalloc.
//
// Who needs it: hosts that must never allocate device memory on their processing
// thread.  cudaMalloc / cudaFree can block for milliseconds and implicitly
// synchronise the device, which a real-time audio host (a plugin callback with a
// hard deadline) cannot tolerate, and some embedding applications own every
// device allocation themselves.  Such callers load the model once at start-up and
// then run transformers through this entry point, which allocates nothing.
//
// Limits and sharing:
//   * the array holds kNoAllocScratchBytes (48 MiB) on every GPU that loads the
//     library, for the life of the process;
//   * one call needs 256-byte-aligned regions for the rotary tables
//     (2 * n * 32 floats, n = T or num_bands) and, per token, dim*2 + heads*4 +
//     max(3*heads*64, 4*dim)*2 + heads*64*2 bytes (4,896 B at dim 384, 8 heads):
//     about 10,000 tokens (batch * T * bands) of a MelBandRoformer d384; larger
//     calls are rejected with MSST_ERR_INVALID;
//   * all calls on a device share the one array and it keeps the last call's
//     contents: calls that overlap on the GPU (different streams or threads)
//     race and corrupt each other; every region is fully written before it is
//     read, so nothing needs clearing between calls;
//   * the first call on a device resolves the array's device address
//     (cudaGetSymbolAddress) for that device, and with CUDA's lazy module
//     loading that first use is also when the driver loads this file's module
//     and backs the array with device memory: make one warm-up call per device
//     at start-up, off the real-time thread and before any stream capture;
//     later calls allocate nothing.
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>

#include "attention.cuh"
#include "kernels.cuh"
#include "model.h"
#include "runtime.h"

namespace msst {

constexpr size_t kNoAllocScratchBytes = 48ull << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {};

// Device address of g_noalloc_scratch on the current device (the host-side
// symbol is only a stand-in and must never be handed to a kernel).
unsigned char* scratch_on_current_device() {
  int dev = 0;
  MSST_CUDA(cudaGetDevice(&dev));
  MSST_REQUIRE(dev >= 0 && dev < 64, "device index out of range for the no-alloc scratch");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      fail(MSST_ERR_CUDA, std::string("cudaGetSymbolAddress(no-alloc scratch) failed: ") + cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  return static_cast<unsigned char*>(g_scratch_addr[dev]);
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// cos / sin of the interleaved-pair rotary embedding, [npos, 32] each: angle
// p * 10000^(-2i / head_dim), the values Model::rope_table computes on the host
// (reference src/model_mel_band_roformer.cu:487-513), here with the device's
// powf / cosf / sinf (within a few ulp of the host's).
__global__ void rope_tables_kernel(float* cos_tab, float* sin_tab, int npos, int head_dim) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= npos * 32) return;
  const int p = idx / 32, i = idx % 32;
  const float freq = 1.0f / powf(10000.0f, (float)(2 * i) / (float)head_dim);
  const float ang = (float)p * freq;
  cos_tab[idx] = cosf(ang);
  sin_tab[idx] = sinf(ang);
}

}  // namespace

void Model::transformer_noalloc(int d, int axis, float* x, int B, int T, cudaStream_t s) {
  MSST_REQUIRE(d >= 0 && d < info_.depth && (axis == 0 || axis == 1), "bad depth index or axis");
  MSST_REQUIRE(B > 0 && T > 0, "bad batch or T");
  const msst_model_info& I = info_;
  const int D = I.dim, nb = I.num_bands, H = I.heads;
  const long long M = (long long)B * T * nb;
  const int npos = axis == 0 ? T : nb;
  const size_t big_cols = (size_t)std::max(3 * inner_, ff_);
  const size_t tab_bytes = align256(sizeof(float) * (size_t)npos * 32);
  const size_t xn_bytes = align256(2 * (size_t)M * D);
  const size_t gates_bytes = align256(4 * (size_t)M * H);
  const size_t big_bytes = align256(2 * (size_t)M * big_cols);
  const size_t ao_bytes = align256(2 * (size_t)M * inner_);
  const size_t need = 2 * tab_bytes + xn_bytes + gates_bytes + big_bytes + ao_bytes;
  if (need > kNoAllocScratchBytes)
    fail(MSST_ERR_INVALID, "msst_model_transformer_noalloc: " + std::to_string(M) + " tokens need " +
                               std::to_string(need) + " bytes of scratch, the fixed limit is " +
                               std::to_string(kNoAllocScratchBytes) + " (split the batch)");

  unsigned char* base = scratch_on_current_device();
  float* cos_tab = reinterpret_cast<float*>(base);
  float* sin_tab = reinterpret_cast<float*>(base + tab_bytes);
  unsigned char* xn = base + 2 * tab_bytes;
  float* gates = reinterpret_cast<float*>(xn + xn_bytes);
  unsigned char* big = xn + xn_bytes + gates_bytes;
  unsigned char* ao = big + big_bytes;

  // rotary tables for this axis, filled on the device (no host table, no copy,
  // no stream synchronisation)
  {
    const int n = npos * 32;
    rope_tables_kernel<<<(n + 255) / 256, 256, 0, s>>>(cos_tab, sin_tab, npos, I.dim_head);
    MSST_CUDA(cudaGetLastError());
  }

  // tensor maps over the scratch regions (host-side encoding only)
  const CUtensorMap m_xn = map_2d(xn, M, D, D, kGemmBM);
  const CUtensorMap m_xn_slot = map_2d(xn, M, D, D, (uint32_t)attn_band_slot(nb));
  const CUtensorMap m_ao = map_2d(ao, M, inner_, inner_, kGemmBM);
  const CUtensorMap m_ffh = map_2d(big, M, ff_, ff_, kGemmBM);
  const CUtensorMap mo_qkv = map_out_2d(big, false, M, 3 * inner_, 3 * inner_);
  const CUtensorMap mo_ffh = map_out_2d(big, false, M, ff_, ff_);
  const CUtensorMap mo_x = map_out_2d(x, true, M, D, D);
  const uint64_t C3 = 3 * (uint64_t)inner_;
  CUtensorMap m_qkv;
  if (axis == 0) {
    const uint64_t dims[4] = {C3, (uint64_t)nb, (uint64_t)T, (uint64_t)B};
    const uint64_t str[3] = {C3 * 2, C3 * 2 * nb, C3 * 2 * nb * T};
    const uint32_t box[4] = {64, 1, 128, 1};
    m_qkv = make_tensor_map(big, 4, dims, str, box);
  } else {
    const uint64_t dims[4] = {C3, (uint64_t)M, 1, 1};
    const uint64_t str[3] = {C3 * 2, C3 * 2 * M, C3 * 2 * M};
    const uint32_t box[4] = {64, (uint32_t)attn_band_slot(nb), 1, 1};
    m_qkv = make_tensor_map(big, 4, dims, str, box);
  }

  const TransformerWeights& tw = axis == 0 ? blocks_[d].first : blocks_[d].second;
  const float scale = std::sqrt((float)D);
  auto one = [&](int m, int n, int k, void* out, long long ldo, const float* bias) {
    GemmGroup g{};
    g.m = m;
    g.n = n;
    g.k = k;
    g.out = out;
    g.ldo = ldo;
    g.out_row_mul = 1;
    g.oy_row = 1;
    g.bias = bias;
    return g;
  };
  for (size_t l = 0; l < tw.layers.size(); ++l) {
    const LayerWeights& L = tw.layers[l];
    RmsNormArgs rn{};
    rn.x = x;
    rn.rows = M;
    rn.D = D;
    rn.gamma = L.g_attn.get<float>();
    rn.scale = scale;
    rn.out16 = xn;
    rn.wg = L.wg.get<float>();
    rn.bg = L.bg.get<float>();
    rn.gates = gates;
    rn.heads = H;
    MSST_CUDA(launch_rmsnorm(rn, bf16_, s));
    if (axis == 1 && band_fused_ok()) {
      // band axis: the QKV projection stays on chip (as the allocating path runs it)
      BandAttnParams bp{};
      bp.num_seqs = B * T;
      bp.F = nb;
      bp.slot = attn_band_slot(nb);
      bp.D = D;
      bp.heads = H;
      bp.inner = inner_;
      bp.scale_log2 = (1.0f / std::sqrt((float)I.dim_head)) * 1.4426950408889634f;
      bp.rope_cos = cos_tab;
      bp.rope_sin = sin_tab;
      bp.gates = gates;
      bp.out = ao;
      bp.out_ld = inner_;
      MSST_CUDA(launch_band_attention_fused(m_xn_slot, L.m_wqkv64, bp, bf16_, num_sms_, s));
    } else {
      {
        GemmParams p{};
        p.num_groups = 1;
        p.groups[0] = one((int)M, 3 * inner_, D, big, 3 * inner_, nullptr);
        p.rope_cols = 2 * inner_;
        p.head_dim = I.dim_head;
        p.pos_div = axis == 0 ? nb : 1;
        p.pos_mod = npos;
        p.rope_cos = cos_tab;
        p.rope_sin = sin_tab;
        gemm(m_xn, L.m_wqkv, mo_qkv, p, kEpiQkvRope, L.bn_qkv, s);
      }
      {
        AttnParams a{};
        a.mode = axis;
        a.B = B;
        a.T = T;
        a.F = nb;
        a.heads = H;
        a.num_tokens = (int)M;
        a.scale_log2 = (1.0f / std::sqrt((float)I.dim_head)) * 1.4426950408889634f;
        a.gates = gates;
        a.out = ao;
        if (axis == 0) {
          a.seq_len = T;
          a.q_tiles = (T + 127) / 128;
        } else {
          a.seq_len = nb;
          a.seqs_per_tile = 128 / attn_band_slot(nb);
          a.q_tiles = (int)(((long long)B * T + a.seqs_per_tile - 1) / a.seqs_per_tile);
        }
        MSST_CUDA(launch_attention(m_qkv, a, bf16_, num_sms_, s));
      }
    }
    {
      GemmParams p{};
      p.num_groups = 1;
      p.groups[0] = one((int)M, D, inner_, x, D, nullptr);
      gemm(m_ao, L.m_wout, mo_x, p, kEpiResid32, L.bn_out, s);
    }
    RmsNormArgs rf{};
    rf.x = x;
    rf.rows = M;
    rf.D = D;
    rf.gamma = L.g_ff.get<float>();
    rf.scale = scale;
    rf.out16 = xn;
    MSST_CUDA(launch_rmsnorm(rf, bf16_, s));
    {
      GemmParams p{};
      p.num_groups = 1;
      p.act = kActGelu;
      p.groups[0] = one((int)M, ff_, D, big, ff_, L.b1.get<float>());
      gemm(m_xn, L.m_w1, mo_ffh, p, kEpiStore16, L.bn_w1, s);
    }
    {
      GemmParams p{};
      p.num_groups = 1;
      p.groups[0] = one((int)M, D, ff_, x, D, L.b2.get<float>());
      gemm(m_ffh, L.m_w2, mo_x, p, kEpiResid32, L.bn_w2, s);
    }
  }
  if (mel_) {
    RmsNormArgs rn{};
    rn.x = x;
    rn.rows = M;
    rn.D = D;
    rn.gamma_pre = tw.g_final.get<float>();
    rn.scale_pre = scale;
    MSST_CUDA(launch_rmsnorm(rn, bf16_, s));
  }
}

}  // namespace msst
