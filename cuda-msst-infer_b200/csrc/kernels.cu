// kernels.cu — coalesced memory-bound kernels of the Roformer path (sm_100a).
#include "common.cuh"
#include "kernels.cuh"

namespace msst {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ long long reflect_idx(long long i, long long n) {
  // one reflection without edge repeat, then a clamp (Tensor::pad_reflect, src/tensor.cu:394-403)
  if (i < 0)
    i = -i;
  else if (i >= n)
    i = 2 * (n - 1) - i;
  return i < 0 ? 0 : (i >= n ? n - 1 : i);
}

// ------------------------------------------------------------------ RMSNorm
template <typename T, int V>
__global__ void __launch_bounds__(256) rmsnorm_kernel(RmsNormArgs a) {
  extern __shared__ float s_wg[];  // [heads * D]
  const int lane = threadIdx.x & 31;
  const int D = a.D;
  if (a.wg != nullptr) {
    for (int i = threadIdx.x; i < a.heads * D; i += blockDim.x) s_wg[i] = a.wg[i];
    __syncthreads();
  }
  const long long warps_total = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < a.rows; r += warps_total) {
    float4* xr = reinterpret_cast<float4*>(a.x + r * D);
    float4 v[V];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      v[k] = xr[lane + 32 * k];
      ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
    }
    ss = warp_sum(ss);
    if (a.gamma_pre != nullptr) {
      const float inv = rsqrtf(ss + 1e-12f);
      const float4* g4 = reinterpret_cast<const float4*>(a.gamma_pre);
      ss = 0.f;
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const float4 g = __ldg(g4 + lane + 32 * k);
        v[k].x = v[k].x * inv * g.x * a.scale_pre;
        v[k].y = v[k].y * inv * g.y * a.scale_pre;
        v[k].z = v[k].z * inv * g.z * a.scale_pre;
        v[k].w = v[k].w * inv * g.w * a.scale_pre;
        xr[lane + 32 * k] = v[k];
        ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
      }
      ss = warp_sum(ss);
    }
    if (a.gamma == nullptr) continue;
    const float inv = rsqrtf(ss + 1e-12f);
    const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float4 g = __ldg(g4 + lane + 32 * k);
      v[k].x = v[k].x * inv * g.x * a.scale;
      v[k].y = v[k].y * inv * g.y * a.scale;
      v[k].z = v[k].z * inv * g.z * a.scale;
      v[k].w = v[k].w * inv * g.w * a.scale;
    }
    long long orow = r;
    if (a.band_major) {
      const long long bt_count = a.rows / a.F;
      orow = (r % a.F) * bt_count + r / a.F;
    }
    uint2* o = reinterpret_cast<uint2*>(reinterpret_cast<T*>(a.out16) + orow * D);
#pragma unroll
    for (int k = 0; k < V; ++k) o[lane + 32 * k] = make_uint2(pack2<T>(v[k].x, v[k].y), pack2<T>(v[k].z, v[k].w));
    if (a.wg != nullptr) {
      for (int h = 0; h < a.heads; ++h) {
        const float4* w4 = reinterpret_cast<const float4*>(s_wg + h * D);
        float d = 0.f;
#pragma unroll
        for (int k = 0; k < V; ++k) {
          const float4 w = w4[lane + 32 * k];
          d += v[k].x * w.x + v[k].y * w.y + v[k].z * w.z + v[k].w * w.w;
        }
        d = warp_sum(d);
        if (lane == h) a.gates[r * a.heads + h] = 1.0f / (1.0f + __expf(-(d + a.bg[h])));
      }
    }
  }
}

// ---------------------------------------------------------------- LayerNorm
// One warp per row (grid-stride over rows); lane l holds columns 4l + 128k, k < V.
// Mean first, then the variance of the centred values from registers (the
// reference's two-pass order, src/ops_norm.cu:160-176).
template <typename OutT, int V>
__global__ void __launch_bounds__(256) layernorm_kernel(LayerNormArgs a) {
  const int lane = threadIdx.x & 31;
  const int D = a.D;
  const float invD = 1.0f / (float)D;
  const long long warps_total = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < a.rows; r += warps_total) {
    const float4* xr = reinterpret_cast<const float4*>(a.x + r * D);
    float4 v[V];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const int c4 = lane + 32 * k;
      v[k] = c4 * 4 < D ? __ldg(xr + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
      s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
    const float mean = warp_sum(s) * invD;
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      if ((lane + 32 * k) * 4 >= D) continue;
      v[k].x -= mean;
      v[k].y -= mean;
      v[k].z -= mean;
      v[k].w -= mean;
      ss += (v[k].x * v[k].x + v[k].y * v[k].y) + (v[k].z * v[k].z + v[k].w * v[k].w);
    }
    const float inv = rsqrtf(warp_sum(ss) * invD + a.eps);
    const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
    const float4* b4 = reinterpret_cast<const float4*>(a.beta);
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const int c4 = lane + 32 * k;
      if (c4 * 4 >= D) continue;
      const float4 g = __ldg(g4 + c4), b = __ldg(b4 + c4);
      const float4 y = make_float4(v[k].x * inv * g.x + b.x, v[k].y * inv * g.y + b.y, v[k].z * inv * g.z + b.z,
                                   v[k].w * inv * g.w + b.w);
      if constexpr (std::is_same<OutT, float>::value) {
        reinterpret_cast<float4*>(a.out)[r * (D / 4) + c4] = y;
      } else {
        reinterpret_cast<uint2*>(a.out)[r * (D / 4) + c4] = make_uint2(pack2<OutT>(y.x, y.y), pack2<OutT>(y.z, y.w));
      }
    }
  }
}

template <typename OutT>
cudaError_t layernorm_dispatch(const LayerNormArgs& a, unsigned blocks, cudaStream_t s) {
  switch ((a.D + 127) / 128) {
#define MSST_LN_CASE(v) \
  case v:               \
    layernorm_kernel<OutT, v><<<blocks, 256, 0, s>>>(a); \
    break;
    MSST_LN_CASE(1)
    MSST_LN_CASE(2)
    MSST_LN_CASE(3)
    MSST_LN_CASE(4)
    MSST_LN_CASE(5)
    MSST_LN_CASE(6)
    MSST_LN_CASE(7)
    MSST_LN_CASE(8)
#undef MSST_LN_CASE
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// RMSNorm + 8 attention-gate projections with the gate weights held in registers
// (8 heads x 4V columns per lane, loaded once per persistent warp) and the eight
// partial dot products reduced by a butterfly transpose-reduce: 4 + 2 + 1
// exchanges halve the set of heads a lane keeps, 2 more finish the sum, so lane
// group h (lanes 4h..4h+3) ends with head h's full dot product (9 shuffles
// instead of 8 separate 5-shuffle reductions).  The next row's x is prefetched
// while the current one is processed.
template <typename T, int V>
__global__ void __launch_bounds__(384, 1) rmsnorm_gates8_kernel(RmsNormArgs a) {
  constexpr int H = 8;
  const int lane = threadIdx.x & 31;
  const int D = a.D;
  float4 wr[H][V];
#pragma unroll
  for (int h = 0; h < H; ++h)
#pragma unroll
    for (int k = 0; k < V; ++k) wr[h][k] = __ldg(reinterpret_cast<const float4*>(a.wg + h * D) + lane + 32 * k);
  const float bgl = __ldg(a.bg + ((lane >> 2) & 7));
  const long long warps_total = (long long)gridDim.x * (blockDim.x >> 5);
  long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  float4 nxt[V];
  if (r < a.rows) {
#pragma unroll
    for (int k = 0; k < V; ++k) nxt[k] = reinterpret_cast<const float4*>(a.x + r * D)[lane + 32 * k];
  }
  for (; r < a.rows; r += warps_total) {
    float4 v[V];
#pragma unroll
    for (int k = 0; k < V; ++k) v[k] = nxt[k];
    const long long rn = r + warps_total;
    if (rn < a.rows) {
#pragma unroll
      for (int k = 0; k < V; ++k) nxt[k] = reinterpret_cast<const float4*>(a.x + rn * D)[lane + 32 * k];
    }
    float4* xr = reinterpret_cast<float4*>(a.x + r * D);
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < V; ++k) ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
    ss = warp_sum(ss);
    if (a.gamma_pre != nullptr) {
      const float inv = rsqrtf(ss + 1e-12f) * a.scale_pre;
      const float4* g4 = reinterpret_cast<const float4*>(a.gamma_pre);
      ss = 0.f;
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const float4 g = __ldg(g4 + lane + 32 * k);
        v[k].x *= inv * g.x;
        v[k].y *= inv * g.y;
        v[k].z *= inv * g.z;
        v[k].w *= inv * g.w;
        xr[lane + 32 * k] = v[k];
        ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
      }
      ss = warp_sum(ss);
    }
    const float inv = rsqrtf(ss + 1e-12f) * a.scale;
    const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
    float part[H];
#pragma unroll
    for (int h = 0; h < H; ++h) part[h] = 0.f;
    uint2* o = reinterpret_cast<uint2*>(reinterpret_cast<T*>(a.out16) + r * D);
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float4 g = __ldg(g4 + lane + 32 * k);
      const float4 y = make_float4(v[k].x * inv * g.x, v[k].y * inv * g.y, v[k].z * inv * g.z, v[k].w * inv * g.w);
      o[lane + 32 * k] = make_uint2(pack2<T>(y.x, y.y), pack2<T>(y.z, y.w));
#pragma unroll
      for (int h = 0; h < H; ++h)
        part[h] += y.x * wr[h][k].x + y.y * wr[h][k].y + y.z * wr[h][k].z + y.w * wr[h][k].w;
    }
    // butterfly: keep heads 4*b4..+3, then 2*b3.., then b2 (b_i = bit i of the lane)
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
    float q4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float mine = b4 ? part[4 + i] : part[i], other = b4 ? part[i] : part[4 + i];
      q4[i] = mine + __shfl_xor_sync(0xffffffffu, other, 16);
    }
    float q2[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float mine = b3 ? q4[2 + i] : q4[i], other = b3 ? q4[i] : q4[2 + i];
      q2[i] = mine + __shfl_xor_sync(0xffffffffu, other, 8);
    }
    float d = (b2 ? q2[1] : q2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? q2[0] : q2[1], 4);
    d += __shfl_xor_sync(0xffffffffu, d, 2);
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    if ((lane & 3) == 0) a.gates[r * H + (lane >> 2)] = __fdividef(1.0f, 1.0f + __expf(-(d + bgl)));
  }
}

// RMSNorm + 8 gate projections at dims 384 and 512 (at 512 the gate weights do
// not fit in registers; at 384 the register form holds too few rows in flight per
// SM): the weights sit in shared memory ([8][D] fp32) and each
// warp normalises two rows at once, so every shared-memory weight load feeds two
// rows' dot products (8 KB of shared-memory reads per row instead of 16).  The
// 16 partial sums (2 rows x 8 heads) are reduced by a butterfly transpose-reduce
// (8 + 4 + 2 + 1 exchanges, then 1 to finish), leaving lane pair 2i, 2i+1 with
// value i = row * 8 + head.  The next pair of rows is prefetched.
template <typename T, int V>
__global__ void __launch_bounds__(256, 2) rmsnorm_gates8x2_kernel(RmsNormArgs a) {
  constexpr int H = 8;
  extern __shared__ float4 s_w4[];  // [H][D/4]
  const int lane = threadIdx.x & 31;
  const int D = a.D;
  for (int i = threadIdx.x; i < H * D / 4; i += blockDim.x) s_w4[i] = __ldg(reinterpret_cast<const float4*>(a.wg) + i);
  __syncthreads();
  const float bgl = __ldg(a.bg + ((lane >> 1) & 7));
  const long long warps_total = (long long)gridDim.x * (blockDim.x >> 5);
  const long long pairs = (a.rows + 1) / 2;
  long long p = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  float4 nxt[2][V];
  auto load_pair = [&](long long pp, float4 (&dst)[2][V]) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const long long r = 2 * pp + j;
#pragma unroll
      for (int k = 0; k < V; ++k)
        dst[j][k] = r < a.rows ? reinterpret_cast<const float4*>(a.x + r * D)[lane + 32 * k] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  if (p < pairs) load_pair(p, nxt);
  for (; p < pairs; p += warps_total) {
    float4 v[2][V];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int k = 0; k < V; ++k) v[j][k] = nxt[j][k];
    if (p + warps_total < pairs) load_pair(p + warps_total, nxt);
    float inv[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < V; ++k) ss += v[j][k].x * v[j][k].x + v[j][k].y * v[j][k].y + v[j][k].z * v[j][k].z + v[j][k].w * v[j][k].w;
      inv[j] = warp_sum(ss);
    }
    if (a.gamma_pre != nullptr) {
      const float4* g4 = reinterpret_cast<const float4*>(a.gamma_pre);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const long long r = 2 * p + j;
        const float s0 = rsqrtf(inv[j] + 1e-12f) * a.scale_pre;
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < V; ++k) {
          const float4 g = __ldg(g4 + lane + 32 * k);
          v[j][k].x *= s0 * g.x;
          v[j][k].y *= s0 * g.y;
          v[j][k].z *= s0 * g.z;
          v[j][k].w *= s0 * g.w;
          if (r < a.rows) reinterpret_cast<float4*>(a.x + r * D)[lane + 32 * k] = v[j][k];
          ss += v[j][k].x * v[j][k].x + v[j][k].y * v[j][k].y + v[j][k].z * v[j][k].z + v[j][k].w * v[j][k].w;
        }
        inv[j] = warp_sum(ss);
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) inv[j] = rsqrtf(inv[j] + 1e-12f) * a.scale;
    const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
    float part[2 * H];
#pragma unroll
    for (int i = 0; i < 2 * H; ++i) part[i] = 0.f;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float4 g = __ldg(g4 + lane + 32 * k);
      float4 y[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        y[j] = make_float4(v[j][k].x * inv[j] * g.x, v[j][k].y * inv[j] * g.y, v[j][k].z * inv[j] * g.z,
                           v[j][k].w * inv[j] * g.w);
        const long long r = 2 * p + j;
        if (r < a.rows)
          reinterpret_cast<uint2*>(reinterpret_cast<T*>(a.out16) + r * D)[lane + 32 * k] =
              make_uint2(pack2<T>(y[j].x, y[j].y), pack2<T>(y[j].z, y[j].w));
      }
#pragma unroll
      for (int h = 0; h < H; ++h) {
        const float4 w = s_w4[h * (D / 4) + lane + 32 * k];
#pragma unroll
        for (int j = 0; j < 2; ++j) part[j * H + h] += y[j].x * w.x + y[j].y * w.y + y[j].z * w.z + y[j].w * w.w;
      }
    }
    // butterfly over 16 values: lane bit 4 picks the upper/lower 8, bit 3 the
    // upper/lower 4 of those, and so on down to bit 1; bit 0 finishes the sum
    float q8[8];
    {
      const bool b = lane & 16;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        q8[i] = (b ? part[8 + i] : part[i]) + __shfl_xor_sync(0xffffffffu, b ? part[i] : part[8 + i], 16);
    }
    float q4[4];
    {
      const bool b = lane & 8;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        q4[i] = (b ? q8[4 + i] : q8[i]) + __shfl_xor_sync(0xffffffffu, b ? q8[i] : q8[4 + i], 8);
    }
    float q2[2];
    {
      const bool b = lane & 4;
#pragma unroll
      for (int i = 0; i < 2; ++i)
        q2[i] = (b ? q4[2 + i] : q4[i]) + __shfl_xor_sync(0xffffffffu, b ? q4[i] : q4[2 + i], 4);
    }
    const bool b1 = lane & 2;
    float d = (b1 ? q2[1] : q2[0]) + __shfl_xor_sync(0xffffffffu, b1 ? q2[0] : q2[1], 2);
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    // value index i = 8*b4 + 4*b3 + 2*b2 + b1 = lane >> 1: row i >> 3, head i & 7
    const long long r = 2 * p + (lane >> 4);
    if ((lane & 1) == 0 && r < a.rows)
      a.gates[r * H + ((lane >> 1) & 7)] = __fdividef(1.0f, 1.0f + __expf(-(d + bgl)));
  }
}

template <typename T>
cudaError_t rmsnorm_dispatch(const RmsNormArgs& a, cudaStream_t s) {
  const int V = a.D / 128;
  const size_t smem = a.wg ? (size_t)a.heads * a.D * sizeof(float) : 0;
  const long long warps = a.rows;
  long long blocks = (warps + 7) / 8;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  if (blocks < 1) return cudaSuccess;
  const double rd = (double)a.rows * a.D;
  LaunchScope scope("rmsnorm", 0.0,
                    rd * 4.0 + (a.gamma_pre ? rd * 4.0 : 0.0) + (a.gamma ? rd * sizeof(T) : 0.0) +
                        (a.wg ? (double)a.rows * a.heads * 4.0 : 0.0),
                    s);
  if (a.wg != nullptr && a.heads == 8 && a.gamma != nullptr && !a.band_major && V <= 2) {
    // one block of 12 warps per SM (the gate weights take 32 * V registers per lane)
    long long gb = (a.rows + 11) / 12;
    if (gb > 148) gb = 148;
    if (V == 1)
      rmsnorm_gates8_kernel<T, 1><<<(unsigned)gb, 384, 0, s>>>(a);
    else
      rmsnorm_gates8_kernel<T, 2><<<(unsigned)gb, 384, 0, s>>>(a);
    return cudaGetLastError();
  }
  if (a.wg != nullptr && a.heads == 8 && a.gamma != nullptr && !a.band_major && (V == 3 || V == 4)) {
    // two persistent blocks of 8 warps per SM, each warp two rows at a time (four
    // rows in flight per warp with the prefetch: dim 384 went from 79 % to 87 % of
    // HBM against the register-weight kernel's one block of 12 warps)
    long long gb = ((a.rows + 1) / 2 + 7) / 8;
    if (gb > 2 * 148) gb = 2 * 148;
    if (V == 3)
      rmsnorm_gates8x2_kernel<T, 3><<<(unsigned)gb, 256, smem, s>>>(a);
    else
      rmsnorm_gates8x2_kernel<T, 4><<<(unsigned)gb, 256, smem, s>>>(a);
    return cudaGetLastError();
  }
  switch (V) {
#define MSST_RMS_CASE(v)                                                                               \
  case v:                                                                                               \
    if (smem > 48 * 1024)                                                                               \
      cudaFuncSetAttribute(rmsnorm_kernel<T, v>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    rmsnorm_kernel<T, v><<<(unsigned)blocks, 256, smem, s>>>(a);                                        \
    break;
    MSST_RMS_CASE(1)
    MSST_RMS_CASE(2)
    MSST_RMS_CASE(3)
    MSST_RMS_CASE(4)
    MSST_RMS_CASE(5)
    MSST_RMS_CASE(6)
    MSST_RMS_CASE(8)
#undef MSST_RMS_CASE
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------------ band input
// One block per (chunk b, frame t).  The frame's STFT values of every channel are
// staged bin-major, [bin][channel][re, im], by coalesced loads: in that order a band
// whose bins form an ascending run (every MelBandRoformer and BS-Roformer table)
// is one contiguous span of the staged row, already in the reference's
// (bin, channel, re/im) folding, so each warp normalises a band with float2
// reads and packed 16-bit stores.  Other tables take an indexed path.
template <typename T>
__global__ void __launch_bounds__(256) band_input_kernel(BandInArgs a) {
  extern __shared__ float s_row[];  // [nbins][C][2]
  const int bt = blockIdx.x;
  const int b = bt / a.T, t = bt - b * a.T;
  const int C = a.C;
  if (C <= 2 && a.nbins <= 5 * 256 && blockDim.x == 256) {
    // up to stereo x 1280 bins: every load of the frame issued before the first use
    float2 z[2][5];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const float2* src = a.spec + ((long long)(b * C + min(c, C - 1)) * a.T + t) * a.nbins;
#pragma unroll
      for (int i = 0; i < 5; ++i) {
        const int f = threadIdx.x + 256 * i;
        z[c][i] = (c < C && f < a.nbins) ? __ldg(src + f) : make_float2(0.f, 0.f);
      }
    }
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int i = 0; i < 5; ++i) {
        const int f = threadIdx.x + 256 * i;
        if (c < C && f < a.nbins)
          *reinterpret_cast<float2*>(s_row + 2 * (f * C + c)) =
              make_float2(z[c][i].x * a.spec_scale, z[c][i].y * a.spec_scale);
      }
  } else {
    for (int c = 0; c < C; ++c) {
      const float2* src = a.spec + ((long long)(b * C + c) * a.T + t) * a.nbins;
#pragma unroll 4
      for (int f = threadIdx.x; f < a.nbins; f += blockDim.x) {
        float2 z = __ldg(src + f);
        z.x *= a.spec_scale;
        z.y *= a.spec_scale;
        *reinterpret_cast<float2*>(s_row + 2 * (f * C + c)) = z;
      }
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  T* orow = reinterpret_cast<T*>(a.out) + (long long)bt * a.ld;
  for (int band = warp; band < a.num_bands; band += nwarps) {
    const int nf = __ldg(a.nfreq + band);
    const int dims = 2 * C * nf;
    const int* bins = a.bin_list + __ldg(a.bin_start + band);
    int first;
    if (a.run_first) {
      first = __ldg(a.run_first + band);
    } else {
      first = __ldg(bins);
      bool run = true;
      for (int q = lane; q < nf; q += 32) run = run && __ldg(bins + q) == first + q;
      if (!__all_sync(0xffffffffu, run)) first = -1;
    }
    const float* g = a.gamma + __ldg(a.gcol + band);
    T* o = orow + __ldg(a.kcol + band);
    const int kp = __ldg(a.kpad + band);
    if (first >= 0 && C == 2 && (reinterpret_cast<uintptr_t>(g) & 15) == 0) {
      // stereo: 4 values per bin, so the band's span and gamma are float4-aligned
      const float4* v4 = reinterpret_cast<const float4*>(s_row + 4 * first);
      const float4* g4 = reinterpret_cast<const float4*>(g);
      float ss = 0.f;
      for (int i = lane; 4 * i < dims; i += 32) {
        const float4 v = v4[i];
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
      }
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss + 1e-12f);
      const float scale = sqrtf((float)dims);
      for (int i = lane; 4 * i < kp; i += 32) {
        uint2 pk = make_uint2(0u, 0u);
        if (4 * i < dims) {
          const float4 v = v4[i], gg = __ldg(g4 + i);
          pk = make_uint2(pack2<T>(v.x * inv * gg.x * scale, v.y * inv * gg.y * scale),
                          pack2<T>(v.z * inv * gg.z * scale, v.w * inv * gg.w * scale));
        }
        reinterpret_cast<uint2*>(o)[i] = pk;
      }
    } else if (first >= 0) {
      const float2* v2 = reinterpret_cast<const float2*>(s_row + 2 * C * first);
      float ss = 0.f;
      for (int i = lane; 2 * i < dims; i += 32) {
        const float2 v = v2[i];
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, ss));
      }
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss + 1e-12f);
      const float scale = sqrtf((float)dims);
      for (int i = lane; 2 * i < kp; i += 32) {
        float2 y = make_float2(0.f, 0.f);
        if (2 * i < dims) {
          const float2 v = v2[i];
          const float2 gg = __ldg(reinterpret_cast<const float2*>(g) + i);
          y = make_float2(v.x * inv * gg.x * scale, v.y * inv * gg.y * scale);
        }
        reinterpret_cast<uint32_t*>(o)[i] = pack2<T>(y.x, y.y);
      }
    } else {
      auto load = [&](int j) -> float {
        const int per_bin = 2 * C;
        const int fl = j / per_bin, rem = j - fl * per_bin;
        return s_row[2 * (__ldg(bins + fl) * C + (rem >> 1)) + (rem & 1)];
      };
      float ss = 0.f;
      for (int j = lane; j < dims; j += 32) {
        const float v = load(j);
        ss += v * v;
      }
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss + 1e-12f);
      const float scale = sqrtf((float)dims);
      for (int j = 2 * lane; j < kp; j += 64) {
        const float y0 = j < dims ? load(j) * inv * __ldg(g + j) * scale : 0.f;
        const float y1 = j + 1 < dims ? load(j + 1) * inv * __ldg(g + j + 1) * scale : 0.f;
        *reinterpret_cast<uint32_t*>(o + j) = pack2<T>(y0, y1);
      }
    }
  }
}

// ------------------------------------------------------------------ mask apply
// One block per (chunk b, stem, frame t): the frame's mask row is staged in shared
// memory by coalesced loads, then threads walk the bins (coalesced STFT reads and
// output writes), summing each bin's band contributions from shared memory, in
// table order; with bin_pack a bin's two contributions and count come in one load.
__global__ void __launch_bounds__(256) mask_apply_kernel(MaskApplyArgs a) {
  extern __shared__ float s_mask[];  // [mask_ld]
  const int t = blockIdx.x % a.T;
  const int rest = blockIdx.x / a.T;
  const int st = rest % a.S, b = rest / a.S;
  const float* mrow = a.mask + st * a.mask_stem_stride + ((long long)b * a.T + t) * a.mask_ld;
  if (((a.mask_ld | (int)a.mask_stem_stride) & 3) == 0 && (reinterpret_cast<uintptr_t>(a.mask) & 15) == 0) {
    const float4* m4 = reinterpret_cast<const float4*>(mrow);
    float4* s4 = reinterpret_cast<float4*>(s_mask);
#pragma unroll 4
    for (int i = threadIdx.x; i < (a.mask_ld >> 2); i += blockDim.x) s4[i] = __ldg(m4 + i);
  } else {
    for (int i = threadIdx.x; i < a.mask_ld; i += blockDim.x) s_mask[i] = __ldg(mrow + i);
  }
  __syncthreads();
  for (int f = threadIdx.x; f < a.nbins; f += blockDim.x) {
    int4 pk = make_int4(-2, -1, 0, 0);
    if (a.bin_pack) pk = __ldg(a.bin_pack + f);
    int k0 = 0, k1 = 0;
    float den;
    if (pk.x == -2) {
      k0 = __ldg(a.contrib_off + f);
      k1 = __ldg(a.contrib_off + f + 1);
      den = __ldg(a.denom + f);
    } else {
      den = __int_as_float(pk.w);
    }
    for (int c = 0; c < a.C; ++c) {
      float2 zz = __ldg(a.spec + ((long long)(b * a.C + c) * a.T + t) * a.nbins + f);
      float mr = 0.f, mi = 0.f;
      if (pk.x == -2) {
        for (int k = k0; k < k1; ++k) {
          const int col = __ldg(a.contrib_col + k) + 2 * c;
          mr += s_mask[col];
          mi += s_mask[col + 1];
        }
      } else {
        if (pk.x >= 0) {
          mr += s_mask[pk.x + 2 * c];
          mi += s_mask[pk.x + 2 * c + 1];
        }
        if (pk.y >= 0) {
          mr += s_mask[pk.y + 2 * c];
          mi += s_mask[pk.y + 2 * c + 1];
        }
      }
      mr = mr / den;
      mi = mi / den;
      zz.x *= a.spec_scale;
      zz.y *= a.spec_scale;
      float2 o = make_float2((zz.x * mr - zz.y * mi) * a.out_scale, (zz.x * mi + zz.y * mr) * a.out_scale);
      if (a.zero_dc && f == 0) o = make_float2(0.f, 0.f);
      a.out[((((long long)b * a.S + st) * a.C + c) * a.T + t) * a.nbins + f] = o;
    }
  }
}

// ------------------------------------------------------------------ STFT / iSTFT
// One block per frame (bc, t); thread i handles samples i + 256u (every warp access
// is 32 consecutive floats); the reflect padding only at the track's two ends.
__global__ void __launch_bounds__(256)
    stft_frames_kernel(const float* __restrict__ audio, long long L, int T, int n_fft, int hop,
                       const float* __restrict__ win, float* __restrict__ frames) {
  const long long row = blockIdx.x;  // bc * T + t
  const int t = (int)(row % T);
  const float* src = audio + (row / T) * L;
  float* dst = frames + row * n_fft;
  const long long base = (long long)t * hop - n_fft / 2;
  if (base >= 0 && base + n_fft <= L) {
    const float* s0 = src + base;
#pragma unroll 8
    for (int n = threadIdx.x; n < n_fft; n += blockDim.x) dst[n] = __ldg(s0 + n) * __ldg(win + n);
  } else {
    for (int n = threadIdx.x; n < n_fft; n += blockDim.x) dst[n] = __ldg(src + reflect_idx(base + n, L)) * __ldg(win + n);
  }
}

// One block per (row, 1024 output samples); thread t handles samples t + 256u.  A
// sample gathers at most kMaxF = ceil(n_fft / hop) frames; their loads are issued
// together.
template <int kMaxF>
__global__ void __launch_bounds__(256)
    istft_ola_kernel(const float* __restrict__ frames, int T, int n_fft, int hop, const float* __restrict__ win,
                     const float* __restrict__ wsum, float* __restrict__ out, int Lout, int ref_compat) {
  const int Lrec = (T - 1) * hop;  // reconstructed samples; the rest of a row is zero
  const int full = Lrec + n_fft;   // untrimmed reconstruction per row
  const int pad = n_fft / 2;
  const float inv_n = 1.0f / (float)n_fft;
  const int row0 = blockIdx.y;
#pragma unroll 1
  for (int u = 0; u < 4; ++u) {
    const int j = blockIdx.x * 1024 + u * 256 + threadIdx.x;
    if (j >= Lout) break;
    float* o = out + (long long)row0 * Lout + j;
    if (j >= Lrec) {
      *o = 0.f;
      continue;
    }
    long long row = row0;
    int p = j + pad;
    if (ref_compat) {
      const long long flat = pad + (long long)row0 * Lrec + j;
      row = flat / full;
      p = (int)(flat - row * full);
    }
    const int t_lo = p >= n_fft ? (p - n_fft) / hop + 1 : 0;
    const int t_hi = min(T - 1, p / hop);
    const float* fr = frames + row * T * (long long)n_fft + (long long)t_lo * n_fft + (p - t_lo * hop);
    float v[kMaxF], w[kMaxF];
#pragma unroll
    for (int i = 0; i < kMaxF; ++i) {
      const bool on = t_lo + i <= t_hi;
      const int n = p - (t_lo + i) * hop;
      v[i] = on ? __ldg(fr + i * (n_fft - hop)) : 0.f;
      w[i] = on ? __ldg(win + n) : 0.f;
    }
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxF; ++i)
      if (t_lo + i <= t_hi) acc += (v[i] * inv_n) * w[i];
    const float ws = __ldg(wsum + p);
    *o = ws > 1e-8f ? acc / ws : acc;
  }
}

// ------------------------------------------------------------------ chunking
// The stitch maps a block to 1024 consecutive samples of one row; thread t handles
// samples t, t + 256, t + 512 and t + 768, so every warp access is 32 consecutive
// floats.  Sample positions fit in 32 bits (the launchers check).
__device__ __forceinline__ int reflect32(int i, int n) {
  if (i < 0)
    i = -i;
  else if (i >= n)
    i = 2 * (n - 1) - i;
  return i < 0 ? 0 : (i >= n ? n - 1 : i);
}

__device__ __forceinline__ float padded_track(const ChunkArgs& a, int c, int p) {
  // value of the reflect-padded track at channel c, padded index p (0 <= p < total)
  const int src = a.border ? reflect32(p - (int)a.border, (int)a.L) : p;
  return __ldg(a.track + (long long)c * a.L + src);
}

// Sample j of chunk k, channel c (j < chunk): the padded track, or for the final
// short chunk its reflect / zero padding (src/inference_app.cpp:144-150).
__device__ __forceinline__ float chunk_sample(const ChunkArgs& a, int k, int c, int j) {
  const int start = k * a.step;
  const int n = min(start + a.chunk, (int)a.total) - start;
  if (n >= a.chunk) return padded_track(a, c, start + j);
  const bool reflect = n > a.chunk / 2;
  int sj = j < n ? j : 2 * (n - 1) - j;
  sj = sj < 0 ? 0 : (sj >= n ? n - 1 : sj);
  if (!reflect && j >= n) return 0.f;
  if (a.ref_compat) {
    const long long flat = (long long)start + (long long)c * n + sj;  // contiguous view of a strided slice
    return padded_track(a, (int)(flat / a.total), (int)(flat % a.total));
  }
  return padded_track(a, c, start + sj);
}

// Frames of chunk first + (row / (C*T)) * stride, channel (row / T) % C, frame row % T
// (torch.stft center=True reflect padding inside the chunk), read straight from the
// track; interior frames of interior chunks are plain copies of track samples.
__global__ void __launch_bounds__(256)
    stft_frames_chunk_kernel(ChunkArgs a, int first, int stride, int T, int n_fft, int hop,
                             const float* __restrict__ win, float* __restrict__ frames) {
  const int row = blockIdx.x;  // (kk * C + c) * T + t
  const int t = row % T;
  const int c = (row / T) % a.C;
  const int k = first + (row / (T * a.C)) * stride;
  float* dst = frames + (long long)row * n_fft;
  const int base = t * hop - n_fft / 2;  // chunk sample of frame sample 0
  const int start = k * a.step;
  const bool whole = start + a.chunk <= (int)a.total;
  const int src0 = start + base - (int)a.border;
  if (whole && base >= 0 && base + n_fft <= a.chunk && src0 >= 0 && src0 + n_fft <= (int)a.L) {
    const float* s0 = a.track + (long long)c * a.L + src0;
    // (a 16-byte-aligned track keeps the aligned-down first load inside it)
    if ((n_fft & 3) == 0 &&
        ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(win) |
          reinterpret_cast<uintptr_t>(a.track)) & 15) == 0) {
      // four samples per thread: the source run starts m floats past a 16-byte boundary,
      // so each group is taken from two aligned float4 loads of the track (the second
      // only where m > 0 and it stays inside the frame's own samples)
      const int m = (int)((reinterpret_cast<uintptr_t>(s0) >> 2) & 3);
      const float4* a4 = reinterpret_cast<const float4*>(s0 - m);
      const float4* w4 = reinterpret_cast<const float4*>(win);
      float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll 2
      for (int g = threadIdx.x; 4 * g < n_fft; g += blockDim.x) {
        const float4 w = __ldg(w4 + g);
        float4 x;
        if (m == 0) {
          x = __ldg(a4 + g);
        } else if (4 * g + 7 - m < n_fft) {
          const float4 lo = __ldg(a4 + g), hi = __ldg(a4 + g + 1);
          x = m == 1 ? make_float4(lo.y, lo.z, lo.w, hi.x)
                     : (m == 2 ? make_float4(lo.z, lo.w, hi.x, hi.y) : make_float4(lo.w, hi.x, hi.y, hi.z));
        } else {
          x = make_float4(__ldg(s0 + 4 * g), __ldg(s0 + 4 * g + 1), __ldg(s0 + 4 * g + 2), __ldg(s0 + 4 * g + 3));
        }
        d4[g] = make_float4(x.x * w.x, x.y * w.y, x.z * w.z, x.w * w.w);
      }
    } else {
#pragma unroll 8
      for (int n = threadIdx.x; n < n_fft; n += blockDim.x) dst[n] = __ldg(s0 + n) * __ldg(win + n);
    }
  } else {
    for (int n = threadIdx.x; n < n_fft; n += blockDim.x) {
      int i = base + n;
      i = i < 0 ? -i : (i >= a.chunk ? 2 * (a.chunk - 1) - i : i);
      i = i < 0 ? 0 : (i >= a.chunk ? a.chunk - 1 : i);
      dst[n] = chunk_sample(a, k, c, i) * __ldg(win + n);
    }
  }
}

__device__ __forceinline__ float fade_weight(int j, int chunk, bool first_chunk, bool last_chunk) {
  // src/inference_app.cpp:192-204,267-276
  const int fs = chunk / 10;
  if (fs <= 0) return 1.f;
  if (j < fs) {
    if (first_chunk) return 1.f;
    if (fs == 1) return 0.f;
    return (float)j / (float)(fs - 1);
  }
  if (j >= chunk - fs) {
    if (last_chunk) return 1.f;
    if (fs == 1) return 0.f;
    return 1.0f - (float)(j - (chunk - fs)) / (float)(fs - 1);
  }
  return 1.f;
}

__global__ void __launch_bounds__(256) stitch_kernel(StitchArgs a) {
  const int r = blockIdx.y;
  const int total = (int)a.total, border = (int)a.border;
  const long long per_slot = (long long)a.rows * a.chunk;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const long long p = a.begin + (long long)blockIdx.x * 1024 + u * 256 + threadIdx.x;
    if (p >= a.end) break;
    const int q = (int)p + border;
    const int k_hi = min(a.num_chunks - 1, q / a.step);
    const int k_lo = q >= a.chunk ? (q - a.chunk) / a.step + 1 : 0;
    float acc = 0.f, wsum = 0.f;
#pragma unroll 2
    for (int k = k_lo; k <= k_hi; ++k) {
      const int start = k * a.step;
      const int j = q - start;
      const float w = fade_weight(j, a.chunk, k == 0, start + a.chunk >= total);
      const long long slot = (long long)(k % a.slot_ranks) * a.slot_cap + k / a.slot_ranks;
      acc += __ldg(a.y + slot * per_slot + (long long)r * a.chunk + j) * w;
      wsum += w;
    }
    a.out[(long long)r * a.L + p] = wsum > 1e-8f ? acc / wsum : acc;
  }
}

// Four consecutive output samples per thread (float4 loads and stores).  Taken when
// the chunk length, step, border, row length and the range start are multiples of 4:
// the chunk boundaries then fall between groups, so the group's four samples share
// one chunk range and every chunk slice is a 16-byte-aligned float4.  Same
// arithmetic, in the same order, per sample as stitch_kernel.
__global__ void __launch_bounds__(256) stitch4_kernel(StitchArgs a) {
  const int r = blockIdx.y;
  const int total = (int)a.total, border = (int)a.border;
  const long long per_slot = (long long)a.rows * a.chunk;
  const long long p = a.begin + 4 * ((long long)blockIdx.x * 256 + threadIdx.x);
  if (p >= a.end) return;
  const int q = (int)p + border;
  const int k_hi = min(a.num_chunks - 1, q / a.step);
  const int k_lo = q >= a.chunk ? (q - a.chunk) / a.step + 1 : 0;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f), wsum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 2
  for (int k = k_lo; k <= k_hi; ++k) {
    const int start = k * a.step;
    const int j = q - start;
    const bool first = k == 0, last = start + a.chunk >= total;
    const float4 w = make_float4(fade_weight(j, a.chunk, first, last), fade_weight(j + 1, a.chunk, first, last),
                                 fade_weight(j + 2, a.chunk, first, last), fade_weight(j + 3, a.chunk, first, last));
    const long long slot = (long long)(k % a.slot_ranks) * a.slot_cap + k / a.slot_ranks;
    const float4 y = __ldg(reinterpret_cast<const float4*>(a.y + slot * per_slot + (long long)r * a.chunk + j));
    acc.x += y.x * w.x;
    acc.y += y.y * w.y;
    acc.z += y.z * w.z;
    acc.w += y.w * w.w;
    wsum.x += w.x;
    wsum.y += w.y;
    wsum.z += w.z;
    wsum.w += w.w;
  }
  float4 o;
  o.x = wsum.x > 1e-8f ? acc.x / wsum.x : acc.x;
  o.y = wsum.y > 1e-8f ? acc.y / wsum.y : acc.y;
  o.z = wsum.z > 1e-8f ? acc.z / wsum.z : acc.z;
  o.w = wsum.w > 1e-8f ? acc.w / wsum.w : acc.w;
  if (p + 4 <= a.end) {
    *reinterpret_cast<float4*>(a.out + (long long)r * a.L + p) = o;
  } else {
    const float ov[4] = {o.x, o.y, o.z, o.w};
    for (int i = 0; i < 4 && p + i < a.end; ++i) a.out[(long long)r * a.L + p + i] = ov[i];
  }
}

__global__ void __launch_bounds__(256) skip_add_kernel(float4* x, const float4* __restrict__ skips, int count,
                                                       long long n4) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 v = x[i];
    for (int j = 0; j < count; ++j) {
      const float4 s = __ldg(skips + (long long)j * n4 + i);
      v.x += s.x;
      v.y += s.y;
      v.z += s.z;
      v.w += s.w;
    }
    x[i] = v;
  }
}

inline unsigned grid_for(long long n) {
  long long b = (n + 255) / 256;
  if (b > 148LL * 32) b = 148LL * 32;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

cudaError_t launch_rmsnorm(const RmsNormArgs& a, int bf16, cudaStream_t s) {
  if (a.D % 128 != 0 || a.D > 1024 || (a.band_major && a.F <= 0) || (a.wg && a.heads > 32))
    return cudaErrorInvalidValue;
  return bf16 ? rmsnorm_dispatch<__nv_bfloat16>(a, s) : rmsnorm_dispatch<__half>(a, s);
}

cudaError_t launch_layernorm(const LayerNormArgs& a, cudaStream_t s) {
  if (a.D < 4 || a.D % 4 != 0 || a.D > 1024 || a.out_kind < 0 || a.out_kind > 2) return cudaErrorInvalidValue;
  if (a.rows <= 0) return cudaSuccess;
  long long blocks = (a.rows + 7) / 8;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  const double out_bytes = a.out_kind == 0 ? 4.0 : 2.0;
  LaunchScope scope("layernorm", 0.0, (double)a.rows * a.D * (4.0 + out_bytes), s);
  if (a.out_kind == 0) return layernorm_dispatch<float>(a, (unsigned)blocks, s);
  if (a.out_kind == 1) return layernorm_dispatch<__half>(a, (unsigned)blocks, s);
  return layernorm_dispatch<__nv_bfloat16>(a, (unsigned)blocks, s);
}

cudaError_t launch_band_input(const BandInArgs& a, int bf16, cudaStream_t s) {
  const long long rows = (long long)a.Bc * a.T;
  if (rows < 1) return cudaSuccess;
  if (rows > 0x7fffffffLL || (a.ld & 1) || a.C < 1) return cudaErrorInvalidValue;
  const size_t smem = sizeof(float2) * (size_t)a.C * a.nbins;
  // the STFT read once, the packed A operand written once
  LaunchScope scope("band_input", 0.0, (double)a.Bc * a.C * a.T * a.nbins * 8.0 + (double)rows * a.ld * 2.0, s);
  if (bf16) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(band_input_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    band_input_kernel<__nv_bfloat16><<<(unsigned)rows, 256, smem, s>>>(a);
  } else {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(band_input_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    band_input_kernel<__half><<<(unsigned)rows, 256, smem, s>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launch_mask_apply(const MaskApplyArgs& a, cudaStream_t s) {
  const long long blocks = (long long)a.Bc * a.S * a.T;
  if (blocks < 1) return cudaSuccess;
  const size_t smem = sizeof(float) * (size_t)a.mask_ld;
  if (blocks > 0x7fffffffLL || smem > 227 * 1024) return cudaErrorInvalidValue;
  const double tb = (double)a.Bc * a.T * a.nbins;
  LaunchScope scope("mask_apply", 0.0,
                    tb * a.C * 8.0 + (double)a.S * a.Bc * a.T * a.mask_ld * 4.0 + tb * a.S * a.C * 8.0, s);
  if (smem > 48 * 1024) cudaFuncSetAttribute(mask_apply_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  mask_apply_kernel<<<(unsigned)blocks, 256, smem, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_stft_frames(const float* audio, long long L, int BC, int T, int n_fft, int hop, const float* win,
                               float* frames, cudaStream_t s) {
  if (n_fft % 4 != 0 || (long long)BC * T > 0x7fffffffLL) return cudaErrorInvalidValue;
  LaunchScope scope("stft_frames", 0.0, (double)BC * L * 4.0 + (double)BC * T * n_fft * 4.0, s);
  stft_frames_kernel<<<(unsigned)((long long)BC * T), 256, 0, s>>>(audio, L, T, n_fft, hop, win, frames);
  return cudaGetLastError();
}

cudaError_t launch_istft_ola(const float* frames, int BSC, int T, int n_fft, int hop, const float* win,
                             const float* wsum, float* out, long long out_len, int ref_compat, cudaStream_t s) {
  const int maxf = (n_fft + hop - 1) / hop;
  if (out_len < (long long)(T - 1) * hop || maxf > 8) return cudaErrorInvalidValue;
  if (out_len + n_fft >= (1LL << 31) || BSC > 65535) return cudaErrorInvalidValue;
  if (out_len == (long long)(T - 1) * hop) ref_compat = 0;  // nothing padded: the rows are plain
  LaunchScope scope("istft_ola", 0.0, (double)BSC * T * n_fft * 4.0 + (double)BSC * (double)out_len * 4.0, s);
  const dim3 grid((unsigned)((out_len + 1023) / 1024), (unsigned)BSC);
  switch (maxf) {
#define MSST_ISTFT_CASE(f)                                                                             \
  case f:                                                                                              \
    istft_ola_kernel<f><<<grid, 256, 0, s>>>(frames, T, n_fft, hop, win, wsum, out, (int)out_len, ref_compat); \
    break;
    MSST_ISTFT_CASE(1)
    MSST_ISTFT_CASE(2)
    MSST_ISTFT_CASE(3)
    MSST_ISTFT_CASE(4)
    MSST_ISTFT_CASE(5)
    MSST_ISTFT_CASE(6)
    MSST_ISTFT_CASE(7)
    MSST_ISTFT_CASE(8)
#undef MSST_ISTFT_CASE
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_stft_frames_chunks(const ChunkArgs& a, int first, int stride, int count, int T, int n_fft,
                                      int hop, const float* win, float* frames, cudaStream_t s) {
  if (count <= 0) return cudaSuccess;
  if (a.total + a.chunk >= (1LL << 31) || (long long)count * a.C * T > 0x7fffffffLL || stride < 1)
    return cudaErrorInvalidValue;
  // the chunk samples read once (frames overlap in L1/L2), the frames written once
  LaunchScope scope("stft_frames", 0.0,
                    (double)count * a.C * a.chunk * 4.0 + (double)count * a.C * T * n_fft * 4.0, s);
  stft_frames_chunk_kernel<<<(unsigned)(count * a.C * T), 256, 0, s>>>(a, first, stride, T, n_fft, hop, win, frames);
  return cudaGetLastError();
}

cudaError_t launch_skip_add(float* x, const float* skips, int count, long long n, cudaStream_t s) {
  if (count <= 0 || n <= 0) return cudaSuccess;
  if (n % 4 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(skips) & 15))
    return cudaErrorInvalidValue;
  LaunchScope scope("skip_add", 0.0, (double)n * 4.0 * (count + 2), s);
  skip_add_kernel<<<grid_for(n / 4), 256, 0, s>>>(reinterpret_cast<float4*>(x),
                                                  reinterpret_cast<const float4*>(skips), count, n / 4);
  return cudaGetLastError();
}

cudaError_t launch_stitch(const StitchArgs& a, cudaStream_t s) {
  if (a.end <= a.begin) return cudaSuccess;
  if (a.total + a.chunk >= (1LL << 31) || a.rows > 65535 || a.slot_ranks < 1 || a.begin < 0 || a.end > a.L)
    return cudaErrorInvalidValue;
  const long long n = a.end - a.begin;
  // every output sample written once; each chunk sample it covers read once (overlaps twice)
  LaunchScope scope("stitch", 0.0, (double)a.rows * n * 4.0 * 2.0, s);
  const bool vec = a.chunk % 4 == 0 && a.step % 4 == 0 && a.border % 4 == 0 && a.L % 4 == 0 && a.begin % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0;
  if (vec)
    stitch4_kernel<<<dim3((unsigned)((n + 1023) / 1024), (unsigned)a.rows), 256, 0, s>>>(a);
  else
    stitch_kernel<<<dim3((unsigned)((n + 1023) / 1024), (unsigned)a.rows), 256, 0, s>>>(a);
  return cudaGetLastError();
}

MSST_DEFINE_ERROR_ACCESSOR(kernels_device_error)

}  // namespace msst
