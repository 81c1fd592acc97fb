// attention.cu — tcgen05 flash attention for the Roformer's axial attention on
// sm_100a (head_dim 64, non-causal).
//
// CTA = 192 threads, persistent over work items (sequence-or-tile, head, q-tile):
//   warp 0     TMA producer: Q tile (double-buffered), K/V tiles into a 3-stage ring
//   warp 1     MMA issuer: S = Q K^T (M128 N128 K64) into one of two TMEM S buffers,
//              O_j = P_j V_j (M128 N64 K128, P from smem) into one of two TMEM O buffers
//   warps 2-5  softmax: one query row per thread; online max/sum in fp32, P written
//              as 16-bit into 128B-swizzled smem (the UMMA A operand), O_j folded into
//              a register accumulator one tile late so PV overlaps the next softmax;
//              epilogue divides by the row sum, applies the head gate, writes the
//              merged-head row.
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,320) O1 [320,384) (512 allocated).
#include "attention.cuh"
#include "common.cuh"

namespace msst {

namespace {

constexpr int kKvStages = 3;
constexpr uint32_t kTileBytes = 128 * 64 * 2;   // one 128x64 16-bit tile
constexpr uint32_t kPBytes = 128 * 128 * 2;     // P tile (two 64-column K-blocks)
constexpr size_t kAttnSmem = 1024 + 2 * kTileBytes + kKvStages * 2 * kTileBytes + 2 * kPBytes + 256;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256;

struct ItemGeom {
  int head;
  int nkv;       // KV tiles
  // mode 0
  int b, f, t0;
  // mode 1
  int r0, rows;  // first token of the packed tile, valid rows (seqs_per_tile * F)
};

__device__ __forceinline__ ItemGeom item_geom(const AttnParams& p, int item) {
  ItemGeom g;
  if (p.mode == 0) {
    const int qt = item % p.q_tiles;
    const int sh = item / p.q_tiles;
    g.head = sh % p.heads;
    const int s = sh / p.heads;
    g.b = s / p.F;
    g.f = s - g.b * p.F;
    g.t0 = qt * 128;
    g.nkv = p.q_tiles;
    g.r0 = 0;
    g.rows = 0;
  } else {
    g.head = item % p.heads;
    const int tile = item / p.heads;
    g.rows = p.seqs_per_tile * p.seq_len;
    g.r0 = tile * g.rows;
    g.nkv = 1;
    g.b = g.f = g.t0 = 0;
  }
  return g;
}

template <typename T>
__global__ void __launch_bounds__(192, 1)
    attention_kernel(const __grid_constant__ CUtensorMap qkv, const __grid_constant__ AttnParams p) {
  constexpr uint32_t kIsBf16 = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                  // 2 tiles
  uint8_t* sKV = sQ + 2 * kTileBytes;                  // stages x (K, V)
  uint8_t* sP = sKV + kKvStages * 2 * kTileBytes;      // 2 P tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kPBytes);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 2;
  uint64_t* kv_full = bars + 4;
  uint64_t* kv_empty = kv_full + kKvStages;
  uint64_t* s_full = kv_empty + kKvStages;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = 3 * p.heads * 64;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
    }
    for (int s = 0; s < kKvStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&qkv);
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int qcount = 0, kvcount = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.total_items; item += gridDim.x, ++qcount) {
        const ItemGeom g = item_geom(p, item);
        const int qb = qcount & 1;
        if (!mbar_wait(&q_empty[qb], ((qcount >> 1) & 1) ^ 1, kErrTimeoutAttnQ, abort_flag)) break;
        mbar_arrive_expect_tx(&q_full[qb], kTileBytes);
        const int xq = g.head * 64;
        if (p.mode == 0)
          tma_load_4d(sQ + qb * kTileBytes, &qkv, &q_full[qb], xq, g.f, g.t0, g.b);
        else
          tma_load_4d(sQ + qb * kTileBytes, &qkv, &q_full[qb], xq, g.r0, 0, 0);
        for (int j = 0; j < g.nkv; ++j, ++kvcount) {
          const int st = kvcount % kKvStages;
          const uint32_t ph = (kvcount / kKvStages) & 1;
          if (!mbar_wait(&kv_empty[st], ph ^ 1, kErrTimeoutAttnKV, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * kTileBytes);
          uint8_t* dk = sKV + st * 2 * kTileBytes;
          const int xk = p.heads * 64 + g.head * 64, xv = 2 * p.heads * 64 + g.head * 64;
          if (p.mode == 0) {
            tma_load_4d(dk, &qkv, &kv_full[st], xk, g.f, j * 128, g.b);
            tma_load_4d(dk + kTileBytes, &qkv, &kv_full[st], xv, g.f, j * 128, g.b);
          } else {
            tma_load_4d(dk, &qkv, &kv_full[st], xk, g.r0, 0, 0);
            tma_load_4d(dk + kTileBytes, &qkv, &kv_full[st], xv, g.r0, 0, 0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_f16(kIsBf16, 128, 0);
      const uint32_t idesc_o = umma_idesc_f16(kIsBf16, 64, 1);
      int qcount = 0, kvcount = 0, scount = 0, pcount = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.total_items; item += gridDim.x, ++qcount) {
        const ItemGeom g = item_geom(p, item);
        const int qb = qcount & 1;
        if (!mbar_wait(&q_full[qb], (qcount >> 1) & 1, kErrTimeoutAttnQ, abort_flag)) break;
        tc_fence_after();
        const uint32_t qaddr = smem_u32(sQ + qb * kTileBytes);
        int prev_stage = -1;
        for (int j = 0; j <= g.nkv; ++j) {
          if (j < g.nkv) {
            const int st = kvcount % kKvStages;
            if (!mbar_wait(&kv_full[st], (kvcount / kKvStages) & 1, kErrTimeoutAttnKV, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t kaddr = smem_u32(sKV + st * 2 * kTileBytes);
            const uint32_t dS = tmem + kColS + (uint32_t)((scount & 1) * 128);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_f16_ss(dS, sw128_desc(qaddr + kk * 32, 16, 1024), sw128_desc(kaddr + kk * 32, 16, 1024), idesc_s,
                          kk > 0 ? 1u : 0u);
            umma_commit(&s_full[scount & 1]);
            ++scount;
            if (j == g.nkv - 1) umma_commit(&q_empty[qb]);
          }
          if (j > 0) {
            // O_{j-1} = P_{j-1} V_{j-1}
            const int pb = pcount & 1;
            if (!mbar_wait(&p_full[pb], (pcount >> 1) & 1, kErrTimeoutAttnP, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t paddr = smem_u32(sP + pb * kPBytes);
            const uint32_t vaddr = smem_u32(sKV + prev_stage * 2 * kTileBytes + kTileBytes);
            const uint32_t dO = tmem + kColO + (uint32_t)(pb * 64);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_f16_ss(dO, sw128_desc(paddr + (kk >> 2) * (kPBytes / 2) + (kk & 3) * 32, 16, 1024),
                          sw128_desc(vaddr + kk * 2048, kTileBytes, 1024), idesc_o, kk > 0 ? 1u : 0u);
            umma_commit(&o_full[pb]);
            umma_commit(&kv_empty[prev_stage]);
            ++pcount;
          }
          if (j < g.nkv) {
            prev_stage = kvcount % kKvStages;
            ++kvcount;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const float c = p.scale_log2;
    int scount = 0, pcount = 0;
    for (int item = blockIdx.x; item < p.total_items; item += gridDim.x) {
      const ItemGeom g = item_geom(p, item);
      float acc[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = 0.f;
      float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
      // band axis: this row's sequence inside the packed tile
      const int seq_lo = p.mode == 1 ? (row / p.seq_len) * p.seq_len : 0;
      const int seq_hi = p.mode == 1 ? min(seq_lo + p.seq_len, g.rows) : 0;
      bool ok = true;
      for (int j = 0; j < g.nkv; ++j) {
        if (!mbar_wait(&s_full[scount & 1], (scount >> 1) & 1, kErrTimeoutAttnS, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sAddr = tmem + lane_off + kColS + (uint32_t)((scount & 1) * 128);
        ++scount;
        int lo, hi;  // valid key columns [lo, hi) of this tile for this row
        if (p.mode == 0) {
          lo = 0;
          hi = min(128, p.seq_len - j * 128);
        } else {
          lo = seq_lo;
          hi = seq_hi;
        }
        // pass 1: row max
        float mx = -INFINITY;
#pragma unroll
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(sAddr + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int col = c0 + i;
            if (col >= lo && col < hi) mx = fmaxf(mx, __uint_as_float(r[i]));
          }
        }
        const float m_new = fmaxf(m, mx);
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        const float alpha = fast_exp2((m - m_use) * c);
        const float mc = m_use * c;
        // pass 2: probabilities -> P smem (128B swizzle, K-major), row sum
        const int pb = pcount & 1;
        uint8_t* prow = sP + pb * kPBytes + row * 128;
        float sum = 0.f;
#pragma unroll
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(sAddr + c0, r);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int col = c0 + 2 * i;
            const float s0 = (col >= lo && col < hi) ? fast_exp2(fmaf(__uint_as_float(r[2 * i]), c, -mc)) : 0.f;
            const float s1 =
                (col + 1 >= lo && col + 1 < hi) ? fast_exp2(fmaf(__uint_as_float(r[2 * i + 1]), c, -mc)) : 0.f;
            sum += s0 + s1;
            pk[i] = pack2<T>(s0, s1);
          }
          uint8_t* blk = prow + (c0 >> 6) * (kPBytes / 2);
          const int chunk0 = (c0 & 63) >> 3;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int ch = (chunk0 + u) ^ (row & 7);
            *reinterpret_cast<uint4*>(blk + ch * 16) = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&p_full[pb]);
        ++pcount;
        l = l * alpha + sum;
        if (j > 0) {
          const int ob = (pcount - 2) & 1;
          if (!mbar_wait(&o_full[ob], ((pcount - 2) >> 1) & 1, kErrTimeoutAttnO, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t oAddr = tmem + lane_off + kColO + (uint32_t)(ob * 64);
#pragma unroll
          for (int c0 = 0; c0 < 64; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(oAddr + c0, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[c0 + i] = fmaf(acc[c0 + i], alpha_prev, __uint_as_float(r[i]));
          }
        }
        alpha_prev = alpha;
        m = m_new;
      }
      if (!ok) break;
      {
        const int ob = (pcount - 1) & 1;
        if (!mbar_wait(&o_full[ob], ((pcount - 1) >> 1) & 1, kErrTimeoutAttnO, abort_flag)) break;
        tc_fence_after();
        const uint32_t oAddr = tmem + lane_off + kColO + (uint32_t)(ob * 64);
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(oAddr + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[c0 + i] = fmaf(acc[c0 + i], alpha_prev, __uint_as_float(r[i]));
        }
      }
      // epilogue: normalise, gate, merged-head store
      long long token;
      bool valid;
      if (p.mode == 0) {
        const int t = g.t0 + row;
        valid = t < p.T;
        token = ((long long)g.b * p.T + t) * p.F + g.f;
      } else {
        valid = row < g.rows && g.r0 + row < p.num_tokens;
        token = (long long)g.r0 + row;
      }
      if (valid) {
        float scale = l > 0.f ? 1.f / l : 0.f;
        if (p.gates != nullptr) scale *= __ldg(p.gates + token * p.heads + g.head);
        uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.out) + token * (p.heads * 64) + g.head * 64);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          o[u] = make_uint4(pack2<T>(acc[8 * u] * scale, acc[8 * u + 1] * scale),
                            pack2<T>(acc[8 * u + 2] * scale, acc[8 * u + 3] * scale),
                            pack2<T>(acc[8 * u + 4] * scale, acc[8 * u + 5] * scale),
                            pack2<T>(acc[8 * u + 6] * scale, acc[8 * u + 7] * scale));
        }
      }
      tc_fence_before();
    }
  }
  (void)C;

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T>
cudaError_t launch_t(const CUtensorMap& m, const AttnParams& p, int num_sms, cudaStream_t s) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kAttnSmem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const int grid = p.total_items < num_sms ? p.total_items : num_sms;
  if (grid <= 0) return cudaSuccess;
  note_launch();
  attention_kernel<T><<<grid, 192, kAttnSmem, s>>>(m, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention(const CUtensorMap& qkv_map, const AttnParams& p, int bf16, int num_sms,
                             cudaStream_t stream) {
  if (p.mode == 1 && (p.seq_len > 128 || p.seqs_per_tile < 1)) return cudaErrorInvalidValue;
  return bf16 ? launch_t<__nv_bfloat16>(qkv_map, p, num_sms, stream) : launch_t<__half>(qkv_map, p, num_sms, stream);
}

MSST_DEFINE_ERROR_ACCESSOR(attention_device_error)

}  // namespace msst
