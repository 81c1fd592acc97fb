// band_attn.cu — band-axis attention block fused with its QKV projection, for
// sm_100a.  Replaces, for the Roformer's band transformer (sequences of the
// num_bands tokens of one frame), the QKV GEMM with its RoPE epilogue and the
// attention kernel: the [tokens, 3*heads*64] QKV activation never reaches HBM.
// Reference: the band-axis apply_attention, src/model_mel_band_roformer.cu:519-591
// (to_qkv, split heads, rotary, scaled_dot_product_attention, gates, merge).
//
// A band sequence (F <= 64 tokens) sits in an aligned slot of 32 or 64 rows of a
// 128-row tile (two sequences per tile for F = 60 or 62), so every query row finds
// all of its keys inside the tile.  Persistent CTAs each take a contiguous range
// of the launch's (tile, head) steps (UnitRange: every CTA the same number, give or
// take one; a range may start or end inside a tile, whose xn the CTA then loads
// itself); per tile and head h:
//   1. QKV_h = xn . [Wq_h; Wk_h; Wv_h]^T        M128 N192 K=dim, into TMEM (two
//                                                 buffers alternate between heads)
//   2. drain (8 warps, each 32 columns of Q, K and V): QKV_h -> registers, rotary
//      on Q and K, 16-bit Q, K, V tiles into shared memory (128B swizzle, as TMA
//      would write them)
//   3. S = Q K^T                                  M128 N128 K64, into TMEM
//   4. softmax (warps 2-5, one row per thread): the row's own slot only; P (16-bit,
//      zero outside the slot) written over the first 64 columns of S in TMEM
//   5. O = P V                                    M128 N64 K128, A from TMEM, into
//                                                 the drained QKV_h buffer
//   6. output (warps 6-9, after draining the next head, while its softmax runs):
//      O / rowsum * gate -> 16-bit -> [token, h*64 ..)
// The MMA warp issues QKV_{h+1} right after S_h, so the tensor pipe computes the
// next head's projection while the softmax of this one runs.
//
// CTA = 320 threads: warp 0 TMA, warp 1 MMA issuer, warps 2-9 as above.  Every
// wait sits on the head-to-head critical path, so none takes the suspend hint.
// TMEM: QKV buffers [0, 192) and [192, 384), S [384, 512) (P over [384, 448)).
// Shared memory: xn tile (dim/64 blocks of 128x64, resident per tile), a ring of
// W stages (192 rows x 64, three 64-row TMA boxes), Q, K, V tiles, row sums.
#include "attention.cuh"
#include "common.cuh"

namespace msst {

namespace {

constexpr int kThreads = 320;
constexpr uint32_t kBlock = 128 * 64 * 2;     // 128 x 64 16-bit tile (16 KB)
constexpr uint32_t kWStage = 192 * 64 * 2;    // W_h k-block: 192 rows x 64 (24 KB)
constexpr uint32_t kColQB0 = 0, kColQB1 = 192, kColS = 384;

// shared memory layout for a model dim D (xn tile D/64 blocks) and W ring depth
__host__ __device__ constexpr int band_w_stages(int D) { return D <= 384 ? 3 : 2; }
__host__ __device__ constexpr size_t band_smem_bytes(int D) {
  return 1024 + (size_t)(D / 64) * kBlock + (size_t)band_w_stages(D) * kWStage + 3 * kBlock + 2 * 128 * 4 + 384;
}

template <typename T, int kNch>
__global__ void __launch_bounds__(kThreads, 1)
    band_attn_kernel(const __grid_constant__ CUtensorMap map_xn, const __grid_constant__ CUtensorMap map_w,
                     const __grid_constant__ BandAttnParams p) {
  constexpr uint32_t kIsBf16 = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nkb = p.D / 64;
  const int nst = band_w_stages(p.D);
  uint8_t* sX = smem;                              // nkb blocks
  uint8_t* sW = sX + nkb * kBlock;                 // nst stages
  uint8_t* sQ = sW + nst * kWStage;
  uint8_t* sK = sQ + kBlock;
  uint8_t* sV = sK + kBlock;
  float* sL = reinterpret_cast<float*>(sV + kBlock);  // [2][128] row sums, by head parity
  uint64_t* bars = reinterpret_cast<uint64_t*>(sL + 256);
  // xn per k-block, so the next tile's k-block kb loads as soon as the last head's
  // projection has read this tile's k-block kb
  uint64_t* x_full = bars + 0;      // [8]
  uint64_t* x_empty = bars + 8;     // [8]
  uint64_t* w_full = bars + 16;     // [3]
  uint64_t* w_empty = bars + 19;    // [3]
  uint64_t* qkv_full = bars + 22;   // [2]
  uint64_t* qb_free = bars + 24;    // [2]
  uint64_t* q_ready = bars + 26;
  uint64_t* smem_free = bars + 27;
  uint64_t* s_full = bars + 28;
  uint64_t* p_full = bars + 29;
  // by head parity: the output warps wait for head g while the softmax warps may
  // already have finished head g + 1, so these two alternate between two barriers
  uint64_t* o_full = bars + 30;     // [2]
  uint64_t* l_ready = bars + 32;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 34);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.heads;
  const int spt = 128 / p.slot;  // sequences per tile
  const int ntiles = (p.num_seqs + spt - 1) / spt;
  // this CTA's (tile, head) steps, in segments of one tile each; step g is the g-th
  // (tile, head) in segment order and segment s loads its tile's xn (phase s & 1)
  const UnitRange range(ntiles, H, (int)blockIdx.x, (int)gridDim.x);
  const int total_g = range.count;

  if (threadIdx.x == 0) {
    for (int kb = 0; kb < 8; ++kb) {
      mbar_init(&x_full[kb], 1);
      mbar_init(&x_empty[kb], 1);
    }
    for (int s = 0; s < 3; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&qkv_full[b], 1);
      mbar_init(&qb_free[b], 4);  // the 4 output warps
      mbar_init(&o_full[b], 1);
      mbar_init(&l_ready[b], 4);  // the 4 softmax warps
    }
    mbar_init(q_ready, 8);  // all 8 math warps drained their columns
    mbar_init(smem_free, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);   // the 4 softmax warps
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_xn);
    tma_prefetch_desc(&map_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      const uint32_t slot_bytes = (uint32_t)p.slot * 128u;
      for (int lt = 0; ok && lt < range.nseg; ++lt) {
        int t, h_begin, h_end;
        range.seg(lt, t, h_begin, h_end);
        // one box of `slot` rows per sequence (rows past the tokens are zero-filled)
        for (int kb = 0; ok && kb < nkb; ++kb) {
          if (!mbar_wait<false>(&x_empty[kb], (lt & 1) ^ 1u, kErrTimeoutSmemEmpty, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&x_full[kb], kBlock);
          for (int k = 0; k < spt; ++k)
            tma_load_2d(sX + kb * kBlock + k * slot_bytes, &map_xn, &x_full[kb], kb * 64, (t * spt + k) * p.F);
        }
        for (int h = h_begin; ok && h < h_end; ++h) {
          for (int kb = 0; kb < nkb; ++kb) {
            if (!mbar_wait<false>(&w_empty[st], ph ^ 1u, kErrTimeoutSmemEmpty, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&w_full[st], kWStage);
            uint8_t* dst = sW + st * kWStage;
            tma_load_2d(dst, &map_w, &w_full[st], kb * 64, h * 64);                      // Wq_h
            tma_load_2d(dst + 8192, &map_w, &w_full[st], kb * 64, p.inner + h * 64);     // Wk_h
            tma_load_2d(dst + 16384, &map_w, &w_full[st], kb * 64, 2 * p.inner + h * 64);  // Wv_h
            if (++st == nst) {
              st = 0;
              ph ^= 1u;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_qkv = umma_idesc_f16(kIsBf16, 192, 0);
      const uint32_t idesc_s = umma_idesc_f16(kIsBf16, 128, 0);
      const uint32_t idesc_o = umma_idesc_f16(kIsBf16, 64, 1);
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      // (segment, head) of the step issue_qkv takes next (steps go in order); heads
      // [q_h0, q_h1) of the segment
      int q_s = 0, q_t, q_h0 = 0, q_h1 = 0;
      if (range.nseg > 0) range.seg(0, q_t, q_h0, q_h1);
      int q_h = q_h0;
      auto issue_qkv = [&](int g) -> bool {
        const int b = g & 1, lt = q_s, h = q_h;
        // the segment's first step waits for its xn; its last releases it
        const bool first_in_tile = h == q_h0, last_in_tile = h == q_h1 - 1;
        if (++q_h == q_h1 && ++q_s < range.nseg) {
          range.seg(q_s, q_t, q_h0, q_h1);
          q_h = q_h0;
        }
        if (!mbar_wait<false>(&qb_free[b], ((g >> 1) & 1) ^ 1u, kErrTimeoutTmemEmpty, abort_flag)) return false;
        tc_fence_after();
        const uint32_t d = tmem + (b ? kColQB1 : kColQB0);
        for (int kb = 0; kb < nkb; ++kb) {
          if (first_in_tile && !mbar_wait<false>(&x_full[kb], lt & 1, kErrTimeoutTmaFull, abort_flag)) return false;
          if (!mbar_wait<false>(&w_full[st], ph, kErrTimeoutTmaFull, abort_flag)) return false;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sX + kb * kBlock);
          const uint32_t b0 = smem_u32(sW + st * kWStage);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_ss(d, sw128_desc(a0 + kk * 32, 16, 1024), sw128_desc(b0 + kk * 32, 16, 1024), idesc_qkv,
                        (kb | kk) != 0 ? 1u : 0u);
          umma_commit(&w_empty[st]);
          if (last_in_tile) umma_commit(&x_empty[kb]);  // the tile's xn k-block is no longer read
          if (++st == nst) {
            st = 0;
            ph ^= 1u;
          }
        }
        umma_commit(&qkv_full[b]);
        return true;
      };
      if (total_g > 0) ok = issue_qkv(0);
      for (int g = 0; ok && g < total_g; ++g) {
        // S_g once the drain has written Q, K, V
        if (!mbar_wait<false>(q_ready, g & 1, kErrTimeoutAttnQ, abort_flag)) break;
        tc_fence_after();
        {
          const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_ss(tmem + kColS, sw128_desc(qa + kk * 32, 16, 1024), sw128_desc(ka + kk * 32, 16, 1024),
                        idesc_s, kk > 0 ? 1u : 0u);
          umma_commit(s_full);
        }
        // q_h: head of step g + 1, the first of a new segment when it equals q_h0
        const bool next_same_tile = g + 1 < total_g && q_h != q_h0;
        if (next_same_tile && !(ok = issue_qkv(g + 1))) break;
        // O_g = P_g V_g into the drained QKV_g buffer
        if (!mbar_wait<false>(p_full, g & 1, kErrTimeoutAttnP, abort_flag)) break;
        tc_fence_after();
        {
          const uint32_t dO = tmem + ((g & 1) ? kColQB1 : kColQB0);
          const uint32_t va = smem_u32(sV);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16_ts(dO, tmem + kColS + (uint32_t)(kk * 8), sw128_desc(va + kk * 2048, kBlock, 1024), idesc_o,
                        kk > 0 ? 1u : 0u);
          umma_commit(&o_full[g & 1]);
          umma_commit(smem_free);
        }
        if (g + 1 < total_g && !next_same_tile && !(ok = issue_qkv(g + 1))) break;
      }
    }
  } else {
    // ------------------------------------------------------------ math warps
    const int q = warp & 3;                 // TMEM lane quarter
    const int hf = (warp - 2) >> 2;         // 0: softmax side, 1: output side
    const int r = q * 32 + lane;            // row of the tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const int slot_of_row = r / p.slot;
    const int in_slot = r - slot_of_row * p.slot;
    const int pos = min(in_slot, p.F - 1);  // rotary position (junk rows past F clamp)
    const float c = p.scale_log2;
    bool ok = true;
    // output of head g (warps 6-9): O / l * gate -> out
    // (segment, tile, head) of the step output() takes next (steps go in order)
    int o_s = 0, o_t = 0, o_h = 0, o_h1 = 0;
    if (range.nseg > 0) range.seg(0, o_t, o_h, o_h1);
    auto output = [&](int g) -> bool {
      const int t = o_t, h = o_h;
      if (++o_h == o_h1 && ++o_s < range.nseg) range.seg(o_s, o_t, o_h, o_h1);
      if (!mbar_wait<false>(&o_full[g & 1], (g >> 1) & 1, kErrTimeoutAttnO, abort_flag)) return false;
      if (!mbar_wait<false>(&l_ready[g & 1], (g >> 1) & 1, kErrTimeoutAttnO, abort_flag)) return false;
      tc_fence_after();
      const uint32_t oAddr = tmem + lane_off + ((g & 1) ? kColQB1 : kColQB0);
      uint32_t ra[32], rb[32];
      tmem_ld32(oAddr, ra);
      tmem_ld32(oAddr + 32, rb);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&qb_free[g & 1]);
      const int seq = t * spt + slot_of_row;
      if (in_slot < p.F && seq < p.num_seqs) {
        const long long token = (long long)seq * p.F + in_slot;
        const float l = sL[(g & 1) * 128 + r];
        float scale = l > 0.f ? 1.f / l : 0.f;
        if (p.gates) scale *= __ldg(p.gates + token * H + h);
        uint4* out = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.out) + token * p.out_ld + h * 64);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint32_t(&rr)[32] = u < 4 ? ra : rb;
          const int o = (u & 3) * 8;
          out[u] = make_uint4(pack2<T>(__uint_as_float(rr[o]) * scale, __uint_as_float(rr[o + 1]) * scale),
                              pack2<T>(__uint_as_float(rr[o + 2]) * scale, __uint_as_float(rr[o + 3]) * scale),
                              pack2<T>(__uint_as_float(rr[o + 4]) * scale, __uint_as_float(rr[o + 5]) * scale),
                              pack2<T>(__uint_as_float(rr[o + 6]) * scale, __uint_as_float(rr[o + 7]) * scale));
        }
      }
      return true;
    };
    // This thread's rotary factors, loaded once: its row's position never changes
    // (sequences sit at fixed slots) and warp half hf rotates pairs [16 hf, 16 hf + 16)
    // of Q and K (per-lane table loads inside the head loop hit one cache line per
    // lane and throttled the whole kernel)
    float rc[16], rs[16];
    {
      const float4* c4 = reinterpret_cast<const float4*>(p.rope_cos + (size_t)pos * 32 + 16 * hf);
      const float4* s4 = reinterpret_cast<const float4*>(p.rope_sin + (size_t)pos * 32 + 16 * hf);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 a = __ldg(c4 + u), b = __ldg(s4 + u);
        rc[4 * u] = a.x, rc[4 * u + 1] = a.y, rc[4 * u + 2] = a.z, rc[4 * u + 3] = a.w;
        rs[4 * u] = b.x, rs[4 * u + 1] = b.y, rs[4 * u + 2] = b.z, rs[4 * u + 3] = b.w;
      }
    }
    for (int g = 0; ok && g < total_g; ++g) {
      const int b = g & 1;
      // ---- drain QKV_g: columns [32 hf, 32 hf + 32) of Q, K and V, rotary on Q and K,
      // 16-bit into sQ / sK / sV
      if (!mbar_wait<false>(&qkv_full[b], (g >> 1) & 1, kErrTimeoutTmemFull, abort_flag)) break;
      tc_fence_after();
      const uint32_t qb = tmem + lane_off + (b ? kColQB1 : kColQB0);
      uint32_t v0[32], v1[32], v2[32];
      tmem_ld32(qb + hf * 32, v0);
      tmem_ld32(qb + 64 + hf * 32, v1);
      tmem_ld32(qb + 128 + hf * 32, v2);
      tmem_ld_wait();
      // Q, K, V of the previous head consumed by its S and P.V MMAs
      if (!mbar_wait<false>(smem_free, (g & 1) ^ 1u, kErrTimeoutAttnKV, abort_flag)) break;
#pragma unroll
      for (int ch = 0; ch < 3; ++ch) {
        uint32_t(&v)[32] = ch == 0 ? v0 : (ch == 1 ? v1 : v2);
        if (ch < 2) {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float x0 = __uint_as_float(v[2 * k]), x1 = __uint_as_float(v[2 * k + 1]);
            v[2 * k] = __float_as_uint(x0 * rc[k] - x1 * rs[k]);
            v[2 * k + 1] = __float_as_uint(x0 * rs[k] + x1 * rc[k]);
          }
        }
        uint8_t* rowp = (ch == 0 ? sQ : (ch == 1 ? sK : sV)) + r * 128;
        const int chunk0 = hf * 4;  // first 16-byte chunk of these 32 columns
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 w = make_uint4(pack2<T>(__uint_as_float(v[8 * u]), __uint_as_float(v[8 * u + 1])),
                                     pack2<T>(__uint_as_float(v[8 * u + 2]), __uint_as_float(v[8 * u + 3])),
                                     pack2<T>(__uint_as_float(v[8 * u + 4]), __uint_as_float(v[8 * u + 5])),
                                     pack2<T>(__uint_as_float(v[8 * u + 6]), __uint_as_float(v[8 * u + 7])));
          *reinterpret_cast<uint4*>(rowp + (((chunk0 + u) ^ (r & 7)) << 4)) = w;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
      if (hf == 0) {
        // ---- softmax of S_g over the row's own slot; P over S's first 64 columns
        if (!mbar_wait<false>(s_full, g & 1, kErrTimeoutAttnS, abort_flag)) break;
        tc_fence_after();
        const uint32_t sAddr = tmem + lane_off + kColS;
        const int c_lo = (slot_of_row * p.slot) >> 5;  // first chunk of the row's slot (kNch chunks)
        float mx = -INFINITY, l = 0.f;
        uint32_t pk[kNch][16];
        // all of the slot's chunks are read before P (which overlays S) is written
        uint32_t sv[kNch][32];
#pragma unroll
        for (int k = 0; k < kNch; ++k) tmem_ld32(sAddr + (c_lo + k) * 32, sv[k]);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < kNch; ++k)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (k * 32 + i < p.F) mx = fmaxf(mx, __uint_as_float(sv[k][i]));
        const float mc = mx * c;
#pragma unroll
        for (int k = 0; k < kNch; ++k) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int col = k * 32 + 2 * i;
            const float e0 = col < p.F ? fast_exp2(__uint_as_float(sv[k][2 * i]) * c - mc) : 0.f;
            const float e1 = col + 1 < p.F ? fast_exp2(__uint_as_float(sv[k][2 * i + 1]) * c - mc) : 0.f;
            l += e0 + e1;
            pk[k][i] = pack2<T>(e0, e1);
          }
        }
        // P chunk ch covers keys [32 ch, 32 ch + 32): the slot's chunks carry values, the
        // rest zeros (c_lo is warp-uniform: a warp's 32 rows lie in one slot)
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          bool put = false;
#pragma unroll
          for (int k = 0; k < kNch; ++k) {
            if (ch == c_lo + k) {
              tmem_st16(sAddr + ch * 16, pk[k]);
              put = true;
            }
          }
          if (!put) {
            uint32_t z[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) z[i] = 0u;
            tmem_st16(sAddr + ch * 16, z);
          }
        }
        tmem_st_wait();
        sL[(g & 1) * 128 + r] = l;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(p_full);
          mbar_arrive(&l_ready[g & 1]);
        }
      } else {
        // ---- output of the previous head while this head's softmax runs
        if (g > 0 && !(ok = output(g - 1))) break;
      }
    }
    if (ok && hf == 1 && total_g > 0) output(total_g - 1);
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <typename T, int kNch>
cudaError_t launch_band_t(const CUtensorMap& mx, const CUtensorMap& mw, const BandAttnParams& p, int num_sms,
                          cudaStream_t s) {
  static std::atomic<unsigned long long> configured{0};
  const size_t smem = band_smem_bytes(p.D);
  cudaError_t e = ensure_smem_limit(band_attn_kernel<T, kNch>, (int)band_smem_bytes(512), configured);
  if (e != cudaSuccess) return e;
  const int spt = 128 / p.slot;
  const int ntiles = (p.num_seqs + spt - 1) / spt;
  const long long units = (long long)ntiles * p.heads;  // (tile, head) steps, split evenly over the CTAs
  const int grid = units < num_sms ? (int)units : num_sms;
  if (grid <= 0) return cudaSuccess;
  // algorithmic cost: the QKV projection of every token and the attention of every
  // query row against its sequence's keys; xn and W read once, the output written once
  const double tokens = (double)p.num_seqs * p.F;
  const double flop = 2.0 * tokens * p.D * 3.0 * p.inner + 4.0 * tokens * p.heads * p.F * 64.0;
  const double bytes = tokens * p.D * sizeof(T) + 3.0 * p.inner * p.D * sizeof(T) + tokens * p.inner * sizeof(T) +
                       (p.gates ? 4.0 * tokens * p.heads : 0.0);
  LaunchScope scope("band_attention_fused", flop, bytes, s);
  band_attn_kernel<T, kNch><<<grid, kThreads, smem, s>>>(mx, mw, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_band_attention_fused(const CUtensorMap& map_xn, const CUtensorMap& map_w, const BandAttnParams& p,
                                        int bf16, int num_sms, cudaStream_t stream) {
  if (p.F < 1 || p.F > 64 || p.slot != attn_band_slot(p.F) || p.D % 64 != 0 || p.D < 64 || p.D > 512 ||
      p.heads < 1 || p.inner != p.heads * 64 || p.num_seqs < 0 || p.out_ld < p.inner)
    return cudaErrorInvalidValue;
  if (p.num_seqs == 0) return cudaSuccess;
  if (p.slot == 32)
    return bf16 ? launch_band_t<__nv_bfloat16, 1>(map_xn, map_w, p, num_sms, stream)
                : launch_band_t<__half, 1>(map_xn, map_w, p, num_sms, stream);
  return bf16 ? launch_band_t<__nv_bfloat16, 2>(map_xn, map_w, p, num_sms, stream)
              : launch_band_t<__half, 2>(map_xn, map_w, p, num_sms, stream);
}

MSST_DEFINE_ERROR_ACCESSOR(band_attention_device_error)

}  // namespace msst
