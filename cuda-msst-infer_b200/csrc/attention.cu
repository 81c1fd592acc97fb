// attention.cu — tcgen05 flash attention for the Roformer's axial attention on
// sm_100a (head_dim 64, non-causal).  Two kernels, both persistent over work items
// that are PAIRS of 128-row query tiles (a, b) of one head:
//   attention_time_kernel (time axis, and msst_sdpa): two consecutive q-tiles of one
//              (sequence, head) unit share every K/V tile; the odd tail tiles of two
//              units form a pair with one K/V stream each.  Split-key softmax
//              halves on 16 warps (see the kernel).
//   attention_band_kernel (band axis): two consecutive packed tiles (sequences at
//              aligned 32/64/128-row slots, block-diagonal mask); each has its own
//              single K/V tile.  CTA = 320 threads:
//   warp 0     TMA producer: Q_a/Q_b, K/V tiles through a 4-stage ring
//   warp 1     MMA issuer: S_w = Q_w K^T (M128 N128 K64) and O_w += P_w V
//              (M128 N64 K128, P read from TMEM), issued per tile as
//              PV_a(j), S_a(j+1), PV_b(j), S_b(j+1) so that S_w(j+1)'s completion
//              also guarantees PV_w(j) has finished reading P_w
//   warps 2-5  softmax of tile a, warps 6-9 softmax of tile b: one query row per
//              thread; steady-state tiles take one pass over S in TMEM (exponent
//              against the running reference max, which moves lazily: only a row
//              sum above 4096 sends a warp through the exact two passes, which
//              move the max and rescale O in TMEM), P
//              written as packed 16-bit pairs into TMEM (the MMA's A operand);
//              fully masked 32-column chunks are skipped per warp.  The epilogue
//              divides by the row sum, applies the head gate and writes the
//              merged-head row.
//   TMEM: S_a [0,128) S_b [128,256) O_a [256,320) O_b [320,384) P_a [384,448) P_b [448,512).
#include "attention.cuh"
#include "common.cuh"

namespace msst {

namespace {

constexpr int kKvStages = 4;
constexpr int kThreads = 320;
constexpr uint32_t kTileBytes = 128 * 64 * 2;   // one 128x64 16-bit tile
constexpr size_t kAttnSmem = 1024 + 2 * kTileBytes + kKvStages * 2 * kTileBytes + 256;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256, kColP = 384;
// A steady-state step exponentiates against the reference max without tracking
// the row's maximum; its row sum bounds every P entry, so a sum above this bound
// (or not finite) sends the row's warp through the exact passes.  4096 leaves P
// far inside fp16's range and is never reached by a row whose scores stay at or
// below the reference max (at most 128 entries of 1 per step).
constexpr float kSumLimit = 4096.0f;
// Of every 4 column pairs of an unmasked 32-column chunk, this many take their
// exponentials from the FMA-pipe polynomial (poly_exp2x2) and the rest from the
// MUFU unit.  With the steady state's per-element max tracking gone, all-MUFU is
// the fastest mix on both axes (fp16 and bf16: 3-5 % ahead of one pair in four,
// whose extra FMA-pipe instructions now cost more issue slots than the MUFU
// work they take over).
#ifndef MSST_ATTN_POLY_PAIRS
#define MSST_ATTN_POLY_PAIRS 0
#endif
constexpr int kPolyPairsPerQuad = MSST_ATTN_POLY_PAIRS;

struct PairGeom {
  int steps;        // K/V tiles streamed for this pair
  bool has_b;       // second query tile present
  bool split;       // time axis: the two tiles belong to different (sequence, head) units,
                    // each with its own K/V stream (tile w uses the steps j with j % 2 == w)
  // time axis: unit of each tile (head, chunk b, band f) and its first query row
  int head, b, f, t0a;
  int head2, b2, f2, t0b;
  // band axis
  int r0a, rows;    // first sequence of tile a; sequences per packed tile
};

// Time axis (modes 0, 2): a unit is one (sequence, head), u = (b * F + f) * heads + head,
// with q_tiles query tiles.  Its tiles go in pairs (2 qp, 2 qp + 1) sharing every K/V
// tile.  When q_tiles is odd the last tile of each unit is a short tail (33 rows of an
// 801-frame sequence); the tails of units 2g and 2g + 1 run as one pair, each with its
// own K/V stream, so no query tile runs without a partner.  Items are ordered by unit
// group g: the full pairs of unit 2g, those of unit 2g + 1, then their tail pair.
__device__ __forceinline__ void time_unit(const AttnParams& p, int u, int& head, int& b, int& f) {
  head = u % p.heads;
  const int s = u / p.heads;
  b = s / p.F;
  f = s - b * p.F;
}

template <bool kBand>
__device__ __forceinline__ PairGeom pair_geom(const AttnParams& p, int item) {
  PairGeom g;
  g.split = false;
  if constexpr (!kBand) {
    const int full = p.q_tiles >> 1;       // full pairs per unit
    const int tail = p.q_tiles & 1;        // a tail tile per unit
    const int per_group = 2 * full + tail;
    const int units = p.units;
    int u0, kind;                          // kind < full: full pair `kind` of unit u0; else the tail
    const int pg = item / per_group, r = item - pg * per_group;
    if (2 * pg + 1 < units || units % 2 == 0) {
      u0 = 2 * pg + (r < 2 * full ? r / full : 0);
      kind = r < 2 * full ? r % full : full;
    } else {
      // the last unit of an odd count, alone in its group: its full pairs, then its tail
      u0 = 2 * pg;
      kind = r;
    }
    time_unit(p, u0, g.head, g.b, g.f);
    g.steps = p.kv_tiles;
    if (kind < full) {
      g.t0a = kind * 256;
      g.has_b = true;
      g.head2 = g.head;
      g.b2 = g.b;
      g.f2 = g.f;
      g.t0b = g.t0a + 128;
    } else {
      g.t0a = g.t0b = full * 256;
      g.has_b = u0 + 1 < units && u0 % 2 == 0;
      if (g.has_b) {
        g.split = true;
        g.steps = 2 * p.kv_tiles;
        time_unit(p, u0 + 1, g.head2, g.b2, g.f2);
      } else {
        g.head2 = g.head;
        g.b2 = g.b;
        g.f2 = g.f;
      }
    }
    g.r0a = g.rows = 0;
  } else {
    g.head = g.head2 = item % p.heads;
    const int pr = item / p.heads;
    g.rows = p.seqs_per_tile;
    g.r0a = 2 * pr * g.rows;
    g.has_b = 2 * pr + 1 < p.q_tiles;
    g.steps = g.has_b ? 2 : 1;
    g.b = g.f = g.t0a = g.b2 = g.f2 = g.t0b = 0;
  }
  return g;
}

// Does query tile w (0 = a, 1 = b) consume K/V step j?
template <bool kBand>
__device__ __forceinline__ bool uses(const PairGeom& g, int w, int j) {
  if constexpr (kBand)
    return j == w;
  else
    return g.split ? (j & 1) == w : true;
}

// K/V tile index of step j of a time-axis pair
__device__ __forceinline__ int kv_block(const PairGeom& g, int j) { return g.split ? (j >> 1) : j; }

// ---------------------------------------------------------------------------
// One softmax pass over a 128-column S row held in TMEM (4 chunks of 32
// columns, loads software-pipelined: chunk ch+1 is in flight while ch is
// processed).  Chunks outside [c_lo, c_hi) are fully masked for the whole warp;
// chunks below `c_full` need no per-column mask (warp-uniform), the others mask
// columns outside [klo, khi).
//   kPass 0: row max of the valid scores -> mx
//   kPass 1, 2: P = exp2(s*c - mc) into TMEM, row sum
// ---------------------------------------------------------------------------
// kStore false (kPass 1, 2 only): P is left in pk for the caller instead of stored.
template <typename T, int kPass, bool kStore = true>
__device__ __forceinline__ void process_chunk(const uint32_t (&r)[32], int ch, bool in_range, bool unmasked, int klo,
                                              int khi, float2 c2, float2 nm2, float& mx, float2& sum2,
                                              uint32_t pAddr, uint32_t (&pk)[16]) {
  if constexpr (kPass == 0) {
    if (!in_range) return;
    float m0 = -INFINITY, m1 = -INFINITY;
    if (unmasked) {
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        m0 = fmaxf(m0, __uint_as_float(r[i]));
        m1 = fmaxf(m1, __uint_as_float(r[i + 1]));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const int col = ch * 32 + i;
        if (col >= klo && col < khi) m0 = fmaxf(m0, __uint_as_float(r[i]));
        if (col + 1 >= klo && col + 1 < khi) m1 = fmaxf(m1, __uint_as_float(r[i + 1]));
      }
    }
    mx = fmaxf(mx, fmaxf(m0, m1));
  } else {
    if (!in_range) {
#pragma unroll
      for (int i = 0; i < 16; ++i) pk[i] = 0u;
    } else if (unmasked) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float2 a = __ffma2_rn(make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), c2, nm2);
        float2 e;
        if ((i & 3) < kPolyPairsPerQuad) {
          e = poly_exp2x2(a);
        } else {
          e.x = fast_exp2(a.x);
          e.y = fast_exp2(a.y);
        }
        sum2 = __fadd2_rn(sum2, e);
        pk[i] = pack2<T>(e.x, e.y);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int col = ch * 32 + 2 * i;
        const bool v0 = col >= klo && col < khi, v1 = col + 1 >= klo && col + 1 < khi;
        const float2 a = __ffma2_rn(make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), c2, nm2);
        const float e0 = v0 ? fast_exp2(a.x) : 0.f, e1 = v1 ? fast_exp2(a.y) : 0.f;
        sum2 = __fadd2_rn(sum2, make_float2(e0, e1));
        pk[i] = pack2<T>(e0, e1);
      }
    }
    // P row chunk -> TMEM (16 columns of packed 16-bit pairs), the A operand of O += P.V
    if constexpr (kStore) tmem_st16(pAddr + ch * 16, pk);
  }
}

template <typename T, int kPass>
__device__ __forceinline__ void process_chunk(const uint32_t (&r)[32], int ch, bool in_range, bool unmasked, int klo,
                                              int khi, float2 c2, float2 nm2, float& mx, float2& sum2,
                                              uint32_t pAddr) {
  uint32_t pk[16];
  process_chunk<T, kPass, true>(r, ch, in_range, unmasked, klo, khi, c2, nm2, mx, sum2, pAddr, pk);
}

// One pass over a 128-column S row held in TMEM (4 chunks of 32 columns, loads
// software-pipelined: chunk ch+1 is in flight while ch is processed).  Chunks
// outside [c_lo, c_hi) get P = 0 (they are loaded all the same: predicated TMEM
// loads keep both register buffers live and spill).
// Chunks in [c_lo, c_full) need no per-column mask.
// kFirst (with kPass 1): the reference max is not known yet; it is taken from the
// first loaded chunk's valid scores (returned in m0), and the pass proceeds as a
// steady-state pass against it (the caller falls back to the exact two passes if
// the row sum shows that a later chunk went far above it); the first chunk is the
// first of the row's window, c_lo.
template <typename T, int kPass, bool kFirst = false>
__device__ __forceinline__ void row_pass(uint32_t sAddr, int c_lo, int c_hi, int c_full, int klo, int khi, float c,
                                         float mc, float& mx, float2& sum2, uint32_t pAddr, float* m0 = nullptr) {
  float2 c2 = make_float2(c, c), nm2 = make_float2(-mc, -mc);
  auto first_max = [&](const uint32_t(&r)[32], int ch) {
    if constexpr (kFirst) {
      if (ch == c_lo) {
        float m = -INFINITY;
        process_chunk<T, 0>(r, ch, true, ch < c_full, klo, khi, c2, nm2, m, sum2, pAddr);
        *m0 = m;
        const float mcf = (m == -INFINITY) ? 0.f : m * c;
        nm2 = make_float2(-mcf, -mcf);
      }
    }
  };
  const bool in0 = c_lo <= 0 && 0 < c_hi, in1 = c_lo <= 1 && 1 < c_hi;
  const bool in2 = c_lo <= 2 && 2 < c_hi, in3 = c_lo <= 3 && 3 < c_hi;
  uint32_t ra[32], rb[32];
  tmem_ld32(sAddr, ra);
  tmem_ld_wait(ra);
  tmem_ld32(sAddr + 32, rb);
  first_max(ra, 0);
  process_chunk<T, kPass>(ra, 0, in0, c_lo <= 0 && 0 < c_full, klo, khi, c2, nm2, mx, sum2, pAddr);
  tmem_ld_wait(rb);
  tmem_ld32(sAddr + 64, ra);
  first_max(rb, 1);
  process_chunk<T, kPass>(rb, 1, in1, c_lo <= 1 && 1 < c_full, klo, khi, c2, nm2, mx, sum2, pAddr);
  tmem_ld_wait(ra);
  tmem_ld32(sAddr + 96, rb);
  first_max(ra, 2);
  process_chunk<T, kPass>(ra, 2, in2, c_lo <= 2 && 2 < c_full, klo, khi, c2, nm2, mx, sum2, pAddr);
  tmem_ld_wait(rb);
  first_max(rb, 3);
  process_chunk<T, kPass>(rb, 3, in3, c_lo <= 3 && 3 < c_full, klo, khi, c2, nm2, mx, sum2, pAddr);
}

// Band axis (mode 1): packed tiles of whole sequences, block-diagonal mask.
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    attention_band_kernel(const __grid_constant__ CUtensorMap qkv, const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap vmap, const __grid_constant__ AttnParams p) {
  constexpr uint32_t kIsBf16 = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                              // Q_a, Q_b
  uint8_t* sKV = sQ + 2 * kTileBytes;              // stages x (K, V)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kKvStages * 2 * kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* kv_full = bars + 2;
  uint64_t* kv_empty = kv_full + kKvStages;
  uint64_t* s_full = kv_empty + kKvStages;  // [2]
  uint64_t* p_full = s_full + 2;            // [2]
  uint64_t* o_done = p_full + 2;            // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    for (int s = 0; s < kKvStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&qkv);
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
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
      int pc = 0, kvc = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.total_items; item += gridDim.x, ++pc) {
        const PairGeom g = pair_geom<true>(p, item);
        if (!mbar_wait<false>(q_empty, (pc & 1) ^ 1, kErrTimeoutAttnQ, abort_flag)) break;
        mbar_arrive_expect_tx(q_full, (g.has_b ? 2 : 1) * kTileBytes);
        const int xq = g.head * 64;
        // one box of `slot` rows per sequence, at its aligned slot of the tile
        const uint32_t slot_bytes = (128u / (uint32_t)g.rows) * 128u;
        for (int w = 0; w < (g.has_b ? 2 : 1); ++w)
          for (int k = 0; k < g.rows; ++k)
            tma_load_4d(sQ + w * kTileBytes + k * slot_bytes, &qkv, q_full, xq,
                        (g.r0a + w * g.rows + k) * p.seq_len, 0, 0);
        const int xk = p.k_col + g.head * 64, xv = p.v_col + g.head * 64;
        for (int j = 0; j < g.steps; ++j, ++kvc) {
          const int st = kvc % kKvStages;
          if (!mbar_wait<false>(&kv_empty[st], ((kvc / kKvStages) & 1) ^ 1, kErrTimeoutAttnKV, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * kTileBytes);
          uint8_t* dk = sKV + st * 2 * kTileBytes;
          for (int k = 0; k < g.rows; ++k) {
            const int r0 = (g.r0a + j * g.rows + k) * p.seq_len;
            tma_load_4d(dk + k * slot_bytes, &kmap, &kv_full[st], xk, r0, 0, 0);
            tma_load_4d(dk + kTileBytes + k * slot_bytes, &vmap, &kv_full[st], xv, r0, 0, 0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_f16(kIsBf16, 128, 0);
      const uint32_t idesc_o = umma_idesc_f16(kIsBf16, 64, 1);
      int pc = 0, kvc = 0;
      uint32_t pcnt[2] = {0, 0};  // P tiles consumed per query tile (phase of p_full)
      bool ok = true;
      // Shared-memory descriptors are built once per operand tile; each 16-element
      // k-step advances the start-address field (bytes >> 4) by a constant: 32 B along
      // a K-major row (S), 16 rows of 128 B down the MN-major V tile (P.V).  The issuing
      // thread is on the kernel's critical path, so its per-MMA work is kept minimal.
      const uint64_t dq0 = sw128_desc(smem_u32(sQ), 16, 1024);
      const uint64_t dkv0 = sw128_desc(smem_u32(sKV), 16, 1024);
      const uint64_t dv0 = sw128_desc(smem_u32(sKV + kTileBytes), kTileBytes, 1024);
      auto issue_s = [&](int w, int st) {
        const uint64_t dq = dq0 + (uint64_t)((w * kTileBytes) >> 4);
        const uint64_t dk = dkv0 + (uint64_t)((st * 2 * kTileBytes) >> 4);
        const uint32_t dS = tmem + kColS + (uint32_t)(w * 128);
        umma_f16_ss(dS, dq, dk, idesc_s, 0u);
#pragma unroll
        for (int kk = 1; kk < 4; ++kk) umma_f16_ss(dS, dq + 2 * kk, dk + 2 * kk, idesc_s, 1u);
        umma_commit(&s_full[w]);
      };
      auto issue_pv = [&](int w, int st, bool first) -> bool {
        if (!mbar_wait<false>(&p_full[w], pcnt[w] & 1, kErrTimeoutAttnP, abort_flag)) return false;
        ++pcnt[w];
        tc_fence_after();
        const uint32_t paddr = tmem + kColP + (uint32_t)(w * 64);
        const uint64_t dv = dv0 + (uint64_t)((st * 2 * kTileBytes) >> 4);
        const uint32_t dO = tmem + kColO + (uint32_t)(w * 64);
        umma_f16_ts(dO, paddr, dv, idesc_o, first ? 0u : 1u);
#pragma unroll
        for (int kk = 1; kk < 8; ++kk) umma_f16_ts(dO, paddr + (uint32_t)(kk * 8), dv + 128 * kk, idesc_o, 1u);
        return true;
      };
      for (int item = blockIdx.x; ok && item < p.total_items; item += gridDim.x, ++pc) {
        const PairGeom g = pair_geom<true>(p, item);
        const int nw = g.has_b ? 2 : 1;
        if (!mbar_wait<false>(q_full, pc & 1, kErrTimeoutAttnQ, abort_flag)) break;
        tc_fence_after();
        int last_used[2] = {-1, -1};  // K/V stage of each tile's previous step
        int used_count[2] = {0, 0};
        for (int j = 0; ok && j < g.steps; ++j) {
          const int st = (kvc + j) % kKvStages;
          if (!mbar_wait<false>(&kv_full[st], ((kvc + j) / kKvStages) & 1, kErrTimeoutAttnKV, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int w = 0; w < nw; ++w) {
            if (!uses<true>(g, w, j)) continue;
            if (last_used[w] >= 0) {
              if (!issue_pv(w, last_used[w], used_count[w] == 1)) {
                ok = false;
                break;
              }
              // the previous K/V stage is free once the last tile using it has issued its PV
              umma_commit(&kv_empty[last_used[w]]);  // each K/V stage serves one tile
            }
            issue_s(w, st);
            last_used[w] = st;
            ++used_count[w];
          }
        }
        if (!ok) break;
        umma_commit(q_empty);  // every S of this pair has been issued
        for (int w = 0; w < nw; ++w) {
          if (!issue_pv(w, last_used[w], used_count[w] == 1)) {
            ok = false;
            break;
          }
          umma_commit(&kv_empty[last_used[w]]);  // each K/V stage serves one tile
          umma_commit(&o_done[w]);
        }
        kvc += g.steps;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int w = (warp - 2) >> 2;  // query tile of this warp group
    const int q = warp & 3;         // TMEM lane quarter
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t sAddr = tmem + lane_off + kColS + (uint32_t)(w * 128);
    const uint32_t oAddr = tmem + lane_off + kColO + (uint32_t)(w * 64);
    const uint32_t pAddr = tmem + lane_off + kColP + (uint32_t)(w * 64);
    const float c = p.scale_log2;
    uint32_t scnt = 0, ocnt = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.total_items; item += gridDim.x) {
      const PairGeom g = pair_geom<true>(p, item);
      if (w == 1 && !g.has_b) continue;
      // rows of this thread / warp
      const int slot = 128 / g.rows;
      const int k = row / slot, rr = row - k * slot;
      const int sq = g.r0a + w * g.rows + k;  // sequence of this row
      const bool valid = rr < p.seq_len && (long long)sq * p.seq_len < p.num_tokens;
      const long long token = (long long)sq * p.seq_len + rr;
      const int lo = k * slot, hi_seq = lo + p.seq_len;
      const bool warp_active = __any_sync(0xffffffffu, valid);
      float m = -INFINITY, l = 0.f;
      int used = 0;
      for (int j = 0; j < g.steps; ++j) {
        if (!uses<true>(g, w, j)) continue;
        if (!mbar_wait<false>(&s_full[w], scnt & 1, kErrTimeoutAttnS, abort_flag)) {
          ok = false;
          break;
        }
        ++scnt;
        tc_fence_after();
        // valid key columns [klo, khi) of this tile for this row: the row's slot; klo is
        // warp-uniform and 32-aligned (a warp's rows lie in one slot)
        const int klo = lo, khi = hi_seq;
        const int c_lo = klo >> 5, c_hi = (khi + 31) >> 5;  // chunks holding any valid column
        if (warp_active) {
          // chunks [c_lo, c_full) need no per-column mask
          const int c_full = khi >> 5;
          float2 sum2 = make_float2(0.f, 0.f);
          bool exact = false;
          if (!exact) {
            // steady state: exponentiate against the current reference max in one pass; a
            // tile's first step takes its reference max from the first 32 columns.  The
            // row sum bounds how far above the reference the row went.
            float amax = -INFINITY;  // unused by the steady-state passes
            if (used == 0) {
              float m0 = -INFINITY;
              row_pass<T, 1, true>(sAddr, c_lo, c_hi, c_full, klo, khi, c, 0.f, amax, sum2, pAddr, &m0);
              m = m0;
            } else {
              const float mc = (m == -INFINITY) ? 0.f : m * c;
              row_pass<T, 1>(sAddr, c_lo, c_hi, c_full, klo, khi, c, mc, amax, sum2, pAddr);
            }
            if (__any_sync(0xffffffffu, !(sum2.x + sum2.y <= kSumLimit))) {
              exact = true;
              sum2 = make_float2(0.f, 0.f);
              if (used == 0) m = -INFINITY;
            }
          }
          if (exact) {
            float mx = -INFINITY;
            row_pass<T, 0>(sAddr, c_lo, c_hi, c_full, klo, khi, c, 0.f, mx, sum2, pAddr);
            // move the reference max to the row's true max (O and l rescaled), so the
            // following steady-state steps stay below the sum bound
            const bool grow = mx > m;
            if (__any_sync(0xffffffffu, grow)) {
              const float m_new = grow ? mx : m;
              const float alpha = (m == -INFINITY) ? 0.f : fast_exp2((m - m_new) * c);
              if (used > 0) {
                // O_w holds the previous tiles' P.V (complete: S_w(j) was issued after PV_w(j-1))
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  uint32_t r[32];
                  tmem_ld32(oAddr + h * 32, r);
                  tmem_ld_wait(r);
#pragma unroll
                  for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                  tmem_st32(oAddr + h * 32, r);
                }
                tmem_st_wait();
              }
              l *= alpha;
              m = m_new;
            }
            const float mc = (m == -INFINITY) ? 0.f : m * c;
            float unused = 0.f;
            row_pass<T, 2>(sAddr, c_lo, c_hi, c_full, klo, khi, c, mc, unused, sum2, pAddr);
          }
          l += sum2.x + sum2.y;
          tmem_st_wait();
        }
        ++used;
        tc_fence_before();
        mbar_arrive(&p_full[w]);
      }
      if (!ok) break;
      // epilogue: O_w complete after the pair's last PV
      if (!mbar_wait<false>(&o_done[w], ocnt & 1, kErrTimeoutAttnO, abort_flag)) break;
      ++ocnt;
      tc_fence_after();
      if (warp_active) {
        float scale = l > 0.f ? 1.f / l : 0.f;
        const int head = w == 0 ? g.head : g.head2;
        if (valid && p.gates != nullptr) scale *= __ldg(p.gates + token * p.heads + head);
        uint4* out = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.out) + token * p.out_ld + head * 64);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t r[32];
          tmem_ld32(oAddr + h * 32, r);
          tmem_ld_wait();
          if (valid) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              if (8 * (4 * h + u) >= p.d_out) break;
              float v[8];
#pragma unroll
              for (int k = 0; k < 8; ++k) v[k] = __uint_as_float(r[8 * u + k]) * scale;
              out[4 * h + u] = make_uint4(pack2<T>(v[0], v[1]), pack2<T>(v[2], v[3]), pack2<T>(v[4], v[5]),
                                          pack2<T>(v[6], v[7]));
            }
          }
        }
      }
      tc_fence_before();
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Time axis (modes 0 and 2) with split-key softmax halves.
//
// The time-axis item schedule (pair_geom), a TMA producer and an MMA issue order like
// attention_band_kernel's, but
// each query tile's softmax runs on 8 warps: the two warps of a TMEM lane quarter
// take keys [0, 64) and [64, 128) of every 128-key block.  Each half keeps its own
// running max m and sum l and accumulates its own O (P_half V_half, 4 MMAs of
// K = 16 each, so a K/V step still costs 12 MMAs per tile), with its P written
// over its own half of S; the halves never wait for each other during the steps.
// At the end of an item the two warps exchange m and l through shared memory (an
// mbarrier per tile and quarter, bounded wait) and each writes 32 of the 64 output
// columns: O = (O_0 a_0 + O_1 a_1) / (l_0 a_0 + l_1 a_1), a_h = 2^((m_h - m) c),
// m = max(m_0, m_1) -- the merge of two online-softmax partial results.
// Twice the softmax warps per tile hide the exponentials' latency (one warp per
// SMSP per tile could not keep the MUFU busy).
// CTA = 576 threads: warp 0 TMA, warp 1 MMA, warps 2-17 softmax (tile (w-2)/8,
// key half ((w-2)/4) & 1, lane quarter w % 4).  18 warps put 5 on two of the SM's
// four register partitions (16K registers each), so a thread has at most 96.
// TMEM: S_a [0,128) S_b [128,256) (P_half over [h*64, h*64 + 32) of S), O_a,0
// [256,320) O_a,1 [320,384) O_b,0 [384,448) O_b,1 [448,512).  S_w(j+1) overwrites
// P_w(j) only after P_w(j).V(j) has read it: the MMAs of one thread run in issue
// order, and S_w(j+1) is issued after that P.V.
// ---------------------------------------------------------------------------
constexpr int kTThreads = 576;
constexpr uint32_t kColO2 = 256;
// the m / l exchange ([item parity][tile][half][m, l][128] floats) after the barriers
constexpr size_t kTimeSmem = kAttnSmem + 2 * 2 * 2 * 2 * 128 * sizeof(float) + 64;

// One pass over a key half (two 32-column chunks) of an S row; chunks >= c_hi get
// P = 0, chunks below c_full need no mask, khi is relative to the half.  The chunks
// are loaded one after the other into one register buffer (the 576-thread CTA has
// 96 registers a thread; the other softmax warps on the SMSP cover the load latency).
// P overlays the half's first 32 S columns, so a pass that may have to be redone
// (kPass 1: the row-sum check decides) leaves P in pk0 / pk1 for the caller to
// store; the exact passes (0, then 2) read S intact and kPass 2 stores P.
template <typename T, int kPass, bool kFirst = false>
__device__ __forceinline__ void half_pass(uint32_t sAddr, int c_hi, int c_full, int khi, float c, float mc, float& mx,
                                          float2& sum2, uint32_t pAddr, uint32_t (&pk0)[16], uint32_t (&pk1)[16],
                                          float* m0 = nullptr) {
  constexpr bool kStore = kPass != 1;
  float2 c2 = make_float2(c, c), nm2 = make_float2(-mc, -mc);
  uint32_t ra[32];
  tmem_ld32(sAddr, ra);
  tmem_ld_wait(ra);
  if constexpr (kFirst) {
    float m = -INFINITY;
    if (0 < c_hi) process_chunk<T, 0, false>(ra, 0, true, 0 < c_full, 0, khi, c2, nm2, m, sum2, pAddr, pk0);
    *m0 = m;
    const float mcf = (m == -INFINITY) ? 0.f : m * c;
    nm2 = make_float2(-mcf, -mcf);
  }
  process_chunk<T, kPass, kStore>(ra, 0, 0 < c_hi, 0 < c_full, 0, khi, c2, nm2, mx, sum2, pAddr, pk0);
  tmem_ld32(sAddr + 32, ra);
  tmem_ld_wait(ra);
  process_chunk<T, kPass, kStore>(ra, 1, 1 < c_hi, 1 < c_full, 0, khi, c2, nm2, mx, sum2, pAddr, pk1);
}

template <typename T>
__global__ void __launch_bounds__(kTThreads, 1)
    attention_time_kernel(const __grid_constant__ CUtensorMap qkv, const __grid_constant__ CUtensorMap kmap,
                          const __grid_constant__ CUtensorMap vmap, const __grid_constant__ AttnParams p) {
  constexpr uint32_t kIsBf16 = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                              // Q_a, Q_b
  uint8_t* sKV = sQ + 2 * kTileBytes;              // stages x (K, V)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kKvStages * 2 * kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* kv_full = bars + 2;
  uint64_t* kv_empty = kv_full + kKvStages;
  uint64_t* s_full = kv_empty + kKvStages;  // [2]
  uint64_t* p_full = s_full + 2;            // [2]
  uint64_t* o_done = p_full + 2;            // [2]
  uint64_t* ml_bar = o_done + 2;            // [2 tiles][4 quarters]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ml_bar + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_ml = reinterpret_cast<float*>(tmem_slot + 4);  // [item parity][tile][half][m, l][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&o_done[i], 1);
    }
    for (int i = 0; i < 8; ++i) mbar_init(&ml_bar[i], 2);
    for (int s = 0; s < kKvStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&qkv);
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
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
      int pc = 0, kvc = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.total_items; item += gridDim.x, ++pc) {
        const PairGeom g = pair_geom<false>(p, item);
        if (!mbar_wait<false>(q_empty, (pc & 1) ^ 1, kErrTimeoutAttnQ, abort_flag)) break;
        mbar_arrive_expect_tx(q_full, (g.has_b ? 2 : 1) * kTileBytes);
        tma_load_4d(sQ, &qkv, q_full, g.head * 64, g.f, g.t0a, g.b);
        if (g.has_b) tma_load_4d(sQ + kTileBytes, &qkv, q_full, g.head2 * 64, g.f2, g.t0b, g.b2);
        const int xk = p.k_col + g.head * 64, xv = p.v_col + g.head * 64;
        const int xk2 = p.k_col + g.head2 * 64, xv2 = p.v_col + g.head2 * 64;
        for (int j = 0; j < g.steps; ++j, ++kvc) {
          const int st = kvc % kKvStages;
          if (!mbar_wait<false>(&kv_empty[st], ((kvc / kKvStages) & 1) ^ 1, kErrTimeoutAttnKV, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * kTileBytes);
          uint8_t* dk = sKV + st * 2 * kTileBytes;
          // a split pair's odd steps stream the second unit's K/V
          const bool second = g.split && (j & 1);
          const int kb = kv_block(g, j) * 128;
          tma_load_4d(dk, &kmap, &kv_full[st], second ? xk2 : xk, second ? g.f2 : g.f, kb, second ? g.b2 : g.b);
          tma_load_4d(dk + kTileBytes, &vmap, &kv_full[st], second ? xv2 : xv, second ? g.f2 : g.f, kb,
                      second ? g.b2 : g.b);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_f16(kIsBf16, 128, 0);
      const uint32_t idesc_o = umma_idesc_f16(kIsBf16, 64, 1);
      int pc = 0, kvc = 0;
      uint32_t pcnt[2] = {0, 0};
      bool ok = true;
      const uint64_t dq0 = sw128_desc(smem_u32(sQ), 16, 1024);
      const uint64_t dkv0 = sw128_desc(smem_u32(sKV), 16, 1024);
      const uint64_t dv0 = sw128_desc(smem_u32(sKV + kTileBytes), kTileBytes, 1024);
      auto issue_s = [&](int w, int st) {
        const uint64_t dq = dq0 + (uint64_t)((w * kTileBytes) >> 4);
        const uint64_t dk = dkv0 + (uint64_t)((st * 2 * kTileBytes) >> 4);
        const uint32_t dS = tmem + kColS + (uint32_t)(w * 128);
        umma_f16_ss(dS, dq, dk, idesc_s, 0u);
#pragma unroll
        for (int kk = 1; kk < 4; ++kk) umma_f16_ss(dS, dq + 2 * kk, dk + 2 * kk, idesc_s, 1u);
        umma_commit(&s_full[w]);
      };
      // O_w,h += P_w,h V[64 h, 64 h + 64): P_w,h sits over S_w's columns [64 h, 64 h + 32)
      auto issue_pv = [&](int w, int st, bool first) -> bool {
        if (!mbar_wait<false>(&p_full[w], pcnt[w] & 1, kErrTimeoutAttnP, abort_flag)) return false;
        ++pcnt[w];
        tc_fence_after();
        const uint64_t dv = dv0 + (uint64_t)((st * 2 * kTileBytes) >> 4);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t pa = tmem + kColS + (uint32_t)(w * 128 + h * 64);
          const uint32_t dO = tmem + kColO2 + (uint32_t)(w * 128 + h * 64);
          umma_f16_ts(dO, pa, dv + 128 * (4 * h), idesc_o, first ? 0u : 1u);
#pragma unroll
          for (int kk = 1; kk < 4; ++kk)
            umma_f16_ts(dO, pa + (uint32_t)(kk * 8), dv + 128 * (4 * h + kk), idesc_o, 1u);
        }
        return true;
      };
      for (int item = blockIdx.x; ok && item < p.total_items; item += gridDim.x, ++pc) {
        const PairGeom g = pair_geom<false>(p, item);
        const int nw = g.has_b ? 2 : 1;
        if (!mbar_wait<false>(q_full, pc & 1, kErrTimeoutAttnQ, abort_flag)) break;
        tc_fence_after();
        int last_used[2] = {-1, -1};
        int used_count[2] = {0, 0};
        for (int j = 0; ok && j < g.steps; ++j) {
          const int st = (kvc + j) % kKvStages;
          if (!mbar_wait<false>(&kv_full[st], ((kvc + j) / kKvStages) & 1, kErrTimeoutAttnKV, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int w = 0; w < nw; ++w) {
            if (!uses<false>(g, w, j)) continue;
            if (last_used[w] >= 0) {
              if (!issue_pv(w, last_used[w], used_count[w] == 1)) {
                ok = false;
                break;
              }
              if (w == nw - 1 || g.split) umma_commit(&kv_empty[last_used[w]]);
            }
            issue_s(w, st);
            last_used[w] = st;
            ++used_count[w];
          }
        }
        if (!ok) break;
        umma_commit(q_empty);
        for (int w = 0; w < nw; ++w) {
          if (!issue_pv(w, last_used[w], used_count[w] == 1)) {
            ok = false;
            break;
          }
          if (w == nw - 1 || g.split) umma_commit(&kv_empty[last_used[w]]);
          umma_commit(&o_done[w]);
        }
        kvc += g.steps;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int w = (warp - 2) >> 3;        // query tile
    const int hf = ((warp - 2) >> 2) & 1; // key half
    const int q = warp & 3;               // TMEM lane quarter
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t sAddr = tmem + lane_off + kColS + (uint32_t)(w * 128 + hf * 64);  // S half and P half
    const uint32_t oAddr = tmem + lane_off + kColO2 + (uint32_t)(w * 128 + hf * 64);  // this half's O
    const uint32_t oBase = tmem + lane_off + kColO2 + (uint32_t)(w * 128);            // O_w,0; O_w,1 at +64
    uint64_t* mlb = &ml_bar[w * 4 + q];
    const float c = p.scale_log2;
    uint32_t scnt = 0, ocnt = 0, mlc = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.total_items; item += gridDim.x) {
      const PairGeom g = pair_geom<false>(p, item);
      if (w == 1 && !g.has_b) continue;
      const int t = (w == 0 ? g.t0a : g.t0b) + row;
      const bool valid = t < p.T;
      const long long token = ((long long)(w == 0 ? g.b : g.b2) * p.T + t) * p.F + (w == 0 ? g.f : g.f2);
      const bool warp_active = __any_sync(0xffffffffu, valid);
      float m = -INFINITY, l = 0.f;
      int used = 0;
      for (int j = 0; j < g.steps; ++j) {
        if (!uses<false>(g, w, j)) continue;
        if (!mbar_wait<false>(&s_full[w], scnt & 1, kErrTimeoutAttnS, abort_flag)) {
          ok = false;
          break;
        }
        ++scnt;
        tc_fence_after();
        // valid keys of this half in this block, relative to the half
        const int khi = max(0, min(64, p.kv_len - kv_block(g, j) * 128 - hf * 64));
        const int c_hi = (khi + 31) >> 5, c_full = khi >> 5;
        if (warp_active) {
          float2 sum2 = make_float2(0.f, 0.f);
          float unused = 0.f;
          uint32_t pk0[16], pk1[16];
          if (used == 0) {
            float m0 = -INFINITY;
            half_pass<T, 1, true>(sAddr, c_hi, c_full, khi, c, 0.f, unused, sum2, sAddr, pk0, pk1, &m0);
            m = m0;
          } else {
            const float mc = (m == -INFINITY) ? 0.f : m * c;
            half_pass<T, 1>(sAddr, c_hi, c_full, khi, c, mc, unused, sum2, sAddr, pk0, pk1);
          }
          if (__all_sync(0xffffffffu, sum2.x + sum2.y <= kSumLimit)) {
            tmem_st16(sAddr, pk0);
            tmem_st16(sAddr + 16, pk1);
          } else {
            // exact passes: the half's row max, O_half and l rescaled to it, P again
            sum2 = make_float2(0.f, 0.f);
            if (used == 0) m = -INFINITY;
            float mx = -INFINITY;
            half_pass<T, 0>(sAddr, c_hi, c_full, khi, c, 0.f, mx, sum2, sAddr, pk0, pk1);
            const bool grow = mx > m;
            if (__any_sync(0xffffffffu, grow)) {
              const float m_new = grow ? mx : m;
              const float alpha = (m == -INFINITY) ? 0.f : fast_exp2((m - m_new) * c);
              if (used > 0) {
                // O_half holds the previous steps' P.V (complete: S_w(j) was issued after PV_w(j-1))
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                  uint32_t r[16], r2[16];
                  tmem_ld16(oAddr + h2 * 32, r);
                  tmem_ld16(oAddr + h2 * 32 + 16, r2);
                  tmem_ld_wait(r, r2);
#pragma unroll
                  for (int i = 0; i < 16; ++i) {
                    r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                    r2[i] = __float_as_uint(__uint_as_float(r2[i]) * alpha);
                  }
                  tmem_st16(oAddr + h2 * 32, r);
                  tmem_st16(oAddr + h2 * 32 + 16, r2);
                }
                tmem_st_wait();
              }
              l *= alpha;
              m = m_new;
            }
            const float mc = (m == -INFINITY) ? 0.f : m * c;
            half_pass<T, 2>(sAddr, c_hi, c_full, khi, c, mc, unused, sum2, sAddr, pk0, pk1);
          }
          l += sum2.x + sum2.y;
          tmem_st_wait();
        }
        ++used;
        tc_fence_before();
        mbar_arrive(&p_full[w]);
      }
      if (!ok) break;
      // merge the two halves: exchange m and l with the other half's warp
      float* ml = s_ml + (((mlc & 1) * 2 + w) * 2) * 256;  // [half][m, l][128]
      ml[hf * 256 + row] = m;
      ml[hf * 256 + 128 + row] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(mlb);
      if (!mbar_wait<false>(mlb, mlc & 1, kErrTimeoutAttnO, abort_flag)) break;
      ++mlc;
      const float m0 = ml[row], m1 = ml[256 + row];
      const float mm = fmaxf(m0, m1);
      const float a0 = m0 == -INFINITY ? 0.f : fast_exp2((m0 - mm) * c);
      const float a1 = m1 == -INFINITY ? 0.f : fast_exp2((m1 - mm) * c);
      const float lt = ml[128 + row] * a0 + ml[256 + 128 + row] * a1;
      // epilogue: both O halves complete after the pair's last P.V
      if (!mbar_wait<false>(&o_done[w], ocnt & 1, kErrTimeoutAttnO, abort_flag)) break;
      ++ocnt;
      tc_fence_after();
      if (warp_active) {
        float scale = lt > 0.f ? 1.f / lt : 0.f;
        const int head = w == 0 ? g.head : g.head2;
        if (valid && p.gates != nullptr) scale *= __ldg(p.gates + token * p.heads + head);
        const float s0 = a0 * scale, s1 = a1 * scale;
        // this warp writes output columns [32 hf, 32 hf + 32), 16 at a time
        uint4* out = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.out) + token * p.out_ld + head * 64 + hf * 32);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t r0[16], r1[16];
          tmem_ld16(oBase + hf * 32 + hh * 16, r0);
          tmem_ld16(oBase + 64 + hf * 32 + hh * 16, r1);
          tmem_ld_wait(r0, r1);
          if (valid) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              if (hf * 32 + hh * 16 + 8 * u >= p.d_out) break;
              float v[8];
#pragma unroll
              for (int k = 0; k < 8; ++k)
                v[k] = __uint_as_float(r0[8 * u + k]) * s0 + __uint_as_float(r1[8 * u + k]) * s1;
              out[2 * hh + u] = make_uint4(pack2<T>(v[0], v[1]), pack2<T>(v[2], v[3]), pack2<T>(v[4], v[5]),
                                           pack2<T>(v[6], v[7]));
            }
          }
        }
      }
      tc_fence_before();
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T>
cudaError_t launch_t(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnParams& p,
                     int num_sms, cudaStream_t s) {
  static std::atomic<unsigned long long> configured[2];
  const bool band = p.mode == 1;
  cudaError_t e = band ? ensure_smem_limit(attention_band_kernel<T>, (int)kAttnSmem, configured[1])
                       : ensure_smem_limit(attention_time_kernel<T>, (int)kTimeSmem, configured[0]);
  if (e != cudaSuccess) return e;

  const int grid = p.total_items < num_sms ? p.total_items : num_sms;
  if (grid <= 0) return cudaSuccess;
  // algorithmic cost: QK^T and PV of every query row against its sequence's keys
  // (4 Nq Nk d FLOPs per head), Q/K/V and the gates read once, the output written once
  const double d = p.mode == 2 ? p.d_out : 64.0;
  const double qrows = (double)p.num_tokens * p.heads;                    // query rows x heads
  const double krows = qrows / p.seq_len * p.kv_len;                      // key rows x heads
  const double flop = 4.0 * qrows * p.kv_len * d;
  const double bytes = (2.0 * qrows + 2.0 * krows) * d * sizeof(T) + (p.gates ? 4.0 * qrows : 0.0);
  LaunchScope scope(p.mode == 0 ? "attention_time" : (p.mode == 1 ? "attention_band" : "attention_sdpa"), flop,
                    bytes, s);
  if (band)
    attention_band_kernel<T><<<grid, kThreads, kAttnSmem, s>>>(mq, mk, mv, p);
  else
    attention_time_kernel<T><<<grid, kTThreads, kTimeSmem, s>>>(mq, mk, mv, p);
  return cudaGetLastError();
}

cudaError_t launch_checked(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnParams& a,
                           int bf16, int num_sms, cudaStream_t stream) {
  if (a.q_tiles < 1) return cudaSuccess;
  return bf16 ? launch_t<__nv_bfloat16>(mq, mk, mv, a, num_sms, stream)
              : launch_t<__half>(mq, mk, mv, a, num_sms, stream);
}

}  // namespace

// Items of the time-axis schedule (see pair_geom): every unit's full pairs, plus one
// item per two units' tail tiles when q_tiles is odd.
static long long time_axis_items(long long units, int q_tiles) {
  return units * (q_tiles / 2) + ((q_tiles & 1) ? (units + 1) / 2 : 0);
}

cudaError_t launch_attention(const CUtensorMap& qkv_map, const AttnParams& p, int bf16, int num_sms,
                             cudaStream_t stream) {
  if (p.mode != 0 && p.mode != 1) return cudaErrorInvalidValue;
  if (p.mode == 1 && (p.seq_len < 1 || p.seq_len > 128 || p.seqs_per_tile != 128 / attn_band_slot(p.seq_len)))
    return cudaErrorInvalidValue;
  AttnParams a = p;
  const long long units = (long long)p.B * p.F * p.heads;
  const long long items =
      p.mode == 0 ? time_axis_items(units, p.q_tiles) : (long long)((p.q_tiles + 1) / 2) * p.heads;
  if (items > 0x7fffffffLL || units > 0x7fffffffLL) return cudaErrorInvalidValue;
  a.total_items = (int)items;
  a.units = (int)units;
  a.kv_len = p.seq_len;
  a.kv_tiles = p.q_tiles;
  a.k_col = p.heads * 64;
  a.v_col = 2 * p.heads * 64;
  a.out_ld = (long long)p.heads * 64;
  a.d_out = 64;
  return launch_checked(qkv_map, qkv_map, qkv_map, a, bf16, num_sms, stream);
}

cudaError_t launch_sdpa(const CUtensorMap& q_map, const CUtensorMap& k_map, const CUtensorMap& v_map,
                        const AttnParams& p, int bf16, int num_sms, cudaStream_t stream) {
  if (p.mode != 2 || p.F != 1 || p.heads != 1 || p.gates != nullptr) return cudaErrorInvalidValue;
  if (p.B < 1 || p.T < 1 || p.kv_len < 1 || p.seq_len != p.T) return cudaErrorInvalidValue;
  if (p.d_out < 8 || p.d_out > 64 || p.d_out % 8 != 0 || p.out_ld < p.d_out || p.out_ld % 8 != 0)
    return cudaErrorInvalidValue;
  if (p.q_tiles != (p.T + 127) / 128 || p.kv_tiles != (p.kv_len + 127) / 128) return cudaErrorInvalidValue;
  if ((long long)p.B * p.T != p.num_tokens) return cudaErrorInvalidValue;
  AttnParams a = p;
  const long long items = time_axis_items(p.B, p.q_tiles);
  if (items > 0x7fffffffLL) return cudaErrorInvalidValue;
  a.total_items = (int)items;
  a.units = p.B;
  a.k_col = a.v_col = 0;
  return launch_checked(q_map, k_map, v_map, a, bf16, num_sms, stream);
}

MSST_DEFINE_ERROR_ACCESSOR(attention_device_error)

}  // namespace msst
