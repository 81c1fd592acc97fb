// common.cuh — sm_100a building blocks shared by the kernels of libmsst_b200:
// mbarriers with bounded waits, TMA tiled loads, tcgen05 (UMMA) descriptors,
// MMA issue/commit and TMEM load/alloc.  Written for B200 (sm_100a) only.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <type_traits>

namespace msst {

// ---------------------------------------------------------------------------
// Device-side error reporting.  Every spin-wait in the library is bounded; a wait
// that gives up records a code here (first one wins) and the kernel unwinds.
// The host reads it with msst_device_error().
// ---------------------------------------------------------------------------
enum DeviceError : unsigned {
  kErrNone = 0,
  kErrTimeoutTmaFull = 1,
  kErrTimeoutSmemEmpty = 2,
  kErrTimeoutTmemFull = 3,
  kErrTimeoutTmemEmpty = 4,
  kErrTimeoutAttnS = 5,
  kErrTimeoutAttnP = 6,
  kErrTimeoutAttnO = 7,
  kErrTimeoutAttnQ = 8,
  kErrTimeoutAttnKV = 9,
  kErrTimeoutFfnS = 10,
  kErrTimeoutFfnP = 11,
  kErrTimeoutFfnO = 12,
  kErrTimeoutFfnFlag = 13,
};

// One flag per translation unit; each .cu exposes a host accessor (see
// MSST_DEFINE_ERROR_ACCESSOR) and the C ABI ORs them together.
static __device__ unsigned g_device_error = 0;

#define MSST_DEFINE_ERROR_ACCESSOR(fn)                                              \
  unsigned fn(bool clear) {                                                         \
    unsigned v = 0;                                                                 \
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return ~0u; \
    if (clear && v) {                                                               \
      unsigned z = 0;                                                               \
      cudaMemcpyToSymbol(g_device_error, &z, sizeof(z));                            \
    }                                                                               \
    return v;                                                                       \
  }

// Wall-clock limit for one mbarrier wait (ns).  Real waits in these kernels last
// microseconds; 2 s only trips on a genuine deadlock.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(unsigned code) { atomicCAS(&g_device_error, 0u, code); }

// Host: accounting of this library's kernel launches.  Each launcher opens a
// LaunchScope right before its <<<>>>: the scope counts the launch
// (msst_kernel_launches) and, while per-kernel timing is on (msst_kernel_timing),
// brackets it with two CUDA events on the launch stream and records the launch's
// algorithmic FLOPs and DRAM bytes under the kernel's name.
class LaunchScope {
 public:
  LaunchScope(const char* name, double flop, double bytes, cudaStream_t s);
  ~LaunchScope();
  LaunchScope(const LaunchScope&) = delete;
  LaunchScope& operator=(const LaunchScope&) = delete;

 private:
  long long slot_;
  cudaStream_t stream_;
};

// Host: raise a kernel's dynamic shared-memory limit on the current device.  The
// attribute is per device, so `done` keeps one bit per device; after the first call
// on a device this costs a cudaGetDevice and an atomic load.
template <typename K>
inline cudaError_t ensure_smem_limit(K kern, int bytes, std::atomic<unsigned long long>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One potentially blocking test of the phase.  kSuspend: the thread may be
// suspended until the phase completes or kSuspendHintNs pass, so a waiting warp
// does not take issue slots from the warps sharing its SM sub-partition (the
// GEMMs); without it the hardware's own short wait applies (the attention
// kernel, whose waits sit on its critical path: 1-3 % faster measured).
constexpr uint32_t kSuspendHintNs = 100000;
template <bool kSuspend = true>
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  if constexpr (kSuspend) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "n"(kSuspendHintNs)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
  }
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns false
// (after recording `code`) when the wall-clock limit passes or another thread of
// the CTA already gave up (*abort != 0).
template <bool kSuspend = true>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned code,
                                          volatile int* abort) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait<kSuspend>(a, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t spins = 1;; ++spins) {
    if (mbar_try_wait<kSuspend>(a, parity)) return true;
    if ((spins & 15u) == 0u) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        record_error(code);
        *abort = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), tiled mode, completion through an mbarrier.  No
// cluster multicast anywhere in this library.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

// Bulk tensor store / reduce-add shared -> global (tracked by the issuing
// thread's bulk async-groups).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   map),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The shared-memory sources of all committed bulk groups have been read.
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// All but the most recent committed bulk group have been read.
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
// All committed bulk groups have completed (writes performed).
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// A persistent CTA's share of a launch's work units, unit u = tile * J + j (j a
// hidden chunk, a head, ...): the contiguous range [U*c/G, U*(c+1)/G) for CTA c of
// G, so every CTA gets the same number of units give or take one, instead of whole
// tiles dealt in rounds of G (where the last round leaves most CTAs idle).  Walked
// in order as segments of one tile each: the tail [j_first, J) of the first tile,
// whole tiles, the head [0, j_last) of the last tile.
struct UnitRange {
  int J, count, nseg, t_first, t_last, j_first, j_last;
  __host__ __device__ __forceinline__ UnitRange(int ntiles, int J_, int c, int G) : J(J_) {
    const long long U = (long long)ntiles * J;
    const long long u0 = U * c / G, u1 = U * (c + 1) / G;
    count = (int)(u1 - u0);
    t_first = (int)(u0 / J);
    j_first = (int)(u0 % J);
    t_last = u1 > u0 ? (int)((u1 - 1) / J) : t_first;
    j_last = u1 > u0 ? (int)((u1 - 1) % J) + 1 : j_first;
    nseg = u1 > u0 ? t_last - t_first + 1 : 0;
  }
  // segment s: tile t, units [j0, j1)
  __host__ __device__ __forceinline__ void seg(int s, int& t, int& j0, int& j1) const {
    t = t_first + s;
    j0 = t == t_first ? j_first : 0;
    j1 = t == t_last ? j_last : J;
  }
};

// A flag word in global memory handed between CTAs of one grid (every CTA
// resident): the writer's earlier global writes, bulk (async-proxy) ones included
// once their groups have completed, are visible to a reader that saw the value.
__device__ __forceinline__ void flag_release(unsigned* f, unsigned v) {
  asm volatile("fence.proxy.async.global;" ::: "memory");
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}

// Bounded wait until *f == v (acquire); false after recording `code` when the
// wall-clock limit passes or another thread of the CTA gave up.
__device__ __forceinline__ bool flag_wait(const unsigned* f, unsigned v, unsigned code, volatile int* abort) {
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t spins = 0;; ++spins) {
    unsigned cur;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(cur) : "l"(f) : "memory");
    if (cur == v) {
      asm volatile("fence.proxy.async.global;" ::: "memory");
      return true;
    }
    if ((spins & 15u) == 15u) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        record_error(code);
        *abort = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 / UMMA
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor for a 128B-swizzled tile (SM100 format:
// start>>4 [0,14), LBO>>4 [16,30), SBO>>4 [32,46), version 1 [46,48),
// base offset 0, layout SWIZZLE_128B = 2 at [61,64)).  K-major tiles: rows of
// 128 B, 8-row groups SBO = 1024 B apart.  MN-major tiles (V in P.V): K rows of
// 128 B, 8-row groups SBO = 1024 B apart, LBO = next 64-element MN group.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulate, A/B fp16 (0) or bf16 (1),
// dense, M = 128 (256 for a CTA-pair MMA).  b_mn_major = 1 when B's N dimension
// is contiguous.
__host__ __device__ constexpr uint32_t umma_idesc_f16(uint32_t ab_bf16, uint32_t n, uint32_t b_mn_major = 0,
                                                      uint32_t m = 128) {
  return (1u << 4)                 // D format f32
         | (ab_bf16 << 7)          // A format
         | (ab_bf16 << 10)         // B format
         | (0u << 15)              // A K-major
         | (b_mn_major << 16)      // B major
         | ((n >> 3) << 17)        // N >> 3
         | ((m >> 4) << 24);       // M >> 4
}

__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D (+)= A . B with A read from TMEM (M rows in lanes, K 16-bit elements packed
// two per 32-bit column) and B from shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation issued so far by this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---------------------------------------------------------------- CTA pairs
// A cluster of two CTAs on neighbouring SMs runs one M = 256 MMA as a pair
// (tcgen05 cta_group::2): rank 0 issues the MMAs, each CTA supplies half of the A
// rows and half of the B rows from its own shared memory (same offsets in both)
// and receives its 128 accumulator rows in its own TMEM.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(addr), "r"(rank));
  return d;
}

// All threads of both CTAs: barrier across the cluster (release/acquire).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier given by its cluster address (possibly the peer CTA's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA load into this CTA's shared memory whose completion is counted on the
// pair leader's mbarrier (bar = its cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void umma_f16_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Completion of the pair's MMAs issued so far, signalled on the mbarrier at the
// same offset in every CTA of cta_mask.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Pair TMEM allocation: one warp of each CTA (same warp index, same dst offset).
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Warp-wide TMEM allocation; the base address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane
// (warp's quarter * 32 + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 16 consecutive 32-bit columns of this thread's TMEM lane (32x32b shape).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// tcgen05.wait::ld that also ties the destination registers of the preceding
// tcgen05.ld to the wait, so no use of them can be scheduled before it (the
// loads write their registers asynchronously).
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]),
        "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]),
        "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
        "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

// Wait for this thread's TMEM loads with two 16-register buffers tied to the wait, so
// that no use of them is scheduled before it.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[16], uint32_t (&s)[16]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]),
        "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(s[0]),
        "+r"(s[1]), "+r"(s[2]), "+r"(s[3]), "+r"(s[4]), "+r"(s[5]), "+r"(s[6]), "+r"(s[7]), "+r"(s[8]), "+r"(s[9]),
        "+r"(s[10]), "+r"(s[11]), "+r"(s[12]), "+r"(s[13]), "+r"(s[14]), "+r"(s[15])
      :
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit columns.
// No memory clobber: the data dependency is carried by the register operands,
// and the store stays ordered with tcgen05.wait::st and the other volatile
// tcgen05 statements, so independent arithmetic may be scheduled around it.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
}

// Make generic-proxy shared-memory writes visible to the async proxy (UMMA / TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Small numeric helpers
// ---------------------------------------------------------------------------
template <typename T>
struct Half2Of;
template <>
struct Half2Of<__half> {
  using type = __half2;
  static __device__ __forceinline__ __half2 pack(float a, float b) { return __floats2half2_rn(a, b); }
};
template <>
struct Half2Of<__nv_bfloat16> {
  using type = __nv_bfloat162;
  static __device__ __forceinline__ __nv_bfloat162 pack(float a, float b) { return __floats2bfloat162_rn(a, b); }
};

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  auto h = Half2Of<T>::pack(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

// Warpgroup register reallocation (every warp of the warpgroup executes it).  The
// shares of all warpgroups must add up to at most the block's launch allocation
// (threads x registers per thread at launch), or the increase never completes.
template <uint32_t N>
__device__ __forceinline__ void warpgroup_reg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void warpgroup_reg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// three-input maximum (PTX max.f32 with three sources, sm_100+)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^a for two lanes on the FMA and integer pipes instead of the MUFU unit, for
// a <= 2^21.  Range reduction: adding 1.5 * 2^23 rounds a to the integer n in the
// low mantissa bits of t, f = a - n lies in [-1/2, 1/2]; 2^f is a degree-3
// polynomial (relative-error minimax on [-1/2, 1/2] by Remez exchange, max
// relative error 7.5e-5, below half an fp16 ulp), and n is added to its
// exponent field by an integer shift-add (t's bits << 23 leave n * 2^23 modulo
// 2^32).  a is clamped at -125 so the exponent stays in the normal range;
// results there (< 2^-124) are far below the 16-bit P they feed.
__device__ __forceinline__ float2 poly_exp2x2(float2 a) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  a.x = fmaxf(a.x, -125.0f);
  a.y = fmaxf(a.y, -125.0f);
  const float2 mg = make_float2(kMagic, kMagic);
  const float2 t = __fadd2_rn(a, mg);
  const float2 neg_n = __ffma2_rn(t, make_float2(-1.0f, -1.0f), mg);
  const float2 f = __fadd2_rn(a, neg_n);
  float2 p = __ffma2_rn(make_float2(0.0551716685f, 0.0551716685f), f, make_float2(0.242611125f, 0.242611125f));
  p = __ffma2_rn(p, f, make_float2(0.693260968f, 0.693260968f));
  p = __ffma2_rn(p, f, make_float2(0.999928057f, 0.999928057f));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

}  // namespace msst
