// capi.cu — the extern "C" boundary of libmsst_b200 (declared in include/msst_b200.h).
// Every entry point catches exceptions and turns them into status codes; the
// message is kept per thread for msst_last_error().
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <string>
#include <utility>

#include "attention.cuh"
#include "gemm.cuh"
#include "kernels.cuh"
#include "model.h"
#include "runtime.h"

struct msst_model {
  msst::Model impl;
  // calls share the model's workspace: see serialized()
  std::mutex mu;
  cudaEvent_t done = nullptr;  // recorded at the end of every call
  cudaStream_t last = nullptr;  // stream of the previous call
  bool used = false;
};


namespace {

thread_local std::string g_last_error;

template <typename F>
int guarded(F&& f) {
  try {
    f();
    return MSST_OK;
  } catch (const msst::Error& e) {
    g_last_error = e.what();
    return e.code;
  } catch (const std::bad_alloc&) {
    g_last_error = "host out of memory";
    return MSST_ERR_CUDA;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return MSST_ERR_INVALID;
  }
}

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Makes `device` current for the scope of one entry point and restores the
// caller's current device on the way out, so a call on a model of another GPU
// leaves the host thread's device (which frameworks such as PyTorch read back
// for their next allocation) as it found it.
class DeviceScope {
 public:
  explicit DeviceScope(int device) {
    MSST_CUDA(cudaGetDevice(&prev_));
    if (prev_ != device) MSST_CUDA(cudaSetDevice(device));
    cur_ = device;
  }
  ~DeviceScope() {
    if (prev_ >= 0 && prev_ != cur_) cudaSetDevice(prev_);
  }
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;

 private:
  int prev_ = -1, cur_ = -1;
};

// A buffer handed to a model entry point must be device memory of the model's GPU
// (or managed memory): a kernel reading a host pointer or another GPU's memory
// without a peer mapping would fault, so such calls are refused up front.
void require_on_device(const void* p, int device, const char* what) {
  cudaPointerAttributes a{};
  MSST_CUDA(cudaPointerGetAttributes(&a, p));
  MSST_REQUIRE(a.type == cudaMemoryTypeManaged || (a.type == cudaMemoryTypeDevice && a.device == device),
               std::string(what) + " must be device memory on the model's GPU (" + std::to_string(device) + ")");
}

// The model-level calls of one msst_model share its workspace, so they run one
// host thread at a time, and a call on a different stream than the previous one
// first makes its stream wait (on the device) for the previous call's work.  The
// event is recorded even when the call fails part way, since some of its work may
// already be queued.  `buffers` are the call's device operands (null entries are
// skipped), checked against the model's device.
template <typename F>
void serialized(msst_model* m, cudaStream_t s, std::initializer_list<std::pair<const void*, const char*>> buffers,
                F&& f) {
  std::lock_guard<std::mutex> lock(m->mu);
  DeviceScope dev(m->impl.device());
  for (const auto& b : buffers)
    if (b.first) require_on_device(b.first, m->impl.device(), b.second);
  if (!m->done) MSST_CUDA(cudaEventCreateWithFlags(&m->done, cudaEventDisableTiming));
  if (m->used && s != m->last) MSST_CUDA(cudaStreamWaitEvent(s, m->done, 0));
  try {
    f();
  } catch (...) {
    if (cudaEventRecord(m->done, s) == cudaSuccess) {
      m->last = s;
      m->used = true;
    }
    throw;
  }
  MSST_CUDA(cudaEventRecord(m->done, s));
  m->last = s;
  m->used = true;
}

int sm_count() {
  static thread_local int dev = -1, n = 0;
  int d = 0;
  MSST_CUDA(cudaGetDevice(&d));
  if (d != dev) {
    dev = d;
    n = msst::device_sm_count();
  }
  return n;
}

int pick_bn(int n) {
  if (n % 256 == 0) return 256;
  if (n % 192 == 0) return 192;
  return n <= 128 ? 128 : 256;
}

void run_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, msst::GemmParams& p, int epi,
              int bn, int bf16, cudaStream_t s) {
  int tiles = 0;
  for (int i = 0; i < p.num_groups; ++i) {
    msst::GemmGroup& g = p.groups[i];
    g.tiles_n = (g.n + bn - 1) / bn;
    g.tile_begin = tiles;
    tiles += ((g.m + msst::kGemmBM - 1) / msst::kGemmBM) * g.tiles_n;
  }
  p.total_tiles = tiles;
  MSST_CUDA(msst::launch_gemm(ma, mb, mo, p, epi, bn, bf16, sm_count(), s));
}

void check_dtype(int dtype) { MSST_REQUIRE(dtype == MSST_F16 || dtype == MSST_BF16, "dtype must be MSST_F16 or MSST_BF16"); }

void check_align(const void* p, const char* what) {
  MSST_REQUIRE((reinterpret_cast<uintptr_t>(p) & 15) == 0, std::string(what) + " must be 16-byte aligned");
}

// Op-level entry points run on the device that owns their first operand (made
// current for the call's scope).
int device_of(const void* p) {
  cudaPointerAttributes a{};
  MSST_CUDA(cudaPointerGetAttributes(&a, p));
  MSST_REQUIRE(a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged, "operand is not device memory");
  if (a.type == cudaMemoryTypeDevice) return a.device;
  int cur = 0;
  MSST_CUDA(cudaGetDevice(&cur));
  return cur;
}

}  // namespace

extern "C" {

const char* msst_last_error(void) { return g_last_error.c_str(); }

unsigned msst_device_error(int clear) { return msst::device_error(clear != 0); }

int msst_version(void) { return 1; }

unsigned long long msst_kernel_launches(int reset) { return msst::launch_count(reset != 0); }

int msst_kernel_timing(int enable) {
  return guarded([&] { msst::set_kernel_timing(enable != 0); });
}

int msst_kernel_timing_report(msst_kernel_stat* out, int cap, int* count) {
  return guarded([&] {
    MSST_REQUIRE(count && (cap == 0 || out) && cap >= 0, "null argument");
    const auto stats = msst::kernel_timing_report();
    *count = (int)stats.size();
    for (int i = 0; i < cap && i < (int)stats.size(); ++i) {
      msst_kernel_stat& o = out[i];
      std::memset(o.name, 0, sizeof(o.name));
      std::strncpy(o.name, stats[i].name.c_str(), sizeof(o.name) - 1);
      o.launches = stats[i].launches;
      o.total_ms = stats[i].ms;
      o.flop = stats[i].flop;
      o.bytes = stats[i].bytes;
    }
  });
}

int msst_rmsnorm(const float* x, long long rows, int D, const float* gamma, float scale, int dtype, void* out16,
                 const float* wg, const float* bg, int heads, float* gates, void* stream) {
  return guarded([&] {
    check_dtype(dtype);
    MSST_REQUIRE(x && gamma && out16 && rows >= 0, "null argument");
    MSST_REQUIRE(D % 128 == 0 && D <= 1024, "D must be a multiple of 128 and <= 1024");
    MSST_REQUIRE(!wg || (bg && gates && heads > 0 && heads <= 32), "gate projection needs bg, gates, 0<heads<=32");
    check_align(x, "x");
    DeviceScope dev_scope(device_of(x));
    msst::RmsNormArgs a{};
    a.x = const_cast<float*>(x);
    a.rows = rows;
    a.D = D;
    a.gamma = gamma;
    a.scale = scale;
    a.out16 = out16;
    a.wg = wg;
    a.bg = bg;
    a.gates = gates;
    a.heads = heads;
    MSST_CUDA(msst::launch_rmsnorm(a, dtype, as_stream(stream)));
  });
}

int msst_gemm(const void* x, long long rows, int K, long long ldx, const void* w, int N, const float* bias,
              int epilogue, int act, int dtype, void* out, long long ldo, void* stream) {
  return guarded([&] {
    check_dtype(dtype);
    MSST_REQUIRE(x && w && out, "null argument");
    MSST_REQUIRE(rows > 0 && rows < (1LL << 31) && N > 0, "bad rows / N");
    MSST_REQUIRE(K > 0 && K % 64 == 0, "K must be a positive multiple of 64");
    MSST_REQUIRE(ldx >= K && (ldx * 2) % 16 == 0, "ldx must be >= K and a multiple of 8 elements");
    MSST_REQUIRE(epilogue >= MSST_EPI_STORE16 && epilogue <= MSST_EPI_GLU32, "bad epilogue");
    MSST_REQUIRE(act >= MSST_ACT_NONE && act <= MSST_ACT_SIGMOID, "bad activation");
    MSST_REQUIRE(epilogue != MSST_EPI_GLU32 || N % 2 == 0, "GLU needs an even N");
    check_align(x, "x");
    check_align(w, "w");
    check_align(out, "out");
    const bool out32 = epilogue != MSST_EPI_STORE16;
    MSST_REQUIRE(ldo >= (epilogue == MSST_EPI_GLU32 ? N / 2 : N) && (ldo * (out32 ? 4 : 2)) % 16 == 0,
                 "ldo must cover the output row and be a multiple of 16 bytes");
    DeviceScope dev_scope(device_of(x));
    const int bn = pick_bn(N);
    const CUtensorMap ma = msst::map_2d(x, (uint64_t)rows, (uint64_t)K, (uint64_t)ldx, msst::kGemmBM);
    const CUtensorMap mb = msst::map_gemm_b(w, (uint64_t)N, (uint64_t)K, (uint64_t)K, bn);
    const CUtensorMap mo = epilogue == MSST_EPI_GLU32
                               ? ma
                               : msst::map_out_2d(out, out32, (uint64_t)rows, (uint64_t)N, (uint64_t)ldo);
    msst::GemmParams p{};
    p.num_groups = 1;
    p.act = act;
    msst::GemmGroup& g = p.groups[0];
    g.m = (int)rows;
    g.n = N;
    g.k = K;
    g.out = out;
    g.ldo = ldo;
    g.out_row_mul = 1;
    g.oy_row = 1;
    g.bias = bias;
    run_gemm(ma, mb, mo, p, epilogue, bn, dtype, as_stream(stream));
  });
}

int msst_gemm_qkv_rope(const void* x, long long rows, int K, const void* w, int heads, const float* cos_tab,
                       const float* sin_tab, int pos_div, int pos_mod, int dtype, void* qkv16, void* stream) {
  return guarded([&] {
    check_dtype(dtype);
    MSST_REQUIRE(x && w && qkv16 && cos_tab && sin_tab, "null argument");
    MSST_REQUIRE(K > 0 && K % 64 == 0 && heads > 0 && pos_div > 0 && pos_mod > 0, "bad shape");
    check_align(x, "x");
    check_align(w, "w");
    DeviceScope dev_scope(device_of(x));
    const int N = 3 * heads * 64;
    const int bn = pick_bn(N);
    const CUtensorMap ma = msst::map_2d(x, (uint64_t)rows, (uint64_t)K, (uint64_t)K, msst::kGemmBM);
    const CUtensorMap mb = msst::map_gemm_b(w, (uint64_t)N, (uint64_t)K, (uint64_t)K, bn);
    msst::GemmParams p{};
    p.num_groups = 1;
    p.pos_div = pos_div;
    p.pos_mod = pos_mod;
    p.rope_cols = 2 * heads * 64;
    p.head_dim = 64;
    p.rope_cos = cos_tab;
    p.rope_sin = sin_tab;
    msst::GemmGroup& g = p.groups[0];
    g.m = (int)rows;
    g.n = N;
    g.k = K;
    g.out = qkv16;
    g.ldo = N;
    g.out_row_mul = 1;
    g.oy_row = 1;
    check_align(qkv16, "qkv16");
    const CUtensorMap mo = msst::map_out_2d(qkv16, false, (uint64_t)rows, (uint64_t)N, (uint64_t)N);
    run_gemm(ma, mb, mo, p, msst::kEpiQkvRope, bn, dtype, as_stream(stream));
  });
}

int msst_attention(const void* qkv16, int B, int T, int F, int heads, int axis, float scale, const float* gates,
                   int dtype, void* out16, void* stream) {
  return guarded([&] {
    check_dtype(dtype);
    MSST_REQUIRE(qkv16 && out16, "null argument");
    MSST_REQUIRE(B > 0 && T > 0 && F > 0 && heads > 0, "bad shape");
    MSST_REQUIRE(axis == MSST_AXIS_TIME || axis == MSST_AXIS_BAND, "bad axis");
    MSST_REQUIRE(axis == MSST_AXIS_TIME || F <= 128, "band axis supports at most 128 bands");
    check_align(qkv16, "qkv16");
    check_align(out16, "out16");
    DeviceScope dev_scope(device_of(qkv16));
    const long long M = (long long)B * T * F;
    MSST_REQUIRE(M < (1LL << 31), "too many tokens");
    const uint64_t C3 = 3ull * heads * 64;
    msst::AttnParams a{};
    a.mode = axis;
    a.B = B;
    a.T = T;
    a.F = F;
    a.heads = heads;
    a.num_tokens = (int)M;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.gates = gates;
    a.out = out16;
    CUtensorMap m;
    if (axis == MSST_AXIS_TIME) {
      a.seq_len = T;
      a.q_tiles = (T + 127) / 128;
      a.total_items = B * F * heads * a.q_tiles;
      const uint64_t dims[4] = {C3, (uint64_t)F, (uint64_t)T, (uint64_t)B};
      const uint64_t str[3] = {C3 * 2, C3 * 2 * F, C3 * 2 * F * T};
      const uint32_t box[4] = {64, 1, 128, 1};
      m = msst::make_tensor_map(qkv16, 4, dims, str, box);
    } else {
      a.seq_len = F;
      a.seqs_per_tile = 128 / msst::attn_band_slot(F);
      a.q_tiles = (int)(((long long)B * T + a.seqs_per_tile - 1) / a.seqs_per_tile);
      a.total_items = a.q_tiles * heads;
      const uint64_t dims[4] = {C3, (uint64_t)M, 1, 1};
      const uint64_t str[3] = {C3 * 2, C3 * 2 * M, C3 * 2 * M};
      const uint32_t box[4] = {64, (uint32_t)msst::attn_band_slot(F), 1, 1};
      m = msst::make_tensor_map(qkv16, 4, dims, str, box);
    }
    MSST_CUDA(msst::launch_attention(m, a, dtype, sm_count(), as_stream(stream)));
  });
}

int msst_layernorm(const float* x, long long rows, int D, const float* gamma, const float* beta, float eps,
                   int out_dtype, void* out, void* stream) {
  return guarded([&] {
    MSST_REQUIRE(out_dtype == MSST_F16 || out_dtype == MSST_BF16 || out_dtype == MSST_F32,
                 "out_dtype must be MSST_F16, MSST_BF16 or MSST_F32");
    MSST_REQUIRE(x && gamma && beta && out && rows >= 0, "null argument");
    MSST_REQUIRE(D >= 4 && D % 4 == 0 && D <= 1024, "D must be a multiple of 4 and <= 1024");
    MSST_REQUIRE(eps >= 0.f, "eps must be >= 0");
    check_align(x, "x");
    check_align(gamma, "gamma");
    check_align(beta, "beta");
    check_align(out, "out");
    if (rows == 0) return;
    DeviceScope dev_scope(device_of(x));
    msst::LayerNormArgs a{};
    a.x = x;
    a.rows = rows;
    a.D = D;
    a.gamma = gamma;
    a.beta = beta;
    a.eps = eps;
    a.out = out;
    a.out_kind = out_dtype == MSST_F32 ? 0 : (out_dtype == MSST_F16 ? 1 : 2);
    MSST_CUDA(msst::launch_layernorm(a, as_stream(stream)));
  });
}

int msst_sdpa(const void* q, const void* k, const void* v, int B, int H, int Nq, int Nk, int head_dim, float scale,
              int dtype, void* out, void* stream) {
  return guarded([&] {
    check_dtype(dtype);
    MSST_REQUIRE(q && k && v && out, "null argument");
    MSST_REQUIRE(B > 0 && H > 0 && Nq > 0 && Nk > 0, "bad shape");
    MSST_REQUIRE(head_dim >= 8 && head_dim <= 64 && head_dim % 8 == 0, "head_dim must be a multiple of 8, <= 64");
    MSST_REQUIRE(std::isfinite(scale), "scale must be finite");
    const long long BH = (long long)B * H;
    MSST_REQUIRE(BH * Nq < (1LL << 31) && BH * Nk < (1LL << 31), "too many rows");
    check_align(q, "q");
    check_align(k, "k");
    check_align(v, "v");
    check_align(out, "out");
    DeviceScope dev_scope(device_of(q));
    const float s = scale == 0.f ? 1.0f / std::sqrt((float)head_dim) : scale;
    msst::AttnParams a{};
    a.mode = 2;
    a.B = (int)BH;
    a.T = Nq;
    a.F = 1;
    a.heads = 1;
    a.seq_len = Nq;
    a.q_tiles = (Nq + 127) / 128;
    a.num_tokens = (int)(BH * Nq);
    a.kv_len = Nk;
    a.kv_tiles = (Nk + 127) / 128;
    a.out_ld = head_dim;
    a.d_out = head_dim;
    a.scale_log2 = s * 1.4426950408889634f;
    a.gates = nullptr;
    a.out = out;
    // {d, 1, N, B*H} with box {64, 1, 128, 1}: columns d..63 and rows past N read as zero
    auto seq_map = [&](const void* base, int n) {
      const uint64_t dims[4] = {(uint64_t)head_dim, 1, (uint64_t)n, (uint64_t)BH};
      const uint64_t str[3] = {(uint64_t)head_dim * 2, (uint64_t)head_dim * 2, (uint64_t)head_dim * 2 * n};
      const uint32_t box[4] = {64, 1, 128, 1};
      return msst::make_tensor_map(base, 4, dims, str, box);
    };
    const CUtensorMap mq = seq_map(q, Nq), mk = seq_map(k, Nk), mv = seq_map(v, Nk);
    MSST_CUDA(msst::launch_sdpa(mq, mk, mv, a, dtype, sm_count(), as_stream(stream)));
  });
}

int msst_grouped_gemm(int num_groups, const msst_gemm_group* groups, const void* x, long long x_rows, long long ldx,
                      const void* w, long long w_rows, long long ldw, int epilogue, int act, int dtype, void* out,
                      long long out_rows, long long ldo, void* stream) {
  return guarded([&] {
    check_dtype(dtype);
    MSST_REQUIRE(groups && x && w && out, "null argument");
    MSST_REQUIRE(num_groups >= 1 && num_groups <= msst::kGemmMaxGroups, "num_groups must be 1..64");
    MSST_REQUIRE(epilogue >= MSST_EPI_STORE16 && epilogue <= MSST_EPI_GLU32, "bad epilogue");
    MSST_REQUIRE(act >= MSST_ACT_NONE && act <= MSST_ACT_SIGMOID, "bad activation");
    MSST_REQUIRE(x_rows > 0 && x_rows < (1LL << 31) && w_rows > 0 && w_rows < (1LL << 31) && out_rows > 0 &&
                     out_rows < (1LL << 31),
                 "bad matrix row counts");
    MSST_REQUIRE(ldx >= 64 && ldx % 8 == 0 && ldw >= 64 && ldw % 8 == 0,
                 "ldx / ldw must be >= 64 and multiples of 8 elements");
    const bool out32 = epilogue != MSST_EPI_STORE16;
    const bool tma_out = epilogue != MSST_EPI_GLU32;
    const int col_align = out32 ? 4 : 8;  // TMA boxes start on 16 bytes
    MSST_REQUIRE(ldo > 0 && ldo % col_align == 0, "ldo must be a multiple of 16 bytes");
    check_align(x, "x");
    check_align(w, "w");
    check_align(out, "out");
    DeviceScope dev_scope(device_of(x));
    msst::GemmParams p{};
    p.num_groups = num_groups;
    p.act = act;
    int nmax = 0;
    for (int i = 0; i < num_groups; ++i) {
      const msst_gemm_group& q = groups[i];
      const std::string gi = "group " + std::to_string(i) + ": ";
      const long long nout = epilogue == MSST_EPI_GLU32 ? q.n / 2 : q.n;
      MSST_REQUIRE(q.m > 0 && q.n > 0 && q.k > 0 && q.k % 64 == 0, gi + "needs m, n > 0 and k a positive multiple of 64");
      MSST_REQUIRE(epilogue != MSST_EPI_GLU32 || q.n % 2 == 0, gi + "GLU needs an even n");
      MSST_REQUIRE(q.a_col0 % 8 == 0 && q.b_col0 % 8 == 0, gi + "a_col0 and b_col0 must be multiples of 8");
      MSST_REQUIRE(q.a_row0 >= 0 && q.a_row0 + q.m <= x_rows && q.a_col0 >= 0 && q.a_col0 + q.k <= ldx,
                   gi + "A slice outside x");
      MSST_REQUIRE(q.b_row0 >= 0 && q.b_row0 + q.n <= w_rows && q.b_col0 >= 0 && q.b_col0 + q.k <= ldw,
                   gi + "B slice outside W");
      MSST_REQUIRE(q.out_row0 >= 0 && q.out_row0 + q.m <= out_rows && q.out_col0 >= 0 && q.out_col0 + nout <= ldo,
                   gi + "output block outside out");
      if (tma_out) {
        MSST_REQUIRE(q.out_col0 % col_align == 0, gi + "out_col0 must start on 16 bytes");
        MSST_REQUIRE(q.m % 32 == 0 || q.out_row0 + q.m == out_rows,
                     gi + "m must be a multiple of 32 unless the block ends at out_rows");
        MSST_REQUIRE(q.n % 32 == 0 || q.out_col0 + q.n == ldo,
                     gi + "n must be a multiple of 32 unless the block ends at column ldo");
      }
      msst::GemmGroup& g = p.groups[i];
      g.m = (int)q.m;
      g.n = q.n;
      g.k = q.k;
      g.a_row0 = (int)q.a_row0;
      g.a_col0 = q.a_col0;
      g.b_row0 = q.b_row0;
      g.b_col0 = q.b_col0;
      g.out_col0 = q.out_col0;
      g.oy0 = (int)q.out_row0;
      g.oy_row = 1;
      g.out = out;
      g.ldo = ldo;
      g.out_row_mul = 1;
      g.out_row_add = q.out_row0;
      g.bias = q.bias;
      nmax = std::max(nmax, q.n);
    }
    const int bn = pick_bn(nmax);
    const CUtensorMap ma = msst::map_2d(x, (uint64_t)x_rows, (uint64_t)ldx, (uint64_t)ldx, msst::kGemmBM);
    const CUtensorMap mb = msst::map_gemm_b(w, (uint64_t)w_rows, (uint64_t)ldw, (uint64_t)ldw, bn);
    const CUtensorMap mo =
        tma_out ? msst::map_out_2d(out, out32, (uint64_t)out_rows, (uint64_t)ldo, (uint64_t)ldo) : ma;
    run_gemm(ma, mb, mo, p, epilogue, bn, dtype, as_stream(stream));
  });
}

int msst_band_gather(const float* spec, int B, int T, const msst_band_tables* t, int dtype, void* out16,
                     long long ldo, void* stream) {
  return guarded([&] {
    check_dtype(dtype);
    MSST_REQUIRE(spec && t && out16 && t->bin_start && t->nfreq && t->bin_list && t->kcol && t->kpad && t->gcol &&
                     t->gamma,
                 "null argument");
    MSST_REQUIRE(B > 0 && T > 0 && t->num_bands > 0 && t->nbins > 0 && t->channels > 0, "bad shape");
    MSST_REQUIRE(ldo >= t->sum_kpad && ldo % 8 == 0, "ldo must cover sum_kpad and be a multiple of 8");
    check_align(out16, "out16");
    DeviceScope dev_scope(device_of(spec));
    msst::BandInArgs bi{};
    bi.spec = reinterpret_cast<const float2*>(spec);
    bi.spec_scale = 1.0f;
    bi.Bc = B;
    bi.C = t->channels;
    bi.T = T;
    bi.nbins = t->nbins;
    bi.num_bands = t->num_bands;
    bi.bin_start = t->bin_start;
    bi.nfreq = t->nfreq;
    bi.bin_list = t->bin_list;
    bi.kcol = t->kcol;
    bi.kpad = t->kpad;
    bi.gcol = t->gcol;
    bi.gamma = t->gamma;
    bi.out = out16;
    bi.ld = ldo;
    MSST_CUDA(msst::launch_band_input(bi, dtype, as_stream(stream)));
  });
}

int msst_mask_apply(const float* spec, const float* masks, int B, int S, int T, const msst_band_tables* t, int zero_dc,
                    float* out, void* stream) {
  return guarded([&] {
    MSST_REQUIRE(spec && masks && t && out && t->contrib_off && t->contrib_col && t->denom, "null argument");
    MSST_REQUIRE(B > 0 && S > 0 && T > 0 && t->nbins > 0 && t->channels > 0 && t->sum_dims > 0, "bad shape");
    DeviceScope dev_scope(device_of(spec));
    msst::MaskApplyArgs ma{};
    ma.spec = reinterpret_cast<const float2*>(spec);
    ma.spec_scale = 1.0f;
    ma.out_scale = 1.0f;
    ma.mask = masks;
    ma.mask_stem_stride = (long long)B * T * t->sum_dims;
    ma.mask_ld = t->sum_dims;
    ma.contrib_off = t->contrib_off;
    ma.contrib_col = t->contrib_col;
    ma.denom = t->denom;
    ma.out = reinterpret_cast<float2*>(out);
    ma.Bc = B;
    ma.S = S;
    ma.C = t->channels;
    ma.T = T;
    ma.nbins = t->nbins;
    ma.zero_dc = zero_dc ? 1 : 0;
    MSST_CUDA(msst::launch_mask_apply(ma, as_stream(stream)));
  });
}

int msst_model_load(const char* path, int device, int precision, msst_model** out) {
  return guarded([&] {
    MSST_REQUIRE(path && out, "null argument");
    *out = nullptr;
    // the caller's current device, restored after the load (which makes `device`
    // current); a file error is reported as such even on a machine without a GPU
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) {
      prev = -1;
      cudaGetLastError();
    }
    auto* m = new msst_model();
    try {
      m->impl.load(path, device, precision);
    } catch (...) {
      delete m;
      if (prev >= 0) cudaSetDevice(prev);
      throw;
    }
    if (prev >= 0) cudaSetDevice(prev);
    *out = m;
  });
}

void msst_model_free(msst_model* m) {
  if (!m) return;
  try {
    DeviceScope dev(m->impl.device());
    if (m->done) cudaEventDestroy(m->done);
    delete m;
  } catch (...) {
    // the device could not be made current: release the host side only
    delete m;
  }
}

int msst_model_get_info(const msst_model* m, msst_model_info* info) {
  return guarded([&] {
    MSST_REQUIRE(m && info, "null argument");
    *info = m->impl.info();
  });
}

int msst_model_forward(msst_model* m, const float* audio, int batch, int channels, long long length, float* out,
                       void* stream) {
  return guarded([&] {
    MSST_REQUIRE(m && audio && out, "null argument");
    serialized(m, as_stream(stream), {{audio, "audio"}, {out, "out"}}, [&] { m->impl.forward(audio, batch, channels, length, out, as_stream(stream)); });
  });
}

int msst_model_masks(msst_model* m, const float* audio, int batch, int channels, long long length, float* masks,
                     void* stream) {
  return guarded([&] {
    MSST_REQUIRE(m && audio && masks, "null argument");
    serialized(m, as_stream(stream), {{audio, "audio"}, {masks, "masks"}}, [&] { m->impl.masks(audio, batch, channels, length, masks, as_stream(stream)); });
  });
}

int msst_model_transformer(msst_model* m, int depth_index, int axis, float* x, int batch, int T, void* stream) {
  return guarded([&] {
    MSST_REQUIRE(m && x, "null argument");
    serialized(m, as_stream(stream), {{x, "x"}}, [&] { m->impl.transformer(depth_index, axis, x, batch, T, as_stream(stream)); });
  });
}

int msst_roformer_attn_block(msst_model* m, int depth_index, int axis, int layer, float* x, int batch, int T,
                             void* stream) {
  return guarded([&] {
    MSST_REQUIRE(m && x, "null argument");
    serialized(m, as_stream(stream), {{x, "x"}}, [&] {
      m->impl.attn_block(depth_index, axis, layer, x, batch, T, as_stream(stream));
    });
  });
}

int msst_roformer_ffn_block(msst_model* m, int depth_index, int axis, int layer, float* x, int batch, int T,
                            void* stream) {
  return guarded([&] {
    MSST_REQUIRE(m && x, "null argument");
    serialized(m, as_stream(stream), {{x, "x"}}, [&] {
      m->impl.ffn_block(depth_index, axis, layer, x, batch, T, as_stream(stream));
    });
  });
}

int msst_model_band_tables(const msst_model* m, msst_band_tables* tables) {
  return guarded([&] {
    MSST_REQUIRE(m && tables, "null argument");
    m->impl.band_tables(tables);
  });
}

int msst_model_transformer_noalloc(msst_model* m, int depth_index, int axis, float* x, int batch, int T,
                                   void* stream) {
  return guarded([&] {
    MSST_REQUIRE(m && x, "null argument");
    serialized(m, as_stream(stream), {{x, "x"}}, [&] {
      m->impl.transformer_noalloc(depth_index, axis, x, batch, T, as_stream(stream));
    });
  });
}

int msst_model_separate(msst_model* m, const float* track, int channels, long long length, float overlap,
                        int chunk_batch, int flags, float* out, void* stream) {
  return guarded([&] {
    MSST_REQUIRE(m && track && out, "null argument");
    serialized(m, as_stream(stream), {{track, "track"}, {out, "out"}}, [&] {
      m->impl.separate(track, channels, length, overlap, chunk_batch, flags, out, as_stream(stream));
    });
  });
}

int msst_model_separate_host(msst_model* m, const float* track_host, int channels, long long length, float overlap,
                             int chunk_batch, int flags, float* out_host) {
  return guarded([&] {
    MSST_REQUIRE(m && track_host && out_host && channels > 0 && length > 0, "null argument");
    serialized(m, m->impl.host_stream(), {}, [&] {
      m->impl.separate_host(track_host, channels, length, overlap, chunk_batch, flags, out_host);
    });
  });
}

int msst_model_forward_chunks(msst_model* m, const float* track, int channels, long long length, float overlap,
                              int first_chunk, int count, int chunk_batch, int flags, float* out, void* stream) {
  return guarded([&] {
    MSST_REQUIRE(m && track && (out || count == 0), "null argument");
    serialized(m, as_stream(stream), {{track, "track"}, {out, "out"}}, [&] {
      m->impl.forward_chunks(track, channels, length, overlap, first_chunk, 1, count, chunk_batch, flags, out,
                             as_stream(stream));
    });
  });
}

int msst_model_forward_chunks_strided(msst_model* m, const float* track, int channels, long long length,
                                      float overlap, int first_chunk, int chunk_stride, int count, int chunk_batch,
                                      int flags, float* out, void* stream) {
  return guarded([&] {
    MSST_REQUIRE(m && track && (out || count == 0), "null argument");
    serialized(m, as_stream(stream), {{track, "track"}, {out, "out"}}, [&] {
      m->impl.forward_chunks(track, channels, length, overlap, first_chunk, chunk_stride, count, chunk_batch, flags,
                             out, as_stream(stream));
    });
  });
}

int msst_model_stitch_range(msst_model* m, const float* chunks, int slot_ranks, int slot_cap, int channels,
                            long long length, float overlap, long long begin, long long end, float* out,
                            void* stream) {
  return guarded([&] {
    MSST_REQUIRE(m && chunks && out, "null argument");
    serialized(m, as_stream(stream), {{chunks, "chunks"}, {out, "out"}}, [&] {
      m->impl.stitch_range(chunks, slot_ranks, slot_cap, channels, length, overlap, begin, end, out,
                           as_stream(stream));
    });
  });
}

int msst_model_chunk_span(const msst_model* m, long long length, float overlap, int chunk_index, int flags,
                          long long* in_ranges, long long* out_begin, long long* out_end) {
  return guarded([&] {
    MSST_REQUIRE(m && in_ranges && out_begin && out_end, "null argument");
    m->impl.chunk_span(length, overlap, chunk_index, flags, in_ranges, out_begin, out_end);
  });
}

int msst_model_stitch(msst_model* m, const float* chunks, int channels, long long length, float overlap, float* out,
                      void* stream) {
  return guarded([&] {
    MSST_REQUIRE(m && chunks && out, "null argument");
    serialized(m, as_stream(stream), {{chunks, "chunks"}, {out, "out"}}, [&] {
      m->impl.stitch(chunks, channels, length, overlap, out, as_stream(stream));
    });
  });
}

int msst_model_chunk_plan(const msst_model* m, long long length, float overlap, int* chunk_size, int* step,
                          long long* border, long long* padded_length, int* num_chunks) {
  return guarded([&] {
    MSST_REQUIRE(m && chunk_size && step && border && padded_length && num_chunks, "null argument");
    m->impl.chunk_plan(length, overlap, chunk_size, step, border, padded_length, num_chunks);
  });
}

}  // extern "C"
