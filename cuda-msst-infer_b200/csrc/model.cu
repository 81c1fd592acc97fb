// model.cu — Roformer model driver: .csm loading, weight packing for the
// tcgen05 kernels, forward pass and chunked separation.
#include "model.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <thread>
#include <cstring>
#include <fstream>

#include "attention.cuh"
#include "kernels.cuh"

namespace msst {

// ===========================================================================
// Minimal JSON (objects, arrays, numbers, strings, booleans, null) for the
// config block of a .csm file (the reference parses it with its own
// JsonValue, src/weights.h:18-78).
// ===========================================================================
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;

  const Json* find(const std::string& k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
  bool has(const std::string& k) const { return find(k) != nullptr; }
  int get_int(const std::string& k, int def) const {
    const Json* v = find(k);
    return (v && v->kind == Num) ? (int)v->num : def;
  }
  bool get_bool(const std::string& k, bool def) const {
    const Json* v = find(k);
    if (!v) return def;
    if (v->kind == Bool) return v->b;
    if (v->kind == Num) return v->num != 0;
    return def;
  }
  std::string get_str(const std::string& k, const std::string& def) const {
    const Json* v = find(k);
    return (v && v->kind == Str) ? v->str : def;
  }
};

class JsonParser {
 public:
  explicit JsonParser(const std::string& s) : s_(s) {}
  Json parse() {
    Json v = value();
    ws();
    return v;
  }

 private:
  const std::string& s_;
  size_t i_ = 0;
  [[noreturn]] void bad() { fail(MSST_ERR_IO, "malformed JSON config at offset " + std::to_string(i_)); }
  void ws() {
    while (i_ < s_.size() && std::isspace((unsigned char)s_[i_])) ++i_;
  }
  char peek() {
    ws();
    return i_ < s_.size() ? s_[i_] : '\0';
  }
  void expect(char c) {
    if (peek() != c) bad();
    ++i_;
  }
  std::string string_lit() {
    expect('"');
    std::string out;
    while (i_ < s_.size() && s_[i_] != '"') {
      char c = s_[i_++];
      if (c == '\\') {
        if (i_ >= s_.size()) bad();
        char e = s_[i_++];
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (i_ + 4 > s_.size()) bad();
            unsigned cp = std::stoul(s_.substr(i_, 4), nullptr, 16);
            i_ += 4;
            if (cp < 0x80) {
              out += (char)cp;
            } else if (cp < 0x800) {
              out += (char)(0xC0 | (cp >> 6));
              out += (char)(0x80 | (cp & 0x3F));
            } else {
              out += (char)(0xE0 | (cp >> 12));
              out += (char)(0x80 | ((cp >> 6) & 0x3F));
              out += (char)(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: out += e;
        }
      } else {
        out += c;
      }
    }
    if (i_ >= s_.size()) bad();
    ++i_;
    return out;
  }
  Json value() {
    Json v;
    char c = peek();
    if (c == '{') {
      ++i_;
      v.kind = Json::Obj;
      if (peek() == '}') {
        ++i_;
        return v;
      }
      for (;;) {
        std::string k = string_lit();
        expect(':');
        v.obj.emplace_back(k, value());
        if (peek() == ',') {
          ++i_;
          continue;
        }
        expect('}');
        return v;
      }
    }
    if (c == '[') {
      ++i_;
      v.kind = Json::Arr;
      if (peek() == ']') {
        ++i_;
        return v;
      }
      for (;;) {
        v.arr.push_back(value());
        if (peek() == ',') {
          ++i_;
          continue;
        }
        expect(']');
        return v;
      }
    }
    if (c == '"') {
      v.kind = Json::Str;
      v.str = string_lit();
      return v;
    }
    if (s_.compare(i_, 4, "true") == 0) {
      i_ += 4;
      v.kind = Json::Bool;
      v.b = true;
      return v;
    }
    if (s_.compare(i_, 5, "false") == 0) {
      i_ += 5;
      v.kind = Json::Bool;
      return v;
    }
    if (s_.compare(i_, 4, "null") == 0) {
      i_ += 4;
      return v;
    }
    size_t end = i_;
    while (end < s_.size() && (std::isdigit((unsigned char)s_[end]) || std::strchr("+-.eE", s_[end]))) ++end;
    if (end == i_) bad();
    v.kind = Json::Num;
    v.num = std::stod(s_.substr(i_, end - i_));
    i_ = end;
    return v;
  }
};

// ===========================================================================
// .csm container (reference src/weights.h:83-96): magic "CSM\0", u32 version 1,
// u32 config length + JSON, u32 tensor count, then per tensor: u32 name
// length + name, u32 ndim, i64 shape[ndim], u32 dtype (0 f32, 1 f16, 2 i64),
// raw row-major data.
// ===========================================================================
struct HostTensor {
  std::vector<int64_t> shape;
  int dtype = 0;
  const uint8_t* data = nullptr;
  size_t numel = 1;

  std::vector<float> f32() const {
    std::vector<float> out(numel);
    if (dtype == 0) {
      std::memcpy(out.data(), data, numel * 4);
    } else if (dtype == 1) {
      const __half* h = reinterpret_cast<const __half*>(data);
      for (size_t i = 0; i < numel; ++i) out[i] = __half2float(h[i]);
    } else {
      const int64_t* q = reinterpret_cast<const int64_t*>(data);
      for (size_t i = 0; i < numel; ++i) out[i] = (float)q[i];
    }
    return out;
  }
  std::vector<int64_t> i64() const {
    std::vector<int64_t> out(numel);
    if (dtype == 2) {
      std::memcpy(out.data(), data, numel * 8);
    } else {
      std::vector<float> f = f32();
      for (size_t i = 0; i < numel; ++i) out[i] = (int64_t)std::llround(f[i]);
    }
    return out;
  }
};

struct Csm {
  std::vector<uint8_t> bytes;
  Json config;
  std::unordered_map<std::string, HostTensor> tensors;

  const HostTensor& get(const std::string& name) const {
    auto it = tensors.find(name);
    if (it == tensors.end()) fail(MSST_ERR_IO, "tensor not found in .csm: " + name);
    return it->second;
  }
  bool has(const std::string& name) const { return tensors.count(name) > 0; }
};

static Csm read_csm(const std::string& path) {
  Csm c;
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  if (!f) fail(MSST_ERR_IO, "cannot open " + path);
  const std::streamsize size = f.tellg();
  f.seekg(0);
  c.bytes.resize((size_t)size);
  if (!f.read(reinterpret_cast<char*>(c.bytes.data()), size)) fail(MSST_ERR_IO, "cannot read " + path);
  size_t off = 0;
  auto need = [&](size_t n) {
    if (off + n > c.bytes.size()) fail(MSST_ERR_IO, "truncated .csm file: " + path);
  };
  auto u32 = [&]() {
    need(4);
    uint32_t v;
    std::memcpy(&v, c.bytes.data() + off, 4);
    off += 4;
    return v;
  };
  need(4);
  if (std::memcmp(c.bytes.data(), "CSM\0", 4) != 0) fail(MSST_ERR_IO, "invalid magic (expected CSM\\0): " + path);
  off = 4;
  const uint32_t version = u32();
  if (version != 1) fail(MSST_ERR_IO, "unsupported .csm version " + std::to_string(version));
  const uint32_t clen = u32();
  need(clen);
  std::string cj(reinterpret_cast<const char*>(c.bytes.data() + off), clen);
  off += clen;
  c.config = JsonParser(cj).parse();
  const uint32_t n = u32();
  for (uint32_t t = 0; t < n; ++t) {
    const uint32_t nl = u32();
    need(nl);
    std::string name(reinterpret_cast<const char*>(c.bytes.data() + off), nl);
    off += nl;
    HostTensor ht;
    const uint32_t nd = u32();
    ht.shape.resize(nd);
    for (uint32_t d = 0; d < nd; ++d) {
      need(8);
      std::memcpy(&ht.shape[d], c.bytes.data() + off, 8);
      off += 8;
      ht.numel *= (size_t)ht.shape[d];
    }
    ht.dtype = (int)u32();
    if (ht.dtype < 0 || ht.dtype > 2) fail(MSST_ERR_IO, "unknown dtype for tensor " + name);
    const size_t esz = ht.dtype == 0 ? 4 : (ht.dtype == 1 ? 2 : 8);
    need(ht.numel * esz);
    ht.data = c.bytes.data() + off;
    off += ht.numel * esz;
    c.tensors.emplace(std::move(name), std::move(ht));
  }
  return c;
}

// ===========================================================================
// Upload helpers.  During Model::load an Uploader stages every tensor through
// two pinned host buffers: the values are converted (to the 16-bit operand type
// where the kernels read 16-bit) by all host threads straight into one buffer
// while the other is copied to the device with cudaMemcpyAsync, so conversion
// and DMA overlap (the reference converts and uploads tensor by tensor from
// pageable memory, src/weights.cu:412-524).  Outside load (tables built on first
// use) the helpers copy synchronously.
// ===========================================================================
static void to16(const float* src, size_t n, uint16_t* dst, int bf16) {
  for (size_t i = 0; i < n; ++i) {
    if (bf16) {
      __nv_bfloat16 h = __float2bfloat16_rn(src[i]);
      std::memcpy(dst + i, &h, 2);
    } else {
      __half h = __float2half_rn(src[i]);
      std::memcpy(dst + i, &h, 2);
    }
  }
}

// fn(begin, end) over [0, n) on up to `threads` host threads (inline when small)
template <typename F>
static void parallel_range(size_t n, unsigned threads, F&& fn) {
  if (n < (1u << 18) || threads <= 1) {
    fn((size_t)0, n);
    return;
  }
  std::vector<std::thread> pool;
  const size_t per = (n + threads - 1) / threads;
  for (unsigned t = 0; t < threads; ++t) {
    const size_t b = t * per, e = std::min(n, b + per);
    if (b >= e) break;
    pool.emplace_back([&fn, b, e] { fn(b, e); });
  }
  for (auto& th : pool) th.join();
}

class Uploader {
 public:
  Uploader() {
    threads_ = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    MSST_CUDA(cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking));
    for (int i = 0; i < 2; ++i) {
      MSST_CUDA(cudaMallocHost(&buf_[i], kStage));
      MSST_CUDA(cudaEventCreateWithFlags(&ev_[i], cudaEventDisableTiming));
    }
  }
  ~Uploader() {
    cudaStreamSynchronize(st_);
    for (int i = 0; i < 2; ++i) {
      if (buf_[i]) cudaFreeHost(buf_[i]);
      if (ev_[i]) cudaEventDestroy(ev_[i]);
    }
    if (st_) cudaStreamDestroy(st_);
  }
  Uploader(const Uploader&) = delete;
  Uploader& operator=(const Uploader&) = delete;

  // copy `bytes` to dst; fill(staging, first element, element count) writes the
  // values of elements [first, first + count) (esize bytes each) into staging
  template <typename Fill>
  void put(void* dst, size_t count, size_t esize, Fill&& fill) {
    const size_t per = kStage / esize;
    for (size_t off = 0; off < count; off += per) {
      const size_t n = std::min(per, count - off);
      MSST_CUDA(cudaEventSynchronize(ev_[cur_]));  // the DMA that last read this buffer is done
      uint8_t* stg = buf_[cur_];
      parallel_range(n, threads_, [&](size_t b, size_t e) { fill(stg + b * esize, off + b, e - b); });
      MSST_CUDA(cudaMemcpyAsync(static_cast<uint8_t*>(dst) + off * esize, stg, n * esize, cudaMemcpyHostToDevice,
                                st_));
      MSST_CUDA(cudaEventRecord(ev_[cur_], st_));
      cur_ ^= 1;
    }
  }
  void finish() { MSST_CUDA(cudaStreamSynchronize(st_)); }

 private:
  static constexpr size_t kStage = 32ull << 20;
  cudaStream_t st_ = nullptr;
  uint8_t* buf_[2] = {nullptr, nullptr};
  cudaEvent_t ev_[2] = {nullptr, nullptr};
  int cur_ = 0;
  unsigned threads_ = 1;
};

thread_local Uploader* t_uploader = nullptr;  // set while Model::load runs on this thread

static DeviceBuffer upload_raw(const void* src, size_t count, size_t esize) {
  DeviceBuffer b(std::max<size_t>(count, 1) * esize);
  if (count == 0) return b;
  if (t_uploader) {
    const uint8_t* s8 = static_cast<const uint8_t*>(src);
    t_uploader->put(b.get(), count, esize,
                    [&](uint8_t* d, size_t first, size_t n) { std::memcpy(d, s8 + first * esize, n * esize); });
  } else {
    MSST_CUDA(cudaMemcpy(b.get(), src, count * esize, cudaMemcpyHostToDevice));
  }
  return b;
}

static DeviceBuffer upload_f32(const std::vector<float>& v) { return upload_raw(v.data(), v.size(), 4); }

static DeviceBuffer upload_i32(const std::vector<int>& v) { return upload_raw(v.data(), v.size(), 4); }

static DeviceBuffer upload_16(const std::vector<float>& v, int bf16) {
  DeviceBuffer b(std::max<size_t>(v.size(), 1) * 2);
  if (v.empty()) return b;
  if (t_uploader) {
    t_uploader->put(b.get(), v.size(), 2, [&](uint8_t* d, size_t first, size_t n) {
      to16(v.data() + first, n, reinterpret_cast<uint16_t*>(d), bf16);
    });
  } else {
    std::vector<uint16_t> h(v.size());
    to16(v.data(), v.size(), h.data(), bf16);
    MSST_CUDA(cudaMemcpy(b.get(), h.data(), h.size() * 2, cudaMemcpyHostToDevice));
  }
  return b;
}

// ===========================================================================
// Workspace for one (batch, T) shape
// ===========================================================================
struct Model::Work {
  int B = 0, T = 0;
  long long M = 0, BT = 0;
  DeviceBuffer frames, spec, ispec, abs, x, xn, gates, big1, big2, ao, mask;
  DeviceBuffer skips;  // skip_connection models: the outputs of depth blocks 0..depth-2
  // fused feed-forward: split-tile flags (8 words per CTA) and the launch counter
  // whose value marks them (launches on one workspace are stream-ordered)
  DeviceBuffer ffn_flags;
  unsigned ffn_epoch = 0;
  CUtensorMap m_abs, m_xn, m_ao, m_big1_ffh, m_big2_ffh, m_qkv_time, m_qkv_band, m_h1, m_h2;
  CUtensorMap m_xn_slot;  // xn in boxes of one band sequence's slot (band_attn.cu)
  // GEMM output maps (TMA stores)
  CUtensorMap mo_qkv, mo_ffh, mo_bs, mo_h1, mo_h2;
};

Model::Model() = default;

Model::~Model() {
  for (auto& kv : plans_) cufftDestroy(kv.second);
  if (host_stream_) cudaStreamDestroy(host_stream_);
  for (cudaStream_t st : copy_streams_)
    if (st) cudaStreamDestroy(st);
  for (cudaEvent_t e : events_) cudaEventDestroy(e);
}

// ===========================================================================
// load
// ===========================================================================
void Model::load(const std::string& path, int device, int precision) {
  const auto t_load0 = std::chrono::steady_clock::now();
  MSST_REQUIRE(precision == MSST_F16 || precision == MSST_BF16, "precision must be MSST_F16 or MSST_BF16");
  device_ = device;
  bf16_ = precision;
  Csm csm = read_csm(path);
  MSST_CUDA(cudaSetDevice(device));
  Uploader uploader;
  struct Scope {
    Uploader* prev;
    explicit Scope(Uploader* u) : prev(t_uploader) { t_uploader = u; }
    ~Scope() { t_uploader = prev; }
  } scope(&uploader);
  num_sms_ = device_sm_count();
  const Json& j = csm.config;

  // model type detection as src/inference_app.cpp:77-98 (Roformers only)
  const std::string mt = j.get_str("model_type", "");
  if (mt == "mel_band_roformer" || mt == "MelBandRoformer")
    mel_ = true;
  else if (mt == "bs_roformer" || mt == "BSRoformer")
    mel_ = false;
  else if (j.has("num_bands") || j.has("mel_scale"))
    mel_ = true;
  else if (j.has("freqs_per_bands"))
    mel_ = false;
  else
    fail(MSST_ERR_UNSUPPORTED, "not a MelBandRoformer / BSRoformer model (conv models stay on the reference path)");

  // config with the reference defaults (src/model_mel_band_roformer.cu:185-208, src/model_bs_roformer.cu:26-59)
  msst_model_info& I = info_;
  I.model_type = mel_ ? 1 : 2;
  I.dim = j.get_int("dim", 384);
  I.depth = j.get_int("depth", mel_ ? 6 : 12);
  const bool stereo = j.get_bool("stereo", true);
  I.num_stems = j.get_int("num_stems", 1);
  const int tdepth = j.get_int("time_transformer_depth", 1);
  const int fdepth = j.get_int("freq_transformer_depth", 1);
  I.dim_head = j.get_int("dim_head", 64);
  I.heads = j.get_int("heads", 8);
  const int me_depth = j.get_int("mask_estimator_depth", mel_ ? 2 : 1);
  const int mlp_mult = j.get_int("mlp_expansion_factor", 4);
  zero_dc_ = j.get_bool("zero_dc", true);
  I.sample_rate = j.get_int("sample_rate", 44100);
  I.n_fft = j.get_int("stft_n_fft", 2048);
  I.hop_length = j.get_int("stft_hop_length", 441);
  const int win_len = j.get_int("stft_win_length", 2048);
  I.chunk_size = j.get_int("chunk_size", I.n_fft * 256);
  I.num_overlap = j.has("num_overlap") ? std::max(1, j.get_int("num_overlap", 2)) : 2;
  I.precision = precision;
  stft_norm_ = j.get_bool("stft_normalized", false);
  skip_ = j.get_bool("skip_connection", false);
  match_len_ = j.get_bool("match_input_audio_length", false);
  I.stft_normalized = stft_norm_;
  I.skip_connection = skip_;
  I.match_input_audio_length = match_len_;
  if (I.dim_head != 64) fail(MSST_ERR_UNSUPPORTED, "dim_head must be 64");
  if (win_len != I.n_fft) fail(MSST_ERR_UNSUPPORTED, "stft_win_length must equal stft_n_fft");
  if (I.n_fft & (I.n_fft - 1)) fail(MSST_ERR_UNSUPPORTED, "stft_n_fft must be a power of two");
  if (I.dim % 128 != 0 || I.dim > 1024) fail(MSST_ERR_UNSUPPORTED, "dim must be a multiple of 128 (<= 1024)");
  C_ = stereo ? 2 : 1;
  I.channels = C_;
  nbins_ = I.n_fft / 2 + 1;
  inner_ = I.heads * I.dim_head;
  ff_ = I.dim * mlp_mult;
  hid_ = I.dim * mlp_mult;
  n_lin_ = mel_ ? me_depth + 1 : me_depth;
  MSST_REQUIRE(n_lin_ >= 1, "mask_estimator_depth must be >= 1");

  // ---- bands
  nfreq_.clear();
  bin_list_.clear();
  std::vector<float> denom(nbins_, 1.0f);
  if (mel_ && csm.has("__precomputed__.freq_indices")) {
    const std::vector<int64_t> fi = csm.get("__precomputed__.freq_indices").i64();
    const std::vector<int64_t> nf = csm.get("__precomputed__.num_freqs_per_band").i64();
    const std::vector<int64_t> nb = csm.get("__precomputed__.num_bands_per_freq").i64();
    I.num_bands = j.get_int("num_bands", (int)nf.size());
    I.bands_from_file = 1;
    MSST_REQUIRE((int)nf.size() == I.num_bands, "num_freqs_per_band length != num_bands");
    size_t k = 0;
    for (int b = 0; b < I.num_bands; ++b) {
      nfreq_.push_back((int)nf[b]);
      for (int64_t q = 0; q < nf[b]; ++q, ++k) {
        MSST_REQUIRE(k * C_ < fi.size(), "freq_indices too short");
        const int64_t v = fi[k * C_];
        MSST_REQUIRE(v % C_ == 0 && v / C_ < nbins_, "freq_indices not channel-interleaved");
        bin_list_.push_back((int)(v / C_));
      }
    }
    MSST_REQUIRE((int)nb.size() == nbins_, "num_bands_per_freq length != n_fft/2+1");
    for (int f = 0; f < nbins_; ++f) denom[f] = std::max((float)nb[f], 1e-8f);
  } else if (mel_) {
    // no precomputed tables in the file: derive them at load, as the reference does
    I.num_bands = j.get_int("num_bands", 60);
    I.bands_from_file = 0;
    mel_bands_from_filterbank(denom);
  } else {
    const Json* fpb = j.find("freqs_per_bands");
    MSST_REQUIRE(fpb && fpb->kind == Json::Arr, "BSRoformer config lacks freqs_per_bands");
    I.bands_from_file = 1;
    int start = 0;
    for (auto& v : fpb->arr) {
      nfreq_.push_back((int)v.num);
      for (int q = 0; q < (int)v.num; ++q) bin_list_.push_back(start + q);
      start += (int)v.num;
    }
    I.num_bands = (int)nfreq_.size();
    MSST_REQUIRE(start == nbins_, "sum(freqs_per_bands) != n_fft/2+1");
  }
  const int nb = I.num_bands;
  MSST_REQUIRE(nb <= kGemmMaxGroups, "too many bands for one grouped GEMM");
  MSST_REQUIRE(nb <= 128, "band-axis attention supports up to 128 bands");
  bin_start_.assign(nb, 0);
  dims_.assign(nb, 0);
  kpad_.assign(nb, 0);
  kcol_.assign(nb, 0);
  dim_off_.assign(nb, 0);
  out3_off_.assign(nb, 0);
  ktot_ = sum_dims_ = sum_out3_ = 0;
  for (int b = 0, s = 0; b < nb; ++b) {
    bin_start_[b] = s;
    s += nfreq_[b];
    dims_[b] = 2 * C_ * nfreq_[b];
    kpad_[b] = (dims_[b] + 63) / 64 * 64;
    kcol_[b] = ktot_;
    ktot_ += kpad_[b];
    dim_off_[b] = sum_dims_;
    sum_dims_ += dims_[b];
    out3_off_[b] = sum_out3_;
    sum_out3_ += 2 * dims_[b];
  }
  I.sum_band_dims = sum_dims_;
  // contributions of every band to every bin (deterministic gather form of the scatter_add)
  std::vector<std::vector<int>> contrib(nbins_);
  for (int b = 0; b < nb; ++b)
    for (int q = 0; q < nfreq_[b]; ++q) contrib[bin_list_[bin_start_[b] + q]].push_back(dim_off_[b] + q * 2 * C_);
  std::vector<int> coff(nbins_ + 1, 0), ccol;
  for (int f = 0; f < nbins_; ++f) {
    coff[f + 1] = coff[f] + (int)contrib[f].size();
    ccol.insert(ccol.end(), contrib[f].begin(), contrib[f].end());
  }
  d_nfreq_ = upload_i32(nfreq_);
  d_bin_start_ = upload_i32(bin_start_);
  d_bin_list_ = upload_i32(bin_list_);
  d_kpad_ = upload_i32(kpad_);
  d_kcol_ = upload_i32(kcol_);
  d_gcol_ = upload_i32(dim_off_);
  {
    // bands whose bins are an ascending run are contiguous spans of a staged STFT row
    std::vector<int> rf(nb, -1);
    for (int b = 0; b < nb; ++b) {
      const int* bl = bin_list_.data() + bin_start_[b];
      bool run = true;
      for (int q = 1; q < nfreq_[b]; ++q) run = run && bl[q] == bl[0] + q;
      if (run && nfreq_[b] > 0) rf[b] = bl[0];
    }
    d_run_first_ = upload_i32(rf);
  }
  d_contrib_off_ = upload_i32(coff);
  d_contrib_col_ = upload_i32(ccol);
  d_denom_ = upload_f32(denom);
  {
    // per-bin summary for the mask merge: the (at most two) contributions and the count
    std::vector<int> pack(4 * (size_t)nbins_);
    for (int f = 0; f < nbins_; ++f) {
      const int n = coff[f + 1] - coff[f];
      int* e = pack.data() + 4 * (size_t)f;
      e[0] = n <= 2 ? (n >= 1 ? ccol[coff[f]] : -1) : -2;
      e[1] = n == 2 ? ccol[coff[f] + 1] : -1;
      e[2] = 0;
      std::memcpy(&e[3], &denom[f], 4);
    }
    d_bin_pack_ = upload_i32(pack);
  }

  // ---- window (periodic Hann, src/ops_stft.cu:253-259)
  {
    std::vector<float> w(I.n_fft);
    for (int i = 0; i < I.n_fft; ++i) w[i] = 0.5f * (1.0f - std::cos(2.0f * (float)M_PI * (float)i / (float)I.n_fft));
    window_ = upload_f32(w);
  }

  const int D = I.dim;
  auto mat = [&](const std::string& name, int rows, int cols) {
    const HostTensor& t = csm.get(name);
    MSST_REQUIRE(t.shape.size() == 2 && t.shape[0] == rows && t.shape[1] == cols, "unexpected shape for " + name);
    return t.f32();
  };
  auto vec = [&](const std::string& name, int n) {
    const HostTensor& t = csm.get(name);
    MSST_REQUIRE((int)t.numel == n, "unexpected size for " + name);
    return t.f32();
  };

  // ---- band split: all bands in one [D, Ktot] matrix, band b at columns kcol[b] (zero padded)
  {
    std::vector<float> W((size_t)D * ktot_, 0.f), bias((size_t)nb * D), gam(sum_dims_);
    for (int b = 0; b < nb; ++b) {
      const std::string p = "band_split.to_features." + std::to_string(b);
      std::vector<float> g = vec(p + ".0.gamma", dims_[b]);
      std::copy(g.begin(), g.end(), gam.begin() + dim_off_[b]);
      std::vector<float> w = mat(p + ".1.weight", D, dims_[b]);
      for (int r = 0; r < D; ++r)
        std::copy(w.begin() + (size_t)r * dims_[b], w.begin() + (size_t)(r + 1) * dims_[b],
                  W.begin() + (size_t)r * ktot_ + kcol_[b]);
      std::vector<float> bb = vec(p + ".1.bias", D);
      std::copy(bb.begin(), bb.end(), bias.begin() + (size_t)b * D);
    }
    w_bs_ = upload_16(W, bf16_);
    b_bs_ = upload_f32(bias);
    g_bs_ = upload_f32(gam);
    m_wbs_ = map_gemm_b(w_bs_.get(), D, ktot_, ktot_, gemm_pick_bn(D));
  }

  // ---- transformers
  blocks_.clear();
  blocks_.resize(I.depth);
  for (int d = 0; d < I.depth; ++d) {
    for (int axis = 0; axis < 2; ++axis) {
      TransformerWeights& tw = axis == 0 ? blocks_[d].first : blocks_[d].second;
      const std::string tp = "layers." + std::to_string(d) + "." + std::to_string(axis);
      const int nl = axis == 0 ? tdepth : fdepth;
      tw.layers.resize(nl);
      for (int l = 0; l < nl; ++l) {
        LayerWeights& L = tw.layers[l];
        const std::string ap = tp + ".layers." + std::to_string(l) + ".0";
        const std::string fp = tp + ".layers." + std::to_string(l) + ".1.net";
        L.g_attn = upload_f32(vec(ap + ".norm.gamma", D));
        L.wqkv = upload_16(mat(ap + ".to_qkv.weight", 3 * inner_, D), bf16_);
        L.wg = upload_f32(mat(ap + ".to_gates.weight", I.heads, D));
        L.bg = upload_f32(vec(ap + ".to_gates.bias", I.heads));
        L.wout = upload_16(mat(ap + ".to_out.0.weight", D, inner_), bf16_);
        L.g_ff = upload_f32(vec(fp + ".0.gamma", D));
        L.w1 = upload_16(mat(fp + ".1.weight", ff_, D), bf16_);
        L.b1 = upload_f32(vec(fp + ".1.bias", ff_));
        L.w2 = upload_16(mat(fp + ".4.weight", D, ff_), bf16_);
        L.b2 = upload_f32(vec(fp + ".4.bias", D));
        L.bn_qkv = gemm_pick_bn(3 * inner_);
        L.bn_out = gemm_pick_bn(D);
        L.bn_w1 = gemm_pick_bn(ff_);
        L.bn_w2 = gemm_pick_bn(D);
        L.m_wqkv = map_gemm_b(L.wqkv.get(), 3 * inner_, D, D, L.bn_qkv);
        L.m_wout = map_gemm_b(L.wout.get(), D, inner_, inner_, L.bn_out);
        L.m_w1 = map_gemm_b(L.w1.get(), ff_, D, D, L.bn_w1);
        L.m_w2 = map_gemm_b(L.w2.get(), D, ff_, ff_, L.bn_w2);
        L.m_w1_f = map_2d(L.w1.get(), ff_, D, D, 128);
        L.m_wqkv64 = map_2d(L.wqkv.get(), 3 * inner_, D, D, 64);
        L.m_w2_f = map_2d(L.w2.get(), D, ff_, ff_, 128);
      }
      if (mel_) tw.g_final = upload_f32(vec(tp + ".norm.gamma", D));
    }
  }
  if (!mel_) final_norm_ = upload_f32(vec("final_norm.gamma", D));

  // ---- mask estimators: layer i of every band stacked along rows; the last
  // layer's rows interleaved (value_j, gate_j) so the GLU pair is adjacent
  stems_.clear();
  stems_.resize(I.num_stems);
  for (int s = 0; s < I.num_stems; ++s) {
    StemWeights& sw = stems_[s];
    for (int i = 0; i < n_lin_; ++i) {
      const bool last = i == n_lin_ - 1;
      const int K = i == 0 ? D : hid_;
      const int rows_total = last ? sum_out3_ : nb * hid_;
      std::vector<float> W((size_t)rows_total * K), bias(rows_total);
      for (int b = 0; b < nb; ++b) {
        const std::string p =
            "mask_estimators." + std::to_string(s) + ".to_freqs." + std::to_string(b) + ".0." + std::to_string(2 * i);
        const int n_out = last ? 2 * dims_[b] : hid_;
        std::vector<float> w = mat(p + ".weight", n_out, K);
        std::vector<float> bb = vec(p + ".bias", n_out);
        const size_t row0 = last ? (size_t)out3_off_[b] : (size_t)b * hid_;
        for (int r = 0; r < n_out; ++r) {
          // GLU: first half = value, second half = gate (src/ops_elementwise.cu:321-343)
          const int dst = last ? (r < dims_[b] ? 2 * r : 2 * (r - dims_[b]) + 1) : r;
          std::copy(w.begin() + (size_t)r * K, w.begin() + (size_t)(r + 1) * K, W.begin() + (row0 + dst) * K);
          bias[row0 + dst] = bb[r];
        }
      }
      sw.w.push_back(upload_16(W, bf16_));
      sw.b.push_back(upload_f32(bias));
      sw.m.push_back(map_gemm_b(sw.w.back().get(), rows_total, K, K, 256));
    }
  }
  uploader.finish();
  if (!host_stream_) MSST_CUDA(cudaStreamCreateWithFlags(&host_stream_, cudaStreamNonBlocking));
  MSST_CUDA(cudaDeviceSynchronize());
  info_.load_ms =
      (float)std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t_load0).count();
}

// MelBandRoformer band tables for a .csm without __precomputed__ tensors.  The
// reference then builds them itself (src/model_mel_band_roformer.cu:214-313,
// taken at :377) from its HTK-scale triangular filterbank (ops::mel_filterbank,
// src/ops_misc.cu:469-525): num_bands + 2 points evenly spaced on the mel scale
// m(f) = 2595 log10(1 + f / 700) between 0 Hz and sr / 2, FFT bin i at
// sr * i / n_fft Hz, band b's triangle rising from point b to point b + 1 and
// falling to point b + 2; filter [0][0] and [last][last] forced to 1; bin i
// belongs to band b where the filter value is > 0.  The arithmetic is fp32 in the
// same order as the reference's, since band membership is decided by exact
// comparisons.
void Model::mel_bands_from_filterbank(std::vector<float>& denom) {
  const msst_model_info& I = info_;
  const int nb = I.num_bands;
  MSST_REQUIRE(nb >= 1, "num_bands must be >= 1");
  const float f_hi = (float)I.sample_rate / 2.0f;
  const auto to_mel = [](float f) { return 2595.0f * std::log10(1.0f + f / 700.0f); };
  const auto to_hz = [](float m) { return 700.0f * (std::pow(10.0f, m / 2595.0f) - 1.0f); };
  const float m_lo = to_mel(0.0f), m_hi = to_mel(f_hi);
  std::vector<float> edge(nb + 2);
  for (int i = 0; i < nb + 2; ++i) edge[i] = to_hz(m_lo + (m_hi - m_lo) * (float)i / (float)(nb + 1));
  std::vector<int> count(nbins_, 0);
  for (int b = 0; b < nb; ++b) {
    const float lo = edge[b], mid = edge[b + 1], hi = edge[b + 2];
    int n = 0;
    for (int f = 0; f < nbins_; ++f) {
      const float hz = (float)I.sample_rate * (float)f / (float)I.n_fft;
      float v = 0.0f;
      if (hz >= lo && hz <= mid) {
        if (mid - lo > 0.0f) v = (hz - lo) / (mid - lo);
      } else if (hz > mid && hz <= hi) {
        if (hi - mid > 0.0f) v = (hi - hz) / (hi - mid);
      }
      if ((b == 0 && f == 0) || (b == nb - 1 && f == nbins_ - 1)) v = 1.0f;
      if (v > 0.0f) {
        bin_list_.push_back(f);
        ++count[f];
        ++n;
      }
    }
    MSST_REQUIRE(n > 0, "mel band " + std::to_string(b) + " covers no FFT bin");
    nfreq_.push_back(n);
  }
  for (int f = 0; f < nbins_; ++f) denom[f] = std::max((float)count[f], 1e-8f);
}

// ===========================================================================
// helpers
// ===========================================================================
const float* Model::rope_table(int n, bool sine) {
  auto& tab = sine ? rope_sin_ : rope_cos_;
  auto it = tab.find(n);
  if (it != tab.end()) return it->second.get<float>();
  // src/model_mel_band_roformer.cu:487-513 (fp32 on the host)
  const int half = info_.dim_head / 2;
  std::vector<float> c((size_t)n * half), s((size_t)n * half);
  for (int p = 0; p < n; ++p)
    for (int i = 0; i < half; ++i) {
      const float freq = 1.0f / std::pow(10000.0f, (float)(2 * i) / (float)info_.dim_head);
      const float ang = (float)p * freq;
      c[(size_t)p * half + i] = std::cos(ang);
      s[(size_t)p * half + i] = std::sin(ang);
    }
  rope_cos_[n] = upload_f32(c);
  rope_sin_[n] = upload_f32(s);
  return (sine ? rope_sin_[n] : rope_cos_[n]).get<float>();
}

const float* Model::istft_wsum(int T) {
  auto it = wsum_.find(T);
  if (it != wsum_.end()) return it->second.get<float>();
  const int n = info_.n_fft, hop = info_.hop_length;
  const size_t full = (size_t)n + (size_t)(T - 1) * hop;
  std::vector<float> w(n), ws(full, 0.f);
  for (int i = 0; i < n; ++i) w[i] = 0.5f * (1.0f - std::cos(2.0f * (float)M_PI * (float)i / (float)n));
  for (int t = 0; t < T; ++t)
    for (int i = 0; i < n; ++i) ws[(size_t)t * hop + i] += w[i] * w[i];
  wsum_[T] = upload_f32(ws);
  return wsum_[T].get<float>();
}

cufftHandle Model::fft_plan(cufftType type, int batch, cudaStream_t s) {
  auto key = std::make_pair((int)type, batch);
  auto it = plans_.find(key);
  cufftHandle h;
  if (it == plans_.end()) {
    int n = info_.n_fft;
    cufftResult r;
    if (type == CUFFT_R2C)
      r = cufftPlanMany(&h, 1, &n, nullptr, 1, n, nullptr, 1, nbins_, CUFFT_R2C, batch);
    else
      r = cufftPlanMany(&h, 1, &n, nullptr, 1, nbins_, nullptr, 1, n, CUFFT_C2R, batch);
    if (r != CUFFT_SUCCESS) fail(MSST_ERR_CUDA, "cufftPlanMany failed (" + std::to_string((int)r) + ")");
    plans_[key] = h;
  } else {
    h = it->second;
  }
  if (cufftSetStream(h, s) != CUFFT_SUCCESS) fail(MSST_ERR_CUDA, "cufftSetStream failed");
  return h;
}

void Model::gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, GemmParams& p, int epi, int bn,
                 cudaStream_t s) {
  int tiles = 0;
  for (int i = 0; i < p.num_groups; ++i) {
    GemmGroup& g = p.groups[i];
    g.tiles_n = (g.n + bn - 1) / bn;
    g.tile_begin = tiles;
    tiles += ((g.m + kGemmBM - 1) / kGemmBM) * g.tiles_n;
  }
  p.total_tiles = tiles;
  MSST_CUDA(launch_gemm(ma, mb, mo, p, epi, bn, bf16_, num_sms_, s));
}

static GemmGroup group(int m, int n, int k, void* out, long long ldo, const float* bias) {
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
}

Model::Work& Model::work(int B, int T) {
  auto key = std::make_pair(B, T);
  auto it = work_.find(key);
  if (it != work_.end()) return *it->second;
  auto w = std::make_unique<Work>();
  const msst_model_info& I = info_;
  const int nb = I.num_bands, D = I.dim, S = I.num_stems;
  w->B = B;
  w->T = T;
  w->BT = (long long)B * T;
  w->M = w->BT * nb;
  const long long M = w->M;
  w->frames.reset(sizeof(float) * (size_t)std::max(B * C_, B * S * C_) * T * I.n_fft);
  w->spec.reset(sizeof(float2) * (size_t)B * C_ * T * nbins_);
  w->ispec.reset(sizeof(float2) * (size_t)B * S * C_ * T * nbins_);
  w->abs.reset(2 * (size_t)w->BT * ktot_);
  w->x.reset(4 * (size_t)M * D);
  w->xn.reset(2 * (size_t)M * D);
  w->gates.reset(4 * (size_t)M * I.heads);
  const size_t big = std::max({(size_t)M * 3 * inner_, (size_t)M * ff_, (size_t)M * hid_});
  w->big1.reset(2 * big);
  w->big2.reset(2 * big);
  w->ao.reset(2 * (size_t)M * inner_);
  w->mask.reset(4 * (size_t)S * w->BT * sum_dims_);
  if (skip_ && I.depth > 1) w->skips.reset(4 * (size_t)(I.depth - 1) * M * D);
  w->ffn_flags.reset(4 * 8 * (size_t)num_sms_);
  MSST_CUDA(cudaMemset(w->ffn_flags.get(), 0, 4 * 8 * (size_t)num_sms_));
  w->m_abs = map_2d(w->abs.get(), w->BT, ktot_, ktot_, kGemmBM);
  w->m_xn = map_2d(w->xn.get(), M, D, D, kGemmBM);
  w->m_xn_slot = map_2d(w->xn.get(), M, D, D, (uint32_t)attn_band_slot(nb));
  w->m_ao = map_2d(w->ao.get(), M, inner_, inner_, kGemmBM);
  w->m_big2_ffh = map_2d(w->big2.get(), M, ff_, ff_, kGemmBM);
  w->m_h1 = map_2d(w->big1.get(), M, hid_, hid_, kGemmBM);
  w->m_h2 = map_2d(w->big2.get(), M, hid_, hid_, kGemmBM);
  w->mo_qkv = map_out_2d(w->big1.get(), false, M, 3 * inner_, 3 * inner_);
  w->mo_ffh = map_out_2d(w->big2.get(), false, M, ff_, ff_);
  // band split writes row (bt*nb + band) of the residual stream: view x as {D, nb, BT}
  w->mo_bs = map_out(w->x.get(), true, D, nb, w->BT, D, (uint64_t)nb * D, /*rows_along_z=*/true);
  // mask-estimator hidden layers: {hid, BT, nb} so every band's rows clip at BT
  w->mo_h1 = map_out(w->big1.get(), false, hid_, w->BT, nb, hid_, (uint64_t)w->BT * hid_);
  w->mo_h2 = map_out(w->big2.get(), false, hid_, w->BT, nb, hid_, (uint64_t)w->BT * hid_);
  {
    const uint64_t C3 = 3 * (uint64_t)inner_;
    const uint64_t dims[4] = {C3, (uint64_t)nb, (uint64_t)T, (uint64_t)B};
    const uint64_t str[3] = {C3 * 2, C3 * 2 * nb, C3 * 2 * nb * T};
    const uint32_t box[4] = {64, 1, 128, 1};
    w->m_qkv_time = make_tensor_map(w->big1.get(), 4, dims, str, box);
    const uint64_t dims2[4] = {C3, (uint64_t)M, 1, 1};
    const uint64_t str2[3] = {C3 * 2, C3 * 2 * M, C3 * 2 * M};
    const uint32_t box2[4] = {64, (uint32_t)attn_band_slot(nb), 1, 1};
    w->m_qkv_band = make_tensor_map(w->big1.get(), 4, dims2, str2, box2);
  }
  Work& ref = *w;
  work_[key] = std::move(w);
  return ref;
}

// ===========================================================================
// forward pieces
// ===========================================================================
void Model::run_front(const float* audio, const ChunkSource& src, int B, long long L, int T, cudaStream_t s,
                      Work& w) {
  const msst_model_info& I = info_;
  // STFT (src/ops_stft.cu:286-365) -> [B*C*T, nbins] complex; chunks are framed straight
  // from the track (the gathered chunk batch is never written)
  if (src.chunks)
    MSST_CUDA(launch_stft_frames_chunks(*src.chunks, src.first, src.stride, B, T, I.n_fft, I.hop_length,
                                        window_.get<float>(), w.frames.get<float>(), s));
  else
    MSST_CUDA(launch_stft_frames(audio, L, B * C_, T, I.n_fft, I.hop_length, window_.get<float>(),
                                 w.frames.get<float>(), s));
  if (cufftExecR2C(fft_plan(CUFFT_R2C, B * C_ * T, s), w.frames.get<cufftReal>(), w.spec.get<cufftComplex>()) !=
      CUFFT_SUCCESS)
    fail(MSST_ERR_CUDA, "cufftExecR2C failed");
  // band gather + per-band RMSNorm -> A of the band-split GEMM
  BandInArgs bi{};
  bi.spec = w.spec.get<float2>();
  bi.Bc = B;
  bi.C = C_;
  bi.T = T;
  bi.nbins = nbins_;
  bi.num_bands = I.num_bands;
  bi.bin_start = d_bin_start_.get<int>();
  bi.nfreq = d_nfreq_.get<int>();
  bi.bin_list = d_bin_list_.get<int>();
  bi.kcol = d_kcol_.get<int>();
  bi.kpad = d_kpad_.get<int>();
  bi.gcol = d_gcol_.get<int>();
  bi.gamma = g_bs_.get<float>();
  bi.out = w.abs.get();
  bi.ld = ktot_;
  bi.spec_scale = stft_norm_ ? 1.0f / std::sqrt((float)I.n_fft) : 1.0f;
  bi.run_first = d_run_first_.get<int>();
  MSST_CUDA(launch_band_input(bi, bf16_, s));
  // band split: one group per band, output rows (bt*nb + band) of the residual stream
  GemmParams p{};
  p.num_groups = I.num_bands;
  for (int b = 0; b < I.num_bands; ++b) {
    GemmGroup g = group((int)w.BT, I.dim, kpad_[b], w.x.get(), I.dim, b_bs_.get<float>() + (size_t)b * I.dim);
    g.a_col0 = kcol_[b];
    g.b_col0 = kcol_[b];
    g.oy0 = b;
    g.oy_row = 0;
    g.oz_row = 1;
    p.groups[b] = g;
  }
  gemm(w.m_abs, m_wbs_, w.mo_bs, p, kEpiStore32, gemm_pick_bn(I.dim), s);
}

void Model::run_transformer(int d, int axis, float* x, int B, int T, const float* pending_gamma, cudaStream_t s,
                            Work& w) {
  const TransformerWeights& tw = axis == 0 ? blocks_[d].first : blocks_[d].second;
  for (int l = 0; l < (int)tw.layers.size(); ++l) {
    run_attn_block(d, axis, l, x, B, T, l == 0 ? pending_gamma : nullptr, s, w);
    run_ffn_block(d, axis, l, x, B, T, s, w);
  }
}

// src/model_mel_band_roformer.cu:519-591 (apply_attention) + residual
void Model::run_attn_block(int d, int axis, int l, float* x, int B, int T, const float* pending_gamma, cudaStream_t s,
                           Work& w) {
  const msst_model_info& I = info_;
  const int D = I.dim, nb = I.num_bands;
  const TransformerWeights& tw = axis == 0 ? blocks_[d].first : blocks_[d].second;
  const LayerWeights& L = tw.layers[l];
  const long long M = (long long)B * T * nb;
  const float scale = std::sqrt((float)D);
  const CUtensorMap mo_x = map_out_2d(x, true, M, D, D);  // residual reduce-add target
  // attention pre-norm (+ pending final norm of the previous transformer) + gates
  RmsNormArgs rn{};
  rn.x = x;
  rn.rows = M;
  rn.D = D;
  rn.gamma_pre = pending_gamma;
  rn.scale_pre = scale;
  rn.gamma = L.g_attn.get<float>();
  rn.scale = scale;
  rn.out16 = w.xn.get();
  rn.wg = L.wg.get<float>();
  rn.bg = L.bg.get<float>();
  rn.gates = w.gates.get<float>();
  rn.heads = I.heads;
  MSST_CUDA(launch_rmsnorm(rn, bf16_, s));
  if (axis == 1 && band_fused_ok()) {
    // band axis: QKV projection, rotary, attention, gates and head merge in one kernel
    BandAttnParams bp{};
    bp.num_seqs = (int)w.BT;
    bp.F = nb;
    bp.slot = attn_band_slot(nb);
    bp.D = D;
    bp.heads = I.heads;
    bp.inner = inner_;
    bp.scale_log2 = (1.0f / std::sqrt((float)I.dim_head)) * 1.4426950408889634f;
    bp.rope_cos = rope_table(nb, false);
    bp.rope_sin = rope_table(nb, true);
    bp.gates = w.gates.get<float>();
    bp.out = w.ao.get();
    bp.out_ld = inner_;
    MSST_CUDA(launch_band_attention_fused(w.m_xn_slot, L.m_wqkv64, bp, bf16_, num_sms_, s));
  } else {
  // QKV + RoPE
  {
    GemmParams p{};
    p.num_groups = 1;
    p.groups[0] = group((int)M, 3 * inner_, D, w.big1.get(), 3 * inner_, nullptr);
    p.rope_cols = 2 * inner_;
    p.head_dim = I.dim_head;
    if (axis == 0) {
      p.pos_div = nb;
      p.pos_mod = T;
    } else {
      p.pos_div = 1;
      p.pos_mod = nb;
    }
    p.rope_cos = rope_table(p.pos_mod, false);
    p.rope_sin = rope_table(p.pos_mod, true);
    gemm(w.m_xn, L.m_wqkv, w.mo_qkv, p, kEpiQkvRope, L.bn_qkv, s);
  }
  // attention (+ gate, head merge)
  {
    AttnParams a{};
    a.mode = axis;
    a.B = B;
    a.T = T;
    a.F = nb;
    a.heads = I.heads;
    a.num_tokens = (int)M;
    a.scale_log2 = (1.0f / std::sqrt((float)I.dim_head)) * 1.4426950408889634f;
    a.gates = w.gates.get<float>();
    a.out = w.ao.get();
    if (axis == 0) {
      a.seq_len = T;
      a.q_tiles = (T + 127) / 128;
      a.total_items = B * nb * I.heads * a.q_tiles;
    } else {
      a.seq_len = nb;
      a.seqs_per_tile = 128 / attn_band_slot(nb);
      a.q_tiles = (int)((w.BT + a.seqs_per_tile - 1) / a.seqs_per_tile);
      a.total_items = a.q_tiles * I.heads;
    }
    MSST_CUDA(launch_attention(axis == 0 ? w.m_qkv_time : w.m_qkv_band, a, bf16_, num_sms_, s));
  }
  }
  // out projection + residual
  {
    GemmParams p{};
    p.num_groups = 1;
    p.groups[0] = group((int)M, D, inner_, x, D, nullptr);
    gemm(w.m_ao, L.m_wout, mo_x, p, kEpiResid32, L.bn_out, s);
  }
}

// src/model_mel_band_roformer.cu:597-622 (apply_feedforward) + residual
// Fused feed-forward when the model's widths allow it (dim a multiple of 128 up to 384,
// hidden a multiple of 128); MSST_FFN_FUSED=0 selects the two-GEMM path.
bool Model::ffn_fused_ok() const {
  static const int env = [] {
    const char* e = getenv("MSST_FFN_FUSED");
    return e ? atoi(e) : 1;
  }();
  return env != 0 && info_.dim % 128 == 0 && info_.dim <= 384 && ff_ % 128 == 0;
}

// Band-axis attention fused with its QKV projection (band_attn.cu) for sequences of
// up to 64 bands; MSST_BAND_FUSED=0 selects the QKV GEMM + attention kernel path.
bool Model::band_fused_ok() const {
  static const int env = [] {
    const char* e = getenv("MSST_BAND_FUSED");
    return e ? atoi(e) : 1;
  }();
  return env != 0 && info_.num_bands <= 64 && info_.dim <= 512 && info_.dim % 64 == 0 && info_.dim_head == 64;
}

void Model::run_ffn_block(int d, int axis, int l, float* x, int B, int T, cudaStream_t s, Work& w) {
  const msst_model_info& I = info_;
  const int D = I.dim, nb = I.num_bands;
  const TransformerWeights& tw = axis == 0 ? blocks_[d].first : blocks_[d].second;
  const LayerWeights& L = tw.layers[l];
  const long long M = (long long)B * T * nb;
  const CUtensorMap mo_x = map_out_2d(x, true, M, D, D);  // residual reduce-add target
  // feed-forward
  RmsNormArgs rf{};
  rf.x = x;
  rf.rows = M;
  rf.D = D;
  rf.gamma = L.g_ff.get<float>();
  rf.scale = std::sqrt((float)D);
  rf.out16 = w.xn.get();
  MSST_CUDA(launch_rmsnorm(rf, bf16_, s));
  if (ffn_fused_ok()) {
    // the hidden activation stays on chip (dim <= 384: S chunk + O fit TMEM)
    FfnParams fp{};
    fp.m = (int)M;
    fp.D = D;
    fp.H = ff_;
    fp.b1 = L.b1.get<float>();
    fp.b2 = L.b2.get<float>();
    fp.flags = w.ffn_flags.get<unsigned>();
    if (++w.ffn_epoch == 0) ++w.ffn_epoch;  // 0 is the buffer's initial value
    fp.epoch = w.ffn_epoch;
    MSST_CUDA(launch_ffn_fused(w.m_xn, L.m_w1_f, L.m_w2_f, mo_x, fp, bf16_, num_sms_, s));
    return;
  }
  {
    GemmParams p{};
    p.num_groups = 1;
    p.act = kActGelu;
    p.groups[0] = group((int)M, ff_, D, w.big2.get(), ff_, L.b1.get<float>());
    gemm(w.m_xn, L.m_w1, w.mo_ffh, p, kEpiStore16, L.bn_w1, s);
  }
  {
    GemmParams p{};
    p.num_groups = 1;
    p.groups[0] = group((int)M, D, ff_, x, D, L.b2.get<float>());
    gemm(w.m_big2_ffh, L.m_w2, mo_x, p, kEpiResid32, L.bn_w2, s);
  }
}

void Model::run_trunk(int B, int T, cudaStream_t s, Work& w) {
  const msst_model_info& I = info_;
  const float* pending = nullptr;
  const long long xn_elems = w.M * I.dim;
  for (int d = 0; d < I.depth; ++d) {
    // skip connections (src/model_mel_band_roformer.cu:846-852,898-901): x += the
    // outputs of every earlier depth block, which therefore carry their final norm
    if (skip_ && d > 0)
      MSST_CUDA(launch_skip_add(w.x.get<float>(), w.skips.get<float>(), d, xn_elems, s));
    for (int axis = 0; axis < 2; ++axis) {
      run_transformer(d, axis, w.x.get<float>(), B, T, pending, s, w);
      const TransformerWeights& tw = axis == 0 ? blocks_[d].first : blocks_[d].second;
      pending = mel_ ? tw.g_final.get<float>() : nullptr;
    }
    if (skip_ && d + 1 < I.depth) {
      if (pending) {
        RmsNormArgs rn{};
        rn.x = w.x.get<float>();
        rn.rows = w.M;
        rn.D = I.dim;
        rn.gamma_pre = pending;
        rn.scale_pre = std::sqrt((float)I.dim);
        MSST_CUDA(launch_rmsnorm(rn, bf16_, s));
        pending = nullptr;
      }
      MSST_CUDA(cudaMemcpyAsync(w.skips.get<float>() + (size_t)d * xn_elems, w.x.get(), 4 * (size_t)xn_elems,
                                cudaMemcpyDeviceToDevice, s));
    }
  }
  // final norm (MelBandRoformer: last transformer's norm_output; BSRoformer:
  // final_norm, src/model_bs_roformer.cu:536-539) -> band-major 16-bit input of
  // the mask estimators
  RmsNormArgs rn{};
  rn.x = w.x.get<float>();
  rn.rows = w.M;
  rn.D = I.dim;
  rn.gamma = mel_ ? pending : final_norm_.get<float>();
  rn.scale = std::sqrt((float)I.dim);
  rn.out16 = w.xn.get();
  rn.band_major = 1;
  rn.F = I.num_bands;
  MSST_CUDA(launch_rmsnorm(rn, bf16_, s));
}

void Model::run_masks(int B, int T, cudaStream_t s, Work& w, float* masks_out) {
  const msst_model_info& I = info_;
  const int nb = I.num_bands, D = I.dim;
  const int BT = (int)w.BT;
  for (int st = 0; st < I.num_stems; ++st) {
    const StemWeights& sw = stems_[st];
    float* mask = masks_out + (size_t)st * w.BT * sum_dims_;
    for (int i = 0; i < n_lin_; ++i) {
      const bool last = i == n_lin_ - 1;
      const CUtensorMap& ma = i == 0 ? w.m_xn : ((i - 1) % 2 == 0 ? w.m_h1 : w.m_h2);
      void* hout = (i % 2 == 0) ? w.big1.get() : w.big2.get();
      const int K = i == 0 ? D : hid_;
      GemmParams p{};
      p.num_groups = nb;
      p.act = kActTanh;
      for (int b = 0; b < nb; ++b) {
        GemmGroup g;
        if (last) {
          g = group(BT, 2 * dims_[b], K, mask, sum_dims_, sw.b[i].get<float>() + out3_off_[b]);
          g.b_row0 = out3_off_[b];
          g.out_col0 = dim_off_[b];
        } else {
          g = group(BT, hid_, K, hout, hid_, sw.b[i].get<float>() + (size_t)b * hid_);
          g.b_row0 = b * hid_;
          g.out_row_add = (long long)b * BT;
          g.oz0 = b;
        }
        g.a_row0 = b * BT;
        p.groups[b] = g;
      }
      const CUtensorMap& mo = (i % 2 == 0) ? w.mo_h1 : w.mo_h2;
      gemm(ma, sw.m[i], mo, p, last ? kEpiGlu32 : kEpiStore16, 256, s);
    }
  }
  (void)B;
  (void)T;
}

void Model::forward(const float* audio, int B, int C, long long L, float* out, cudaStream_t s) {
  forward_impl(audio, B, C, L, out, false, s);
}

void Model::forward_impl(const float* audio, int B, int C, long long L, float* out, bool fix_padding,
                         cudaStream_t s, const ChunkSource& src) {
  const msst_model_info& I = info_;
  MSST_REQUIRE(C == C_, "channel count does not match the model (stereo=" + std::to_string(C_ == 2) + ")");
  MSST_REQUIRE(B >= 1 && L > I.n_fft / 2, "audio too short");
  const int T = (int)(L / I.hop_length + 1);
  Work& w = work(B, T);
  run_front(audio, src, B, L, T, s, w);
  run_trunk(B, T, s, w);
  run_masks(B, T, s, w, w.mask.get<float>());
  // mask merge + complex multiply + zero DC -> C2R input
  MaskApplyArgs ma{};
  ma.spec = w.spec.get<float2>();
  ma.mask = w.mask.get<float>();
  ma.mask_stem_stride = w.BT * sum_dims_;
  ma.mask_ld = sum_dims_;
  ma.contrib_off = d_contrib_off_.get<int>();
  ma.contrib_col = d_contrib_col_.get<int>();
  ma.denom = d_denom_.get<float>();
  ma.bin_pack = d_bin_pack_.get<int4>();
  ma.out = w.ispec.get<float2>();
  ma.Bc = B;
  ma.S = I.num_stems;
  ma.C = C_;
  ma.T = T;
  ma.nbins = nbins_;
  ma.zero_dc = zero_dc_ ? 1 : 0;
  ma.spec_scale = stft_norm_ ? 1.0f / std::sqrt((float)I.n_fft) : 1.0f;
  ma.out_scale = stft_norm_ ? std::sqrt((float)I.n_fft) : 1.0f;
  MSST_CUDA(launch_mask_apply(ma, s));
  // iSTFT (src/ops_stft.cu:371-489)
  const int BSC = B * I.num_stems * C_;
  if (cufftExecC2R(fft_plan(CUFFT_C2R, BSC * T, s), w.ispec.get<cufftComplex>(), w.frames.get<cufftReal>()) !=
      CUFFT_SUCCESS)
    fail(MSST_ERR_CUDA, "cufftExecC2R failed");
  // output length: (T-1)*hop, or the input's length for match_input_audio_length models
  // (src/model_mel_band_roformer.cu:764,1021; src/model_bs_roformer.cu:436,595), whose
  // zero padding reproduces the reference's unless fix_padding
  MSST_CUDA(launch_istft_ola(w.frames.get<float>(), BSC, T, I.n_fft, I.hop_length, window_.get<float>(),
                             istft_wsum(T), out, out_length(L), fix_padding ? 0 : 1, s));
}

long long Model::out_length(long long L) const {
  return match_len_ ? L : (L / info_.hop_length) * info_.hop_length;
}

void Model::masks(const float* audio, int B, int C, long long L, float* masks_out, cudaStream_t s) {
  const msst_model_info& I = info_;
  MSST_REQUIRE(C == C_, "channel count does not match the model");
  const int T = (int)(L / I.hop_length + 1);
  Work& w = work(B, T);
  run_front(audio, ChunkSource(), B, L, T, s, w);
  run_trunk(B, T, s, w);
  run_masks(B, T, s, w, masks_out);
}

void Model::attn_block(int d, int axis, int layer, float* x, int B, int T, cudaStream_t s) {
  MSST_REQUIRE(d >= 0 && d < info_.depth && (axis == 0 || axis == 1), "bad depth index or axis");
  const TransformerWeights& tw = axis == 0 ? blocks_[d].first : blocks_[d].second;
  MSST_REQUIRE(layer >= 0 && layer < (int)tw.layers.size(), "bad layer index");
  Work& w = work(B, T);
  run_attn_block(d, axis, layer, x, B, T, nullptr, s, w);
}

void Model::ffn_block(int d, int axis, int layer, float* x, int B, int T, cudaStream_t s) {
  MSST_REQUIRE(d >= 0 && d < info_.depth && (axis == 0 || axis == 1), "bad depth index or axis");
  const TransformerWeights& tw = axis == 0 ? blocks_[d].first : blocks_[d].second;
  MSST_REQUIRE(layer >= 0 && layer < (int)tw.layers.size(), "bad layer index");
  Work& w = work(B, T);
  run_ffn_block(d, axis, layer, x, B, T, s, w);
}

void Model::band_tables(msst_band_tables* t) const {
  t->num_bands = info_.num_bands;
  t->nbins = nbins_;
  t->channels = C_;
  t->sum_kpad = ktot_;
  t->sum_dims = sum_dims_;
  t->bin_start = d_bin_start_.get<int>();
  t->nfreq = d_nfreq_.get<int>();
  t->bin_list = d_bin_list_.get<int>();
  t->kcol = d_kcol_.get<int>();
  t->kpad = d_kpad_.get<int>();
  t->gcol = d_gcol_.get<int>();
  t->gamma = g_bs_.get<float>();
  t->contrib_off = d_contrib_off_.get<int>();
  t->contrib_col = d_contrib_col_.get<int>();
  t->denom = d_denom_.get<float>();
}

void Model::transformer(int d, int axis, float* x, int B, int T, cudaStream_t s) {
  MSST_REQUIRE(d >= 0 && d < info_.depth && (axis == 0 || axis == 1), "bad depth index or axis");
  Work& w = work(B, T);
  run_transformer(d, axis, x, B, T, nullptr, s, w);
  if (mel_) {
    const TransformerWeights& tw = axis == 0 ? blocks_[d].first : blocks_[d].second;
    RmsNormArgs rn{};
    rn.x = x;
    rn.rows = (long long)B * T * info_.num_bands;
    rn.D = info_.dim;
    rn.gamma_pre = tw.g_final.get<float>();
    rn.scale_pre = std::sqrt((float)info_.dim);
    MSST_CUDA(launch_rmsnorm(rn, bf16_, s));
  }
}

// ===========================================================================
// chunked separation (src/inference_app.cpp:59-70,100-324)
// ===========================================================================
void Model::chunk_plan(long long L, float overlap, int* chunk, int* step, long long* border, long long* total,
                       int* num_chunks) const {
  const int cs = info_.chunk_size;
  int st;
  if (overlap > 0.0f && overlap < 1.0f) {
    st = std::max(1, (int)std::lround(cs * (1.0f - overlap)));
  } else {
    int n = info_.num_overlap;
    if (overlap >= 1.0f) n = std::max(1, (int)std::lround(overlap));
    st = std::max(1, cs / std::max(1, n));
  }
  long long b = cs - st;
  const bool padded = L > 2 * b && b > 0;
  if (!padded) b = 0;
  const long long tot = L + 2 * b;
  *chunk = cs;
  *step = st;
  *border = b;
  *total = tot;
  *num_chunks = (int)((tot + st - 1) / st);
}

// Sample ranges of chunk k of a track's plan: in[0..1] and in[2..3] are the two
// ranges [begin, end) of the track that its gather reads (its own reflect-padded
// window; for a short final chunk with the reference's contiguous-source padding
// also the track's first samples, else an empty second range), and
// [*out_lo, *out_hi) the output samples its overlap-add touches.
void Model::chunk_span(long long L, float overlap, int k, int flags, long long* in, long long* out_lo,
                       long long* out_hi) const {
  int chunk, step, n;
  long long border, total;
  chunk_plan(L, overlap, &chunk, &step, &border, &total, &n);
  MSST_REQUIRE(k >= 0 && k < n, "chunk index outside the track's plan");
  const long long s0 = (long long)k * step, e0 = std::min(s0 + chunk, total);
  // padded positions [a, b) -> track samples: reflect is monotone between its
  // breakpoints, so the extremes are at the range ends and the breakpoints
  auto cover = [&](long long a, long long b, long long* r) {
    long long lo = L, hi = 0;
    if (b > a) {
      const long long pts[6] = {a, b - 1, border - 1, border, border + L - 1, border + L};
      for (long long q : pts) {
        if (q < a || q >= b) continue;
        long long i = border ? q - border : q;
        if (i < 0) i = -i;
        else if (i >= L) i = 2 * (L - 1) - i;
        i = std::min(std::max(i, 0LL), L - 1);
        lo = std::min(lo, i);
        hi = std::max(hi, i + 1);
      }
    }
    r[0] = std::min(lo, hi);
    r[1] = hi;
  };
  cover(s0, e0, in);
  const bool ref_compat = !(flags & MSST_SEPARATE_FIX_TAIL_PADDING);
  if (e0 - s0 < chunk && ref_compat && C_ > 1)
    cover(0, std::min(total, (long long)(C_ - 1) * (e0 - s0)), in + 2);
  else
    in[2] = in[3] = 0;
  *out_lo = std::min(std::max(s0 - border, 0LL), L);
  *out_hi = std::min(std::max(e0 - border, 0LL), L);
}

cudaEvent_t Model::pipeline_event(size_t i) {
  while (events_.size() <= i) {
    cudaEvent_t e;
    MSST_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    events_.push_back(e);
  }
  return events_[i];
}

cudaStream_t Model::copy_stream(int which) {
  cudaStream_t& st = copy_streams_[which];
  if (!st) MSST_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  return st;
}

void Model::stitch_range(const float* chunks, int slot_ranks, int slot_cap, int C, long long L, float overlap,
                         long long begin, long long end, float* out, cudaStream_t s) {
  int chunk, step, n;
  long long border, total;
  chunk_plan(L, overlap, &chunk, &step, &border, &total, &n);
  MSST_REQUIRE(slot_ranks >= 1 && slot_cap >= (n + slot_ranks - 1) / slot_ranks, "chunk slot layout too small");
  MSST_REQUIRE(begin >= 0 && begin <= end && end <= L, "stitch range outside the track");
  StitchArgs a{};
  a.y = chunks;
  a.rows = info_.num_stems * C;
  a.chunk = chunk;
  a.step = step;
  a.num_chunks = n;
  a.border = border;
  a.total = total;
  a.L = L;
  a.slot_ranks = slot_ranks;
  a.slot_cap = slot_cap;
  a.out = out;
  a.begin = begin;
  a.end = end;
  MSST_CUDA(launch_stitch(a, s));
}

// Chunked separation (src/inference_app.cpp:100-324): the chunk outputs of the
// whole plan are kept ([num_chunks, stems*C, chunk]), and after every forward
// batch the output samples no later chunk touches are stitched.  With host
// buffers the track goes up in per-batch pieces on one copy stream (all issued
// first, each batch waits only for its own piece) and every stitched range goes
// down on another as soon as it is final, so the copies overlap the compute.
void Model::separate_pipeline(const float* track, const float* track_host, int C, long long L, float overlap,
                              int chunk_batch, int flags, float* out, float* out_host, cudaStream_t s) {
  const msst_model_info& I = info_;
  MSST_REQUIRE(C == C_, "channel count does not match the model");
  const int S = I.num_stems;
  const size_t row_bytes = sizeof(float) * (size_t)L;
  if (I.chunk_size <= 0 || L <= I.chunk_size) {
    // short input: one forward over the whole track (src/inference_app.cpp:463-472)
    MSST_REQUIRE(match_len_ || L % I.hop_length == 0,
                 "whole-track forward needs length % hop_length == 0 (or a match_input_audio_length model)");
    if (track_host) MSST_CUDA(cudaMemcpyAsync(const_cast<float*>(track), track_host, row_bytes * C,
                                              cudaMemcpyHostToDevice, s));
    forward_impl(track, 1, C, L, out, (flags & MSST_SEPARATE_FIX_TAIL_PADDING) != 0, s);
    if (out_host) MSST_CUDA(cudaMemcpyAsync(out_host, out, row_bytes * S * C, cudaMemcpyDeviceToHost, s));
    return;
  }
  int chunk, step, nchunks;
  long long border, total;
  chunk_plan(L, overlap, &chunk, &step, &border, &total, &nchunks);
  MSST_REQUIRE(chunk % I.hop_length == 0, "chunk_size must be a multiple of hop_length");
  const int eb = std::max(1, std::min(chunk_batch > 0 ? chunk_batch : 2, nchunks));
  ChunkArgs ci{};
  ci.track = track;
  ci.C = C;
  ci.L = L;
  ci.border = border;
  ci.total = total;
  ci.chunk = chunk;
  ci.step = step;
  ci.ref_compat = (flags & MSST_SEPARATE_FIX_TAIL_PADDING) ? 0 : 1;
  const size_t per_chunk = (size_t)S * C * chunk;
  sep_chunks_.ensure(sizeof(float) * per_chunk * nchunks);
  float* ys = sep_chunks_.get<float>();
  const int nbatch = (nchunks + eb - 1) / eb;
  if (track_host) {
    // the track goes up as a growing prefix: each batch's piece ends where its chunks stop reading
    cudaStream_t up = copy_stream(0);
    MSST_CUDA(cudaEventRecord(pipeline_event(0), s));  // the buffer may still be read by earlier work
    MSST_CUDA(cudaStreamWaitEvent(up, pipeline_event(0), 0));
    long long copied = 0;
    for (int b = 0; b < nbatch; ++b) {
      long long need = copied;
      for (int k = b * eb; k < std::min(nchunks, (b + 1) * eb); ++k) {
        long long in[4], olo, ohi;
        chunk_span(L, overlap, k, flags, in, &olo, &ohi);
        need = std::max(need, std::max(in[1], in[3]));
      }
      if (need > copied)
        MSST_CUDA(cudaMemcpy2DAsync(const_cast<float*>(track) + copied, row_bytes, track_host + copied, row_bytes,
                                    sizeof(float) * (size_t)(need - copied), (size_t)C, cudaMemcpyHostToDevice, up));
      copied = need;
      MSST_CUDA(cudaEventRecord(pipeline_event(1 + b), up));
    }
  }
  long long done = 0;
  for (int b = 0; b < nbatch; ++b) {
    const int g0 = b * eb, cnt = std::min(eb, nchunks - g0);
    if (track_host) MSST_CUDA(cudaStreamWaitEvent(s, pipeline_event(1 + b), 0));
    ChunkSource src;
    src.chunks = &ci;
    src.first = g0;
    forward_impl(nullptr, cnt, C, chunk, ys + (size_t)g0 * per_chunk, false, s, src);
    // without host output, one stitch at the end (a single large launch)
    if (!out_host && g0 + cnt < nchunks) continue;
    long long upto = L;
    if (g0 + cnt < nchunks) {
      long long in[4], olo, ohi;
      chunk_span(L, overlap, g0 + cnt, flags, in, &olo, &ohi);
      upto = olo;
    }
    if (upto > done) {
      stitch_range(ys, 1, nchunks, C, L, overlap, done, upto, out, s);
      if (out_host) {
        cudaStream_t down = copy_stream(1);
        cudaEvent_t ev = pipeline_event(1 + nbatch + b);
        MSST_CUDA(cudaEventRecord(ev, s));
        MSST_CUDA(cudaStreamWaitEvent(down, ev, 0));
        MSST_CUDA(cudaMemcpy2DAsync(out_host + done, row_bytes, out + done, row_bytes,
                                    sizeof(float) * (size_t)(upto - done), (size_t)S * C, cudaMemcpyDeviceToHost,
                                    down));
      }
      done = upto;
    }
  }
  if (out_host) {
    // the call's stream covers the copies, so the caller's sync (and the next call) sees them
    cudaEvent_t ev = pipeline_event(1 + 2 * nbatch);
    MSST_CUDA(cudaEventRecord(ev, copy_stream(1)));
    MSST_CUDA(cudaStreamWaitEvent(s, ev, 0));
  }
}

void Model::separate(const float* track, int C, long long L, float overlap, int chunk_batch, int flags, float* out,
                     cudaStream_t s) {
  separate_pipeline(track, nullptr, C, L, overlap, chunk_batch, flags, out, nullptr, s);
}

void Model::forward_chunks(const float* track, int C, long long L, float overlap, int first, int stride, int count,
                           int chunk_batch, int flags, float* out, cudaStream_t s) {
  const msst_model_info& I = info_;
  MSST_REQUIRE(C == C_, "channel count does not match the model");
  int chunk, step, nchunks;
  long long border, total;
  chunk_plan(L, overlap, &chunk, &step, &border, &total, &nchunks);
  MSST_REQUIRE(chunk % I.hop_length == 0, "chunk_size must be a multiple of hop_length");
  MSST_REQUIRE(stride >= 1, "chunk stride must be >= 1");
  MSST_REQUIRE(first >= 0 && count >= 0 && (count == 0 || first + (long long)(count - 1) * stride < nchunks),
               "chunk range outside the track's plan");
  if (count == 0) return;
  const int S = I.num_stems;
  const int eb = std::max(1, std::min(chunk_batch > 0 ? chunk_batch : 2, count));
  ChunkArgs ci{};
  ci.track = track;
  ci.C = C;
  ci.L = L;
  ci.border = border;
  ci.total = total;
  ci.chunk = chunk;
  ci.step = step;
  ci.ref_compat = (flags & MSST_SEPARATE_FIX_TAIL_PADDING) ? 0 : 1;
  const size_t per_chunk = (size_t)S * C * chunk;
  for (int i0 = 0; i0 < count; i0 += eb) {
    const int cnt = std::min(eb, count - i0);
    ChunkSource src;
    src.chunks = &ci;
    src.first = first + i0 * stride;
    src.stride = stride;
    forward_impl(nullptr, cnt, C, chunk, out + (size_t)i0 * per_chunk, false, s, src);
  }
}

void Model::stitch(const float* chunks, int C, long long L, float overlap, float* out, cudaStream_t s) {
  int chunk, step, n;
  long long border, total;
  chunk_plan(L, overlap, &chunk, &step, &border, &total, &n);
  stitch_range(chunks, 1, n, C, L, overlap, 0, L, out, s);
}

// Created at load on the model's device.
cudaStream_t Model::host_stream() { return host_stream_; }

void Model::separate_host(const float* track_host, int C, long long L, float overlap, int chunk_batch, int flags,
                          float* out_host) {
  const size_t in_bytes = sizeof(float) * (size_t)C * L;
  const size_t out_bytes = in_bytes * (size_t)info_.num_stems;
  host_in_.ensure(in_bytes);
  host_out_.ensure(out_bytes);
  separate_pipeline(host_in_.get<float>(), track_host, C, L, overlap, chunk_batch, flags, host_out_.get<float>(),
                    out_host, host_stream_);
  MSST_CUDA(cudaStreamSynchronize(host_stream_));
}

}  // namespace msst
