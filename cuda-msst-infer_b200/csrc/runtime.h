// runtime.h — host-side plumbing of libmsst_b200: errors, device buffers,
// TMA tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/msst_b200.h"

namespace msst {

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] inline void fail(int code, const std::string& msg) { throw Error(code, msg); }

#define MSST_CUDA(call)                                                                               \
  do {                                                                                                \
    cudaError_t e_ = (call);                                                                          \
    if (e_ != cudaSuccess)                                                                            \
      ::msst::fail(MSST_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_) + " (" + __FILE__ + \
                                      ":" + std::to_string(__LINE__) + ")");                          \
  } while (0)

#define MSST_REQUIRE(cond, msg)                                     \
  do {                                                              \
    if (!(cond)) ::msst::fail(MSST_ERR_INVALID, std::string(msg)); \
  } while (0)

// Owning device allocation.
class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  explicit DeviceBuffer(size_t bytes) { reset(bytes); }
  ~DeviceBuffer() { release(); }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  DeviceBuffer(DeviceBuffer&& o) noexcept : p_(o.p_), n_(o.n_) { o.p_ = nullptr, o.n_ = 0; }
  DeviceBuffer& operator=(DeviceBuffer&& o) noexcept {
    if (this != &o) {
      release();
      p_ = o.p_;
      n_ = o.n_;
      o.p_ = nullptr;
      o.n_ = 0;
    }
    return *this;
  }
  void reset(size_t bytes) {
    release();
    if (bytes) MSST_CUDA(cudaMalloc(&p_, bytes));
    n_ = bytes;
  }
  // grow-only
  void ensure(size_t bytes) {
    if (bytes > n_) reset(bytes);
  }
  void release() {
    if (p_) cudaFree(p_);
    p_ = nullptr;
    n_ = 0;
  }
  template <typename T = void>
  T* get() const {
    return static_cast<T*>(p_);
  }
  size_t bytes() const { return n_; }

 private:
  void* p_ = nullptr;
  size_t n_ = 0;
};

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    MSST_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !p) fail(MSST_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Tiled tensor map (16-bit elements and 128B swizzle unless told otherwise).
// dims/strides innermost first; strides in bytes for dims 1..rank-1.
inline CUtensorMap make_tensor_map(const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                                   const uint32_t* box,
                                   CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_UINT16,
                                   CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap m;
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides_bytes[i];
  CUresult r = tensor_map_encoder()(&m, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, e,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(MSST_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return m;
}

// Output map of the GEMM epilogue: 3-D {cols, Y, Z}; a warp's 32 staged rows
// run along Y (box {32, 32, 1}) or, with rows_along_z, along Z (box {32, 1, 32}).
// fp32 outputs (stores and residual reduce-adds) use 128B swizzle over 128 B
// staging rows; 16-bit outputs use 64B swizzle over 64 B rows.
inline CUtensorMap map_out(const void* base, bool fp32, uint64_t cols, uint64_t Y, uint64_t Z, uint64_t y_stride_elems,
                           uint64_t z_stride_elems, bool rows_along_z = false) {
  const uint64_t esz = fp32 ? 4 : 2;
  const uint64_t dims[3] = {cols, Y, Z};
  const uint64_t strides[2] = {y_stride_elems * esz, z_stride_elems * esz};
  const uint32_t box[3] = {32, rows_along_z ? 1u : 32u, rows_along_z ? 32u : 1u};
  return make_tensor_map(base, 3, dims, strides, box,
                         fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                         fp32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

// Plain row-major output [rows, cols] with row stride ld.
inline CUtensorMap map_out_2d(const void* base, bool fp32, uint64_t rows, uint64_t cols, uint64_t ld) {
  return map_out(base, fp32, cols, rows, 1, ld, ld * rows);
}

// Row-major 16-bit matrix [rows, cols] (row stride ld elements) read in boxes of
// 64 columns x box_rows rows.
inline CUtensorMap map_2d(const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
  const uint64_t dims[2] = {cols, rows};
  const uint64_t strides[1] = {ld * 2};
  const uint32_t box[2] = {64, box_rows};
  return make_tensor_map(base, 2, dims, strides, box);
}

// The B (weight) operand of a GEMM with column tile bn: boxes of 64 columns x
// bn/2 rows (a CTA pair loads one half each; a single CTA loads both).
inline CUtensorMap map_gemm_b(const void* base, uint64_t rows, uint64_t cols, uint64_t ld, int bn) {
  return map_2d(base, rows, cols, ld, (uint32_t)(bn / 2));
}

// Column tile of the GEMM for an output width n (a weight's B map is encoded
// for it: map_gemm_b(..., gemm_pick_bn(n))).
inline int gemm_pick_bn(int n) {
  if (n % 256 == 0) return 256;
  if (n % 192 == 0) return 192;
  return n <= 128 ? 128 : 256;
}

inline int device_sm_count() {
  int dev = 0, n = 0;
  MSST_CUDA(cudaGetDevice(&dev));
  MSST_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  return n;
}

// Per-translation-unit device error flags, ORed by msst_device_error().
unsigned gemm_device_error(bool clear);
unsigned attention_device_error(bool clear);
unsigned kernels_device_error(bool clear);
unsigned band_attention_device_error(bool clear);

inline unsigned device_error(bool clear) {
  return gemm_device_error(clear) | attention_device_error(clear) | kernels_device_error(clear) |
         band_attention_device_error(clear);
}

// Launch accounting (launch_stats.cu; see LaunchScope in common.cuh).
struct KernelStat {
  std::string name;
  unsigned long long launches = 0;
  double ms = 0, flop = 0, bytes = 0;
};
unsigned long long launch_count(bool reset);
void set_kernel_timing(bool on);
std::vector<KernelStat> kernel_timing_report();

}  // namespace msst
