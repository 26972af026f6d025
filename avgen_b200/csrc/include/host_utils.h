// Host-side helpers shared by the avgen_b200 CUDA extension: error checking, the
// per-device error word that bounded device waits report into, SM counts, and
// TMA tensor-map construction through the driver entry point (no -lcuda link).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdexcept>
#include <string>
#include <sstream>

#include <mutex>
#include <utility>

namespace avgen {
template <typename... Args>
inline std::string cat_msg(Args&&... args) {
  std::ostringstream os;
  (os << ... << args);
  return os.str();
}
}  // namespace avgen

// Throws std::runtime_error (a Python RuntimeError through pybind11).
#define AVGEN_CHECK(cond, ...)                                                    \
  do {                                                                            \
    if (!(cond)) throw std::runtime_error(::avgen::cat_msg("avgen_b200: ", __VA_ARGS__)); \
  } while (0)

#define AVGEN_CUDA_CHECK(expr)                                                        \
  do {                                                                                \
    cudaError_t _e = (expr);                                                          \
    AVGEN_CHECK(_e == cudaSuccess, "CUDA error: ", cudaGetErrorString(_e), " at ",     \
                __FILE__, ":", __LINE__);                                             \
  } while (0)

namespace avgen {

constexpr int kMaxDevices = 64;

// Device word that kernels write a non-zero error code into when a bounded wait
// runs out. Allocated once per device and kept for the life of the process.
inline int* error_word(int device) {
  static int* words[kMaxDevices] = {nullptr};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  AVGEN_CHECK(device >= 0 && device < kMaxDevices, "bad device index");
  if (words[device] == nullptr) {
    int prev = -1;
    AVGEN_CUDA_CHECK(cudaGetDevice(&prev));
    AVGEN_CUDA_CHECK(cudaSetDevice(device));
    AVGEN_CUDA_CHECK(cudaMalloc(&words[device], sizeof(int)));
    AVGEN_CUDA_CHECK(cudaMemset(words[device], 0, sizeof(int)));
    AVGEN_CUDA_CHECK(cudaSetDevice(prev));
  }
  return words[device];
}

// Runs a callable once per device, thread-safely. Kernel attributes (the
// dynamic shared-memory limit among them) are per device, so a per-process
// flag would leave every device but the first one without them.
class PerDeviceOnce {
 public:
  template <typename Fn>
  void run(int device, Fn&& fn) {
    AVGEN_CHECK(device >= 0 && device < kMaxDevices, "bad device index ", device);
    std::call_once(flags_[device], std::forward<Fn>(fn));
  }

 private:
  std::once_flag flags_[kMaxDevices];
};

// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current device
// (once per device for each `once`).
template <typename Kernel>
inline void raise_smem_limit(PerDeviceOnce& once, Kernel kernel, int bytes) {
  int device = 0;
  AVGEN_CUDA_CHECK(cudaGetDevice(&device));
  once.run(device, [&] {
    AVGEN_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  });
}

inline int num_sms(int device) {
  AVGEN_CHECK(device >= 0 && device < kMaxDevices, "bad device index ", device);
  static PerDeviceOnce once;
  static int cache[kMaxDevices] = {0};
  once.run(device, [&] {
    int n = 0;
    AVGEN_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
    cache[device] = n;
  });
  return cache[device];
}

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    AVGEN_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    AVGEN_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr,
                "cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major matrix [outer, inner] with row stride
// `row_stride` elements, loading boxes of [box_outer, box_inner] with the
// 128-byte swizzle the UMMA descriptors expect (box_inner * 2 must be <= 128).
inline CUtensorMap make_tmap_2d_bf16(const void* ptr, int64_t inner, int64_t outer,
                                     int64_t row_stride, int box_inner, int box_outer,
                                     CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                    const_cast<void*>(ptr), dims, strides, box, estr,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  AVGEN_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", static_cast<int>(r),
              ") inner=", inner, " outer=", outer, " stride=", row_stride);
  return map;
}

// 3-D bf16 tensor map [d2, d1, d0] (d0 innermost) with explicit strides (elements).
inline CUtensorMap make_tmap_3d_bf16(const void* ptr, int64_t d0, int64_t d1, int64_t d2,
                                     int64_t s1, int64_t s2, int b0, int b1, int b2,
                                     CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap map;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1),
                        static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s1 * 2), static_cast<cuuint64_t>(s2 * 2)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(b0), static_cast<cuuint32_t>(b1),
                       static_cast<cuuint32_t>(b2)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                                    const_cast<void*>(ptr), dims, strides, box, estr,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  AVGEN_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3d) failed (", static_cast<int>(r), ")");
  return map;
}

}  // namespace avgen
