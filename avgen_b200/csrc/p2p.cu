// Intra-node peer-memory runtime for the fused NVLink paths (no counterpart in
// the reference, whose collectives all go through NCCL).
//
//   * symmetric buffers: cudaMalloc'd outside the caching allocator, exported
//     with CUDA IPC handles that the ranks exchange over the process group and
//     map into each peer's address space (every GPU of an NVSwitch node reaches
//     every other at full NVLink bandwidth);
//   * peer copies issued as cudaMemcpyAsync on a copy stream (NVLink copy engines);
//   * flag writes as stream memory operations (cuStreamWriteValue32 through the
//     driver entry point), executed by the GPU front end after the preceding
//     copies, never by SMs, so a kernel that occupies every SM can wait on them
//     (boundedly) without starving them. Streams themselves never wait on flags:
//     an unbounded stream-side wait could deadlock against implicit ordering.
#include <mutex>

#include "include/host_utils.h"
#include "include/launchers.h"
#include "include/sm100.cuh"

namespace avgen {
namespace {

using WriteValueFn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

template <typename Fn>
Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  AVGEN_CUDA_CHECK(cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q));
  AVGEN_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr, name, " is unavailable");
  return reinterpret_cast<Fn>(p);
}

WriteValueFn write_value_fn() {
  static WriteValueFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] { fn = driver_fn<WriteValueFn>("cuStreamWriteValue32"); });
  return fn;
}

}  // namespace

void* p2p_alloc(size_t bytes, int device) {
  int prev = 0;
  AVGEN_CUDA_CHECK(cudaGetDevice(&prev));
  AVGEN_CUDA_CHECK(cudaSetDevice(device));
  void* ptr = nullptr;
  AVGEN_CUDA_CHECK(cudaMalloc(&ptr, bytes));
  AVGEN_CUDA_CHECK(cudaMemset(ptr, 0, bytes));
  AVGEN_CUDA_CHECK(cudaSetDevice(prev));
  return ptr;
}

void p2p_free(void* ptr) { AVGEN_CUDA_CHECK(cudaFree(ptr)); }

void p2p_export(void* ptr, char* handle64) {
  cudaIpcMemHandle_t h;
  AVGEN_CUDA_CHECK(cudaIpcGetMemHandle(&h, ptr));
  static_assert(sizeof(h) == 64, "CUDA IPC handle is 64 bytes");
  memcpy(handle64, &h, 64);
}

void* p2p_open(const char* handle64, int device) {
  int prev = 0;
  AVGEN_CUDA_CHECK(cudaGetDevice(&prev));
  AVGEN_CUDA_CHECK(cudaSetDevice(device));
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  void* ptr = nullptr;
  AVGEN_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  AVGEN_CUDA_CHECK(cudaSetDevice(prev));
  return ptr;
}

void p2p_close(void* ptr) { AVGEN_CUDA_CHECK(cudaIpcCloseMemHandle(ptr)); }

void stream_write(cudaStream_t stream, void* flag, unsigned value) {
  const CUresult r = write_value_fn()(reinterpret_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(flag), value,
                                      CU_STREAM_WRITE_VALUE_DEFAULT);
  AVGEN_CHECK(r == CUDA_SUCCESS, "cuStreamWriteValue32 failed (", static_cast<int>(r), ")");
}

void p2p_copy(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
  AVGEN_CUDA_CHECK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, stream));
}

}  // namespace avgen
