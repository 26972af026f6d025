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
#include <algorithm>
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

// dst = sum of nsrc bf16 tensors of n8 * 8 elements each (fp32 accumulation):
// the owner-side reduction of context-parallel dK/dV partials pushed by peers.
__global__ void slab_sum_kernel(const __nv_bfloat16* const* srcs, int nsrc, __nv_bfloat16* dst, long n8) {
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < nsrc; ++s) {
      const uint4 v = reinterpret_cast<const uint4*>(srcs[s])[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[2 * e] += bf16_lo(w[e]);
        acc[2 * e + 1] += bf16_hi(w[e]);
      }
    }
    uint4 o;
    o.x = pack_bf16(acc[0], acc[1]);
    o.y = pack_bf16(acc[2], acc[3]);
    o.z = pack_bf16(acc[4], acc[5]);
    o.w = pack_bf16(acc[6], acc[7]);
    reinterpret_cast<uint4*>(dst)[i] = o;
  }
}

}  // namespace

void slab_sum_launch(const void* const* srcs_dev, int nsrc, void* dst, long n, int device, cudaStream_t stream) {
  AVGEN_CHECK(n % 8 == 0, "slab_sum: element count must be a multiple of 8");
  if (n == 0) return;
  const long n8 = n / 8;
  const long blocks = std::max<long>(1, std::min<long>((n8 + 255) / 256, 8L * num_sms(device)));
  slab_sum_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16* const*>(srcs_dev), nsrc,
                                               reinterpret_cast<__nv_bfloat16*>(dst), n8);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

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
