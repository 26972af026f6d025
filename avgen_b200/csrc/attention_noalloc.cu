// Allocation-free C entry point for the attention backward: the definitions
// of include/attention_noalloc.h, whose comment states the contract (scratch
// limit, the shared array and the race between overlapping calls, status
// codes). No counterpart exists in the reference framework, which ships no
// native code.

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <exception>
#include <mutex>

#include "include/attention_noalloc.h"
#include "include/launchers.h"

namespace {

constexpr long kNoAllocScratchFloats = 1L << 20;  // 4 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
static __device__ __align__(256) int g_noalloc_err[1];

struct DeviceSlots {
  float* scratch = nullptr;
  int* err = nullptr;
};

DeviceSlots g_slots[kMaxDevices];
std::once_flag g_once[kMaxDevices];
cudaError_t g_resolve_status[kMaxDevices];
thread_local char g_last_error[256] = {0};

void set_error(const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
}

// Address of the scratch and error word on `device` (resolved once per device).
cudaError_t resolve(int device, DeviceSlots& out) {
  std::call_once(g_once[device], [device] {
    void* scratch = nullptr;
    void* err = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&err, g_noalloc_err);
    g_resolve_status[device] = e;
    if (e == cudaSuccess) {
      g_slots[device].scratch = static_cast<float*>(scratch);
      g_slots[device].err = static_cast<int*>(err);
    }
  });
  out = g_slots[device];
  return g_resolve_status[device];
}

}  // namespace

extern "C" {

// Declared (with the argument layout) in include/attention_noalloc.h.
__attribute__((visibility("default"))) int avgen_attn_bwd_noalloc(
    const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse, long lse_ld,
    void* dq, void* dk, void* dv, const unsigned int* kmask, int kmask_words, int B, int H, int Hk, int Lq, int Lk,
    float scale, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr || dout == nullptr || lse == nullptr ||
      dq == nullptr || dk == nullptr || dv == nullptr || B <= 0 || H <= 0 || Hk <= 0 || Lq <= 0 || Lk <= 0 ||
      H % Hk != 0 || lse_ld < Lq || lse_ld % 4 != 0 || (kmask != nullptr && kmask_words < (Lk + 31) / 32)) {
    set_error("avgen_attn_bwd_noalloc: invalid argument");
    return 1;
  }
  if (static_cast<long>(B) * H * lse_ld > kNoAllocScratchFloats) {
    set_error("avgen_attn_bwd_noalloc: B * H * lse_ld exceeds the 1,048,576-float scratch");
    return 2;
  }
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
    set_error("avgen_attn_bwd_noalloc: no current CUDA device");
    return 3;
  }
  if (stream != nullptr) {  // the scratch address is per device: the stream must run on this one
    int stream_device = -1;
    if (cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &stream_device) != cudaSuccess ||
        stream_device != device) {
      set_error("avgen_attn_bwd_noalloc: the stream does not belong to the current device");
      return 1;
    }
  }
  DeviceSlots slots;
  if (resolve(device, slots) != cudaSuccess) {
    set_error("avgen_attn_bwd_noalloc: cudaGetSymbolAddress failed");
    return 3;
  }
  avgen::AttnBwdDesc d;
  d.device = device;
  d.B = B;
  d.H = H;
  d.Hk = Hk;
  d.Lq = Lq;
  d.Lk = Lk;
  d.D = 128;
  d.scale = scale;
  d.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);  // scale * log2(e)
  d.q = q;
  d.k = k;
  d.v = v;
  d.o = o;
  d.dout = dout;
  d.o_sh = 128;
  d.o_sl = static_cast<long>(H) * 128;
  d.o_sb = static_cast<long>(Lq) * H * 128;
  d.lse = lse;
  d.delta = slots.scratch;
  d.stat_ld = lse_ld;
  d.kmask = kmask;
  d.kmask_words = kmask_words;
  d.dq = static_cast<__nv_bfloat16*>(dq);
  d.dk = static_cast<__nv_bfloat16*>(dk);
  d.dv = static_cast<__nv_bfloat16*>(dv);
  d.dq_acc = nullptr;  // two-pass kernels: no dQ accumulator
  d.err = slots.err;
  try {
    avgen::attn_bwd_launch(d, static_cast<cudaStream_t>(stream));
  } catch (const std::exception& exc) {
    set_error(exc.what());
    return 4;
  }
  return 0;
}

__attribute__((visibility("default"))) const char* avgen_attn_bwd_noalloc_last_error(void) { return g_last_error; }

__attribute__((visibility("default"))) int avgen_attn_bwd_noalloc_device_error(int* out, int clear) {
  if (out == nullptr) {
    set_error("avgen_attn_bwd_noalloc_device_error: null output");
    return 1;
  }
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
    set_error("avgen_attn_bwd_noalloc_device_error: no current CUDA device");
    return 3;
  }
  DeviceSlots slots;
  if (resolve(device, slots) != cudaSuccess) {
    set_error("avgen_attn_bwd_noalloc_device_error: cudaGetSymbolAddress failed");
    return 3;
  }
  int word = 0;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(&word, slots.err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess ||
      (clear != 0 && cudaMemset(slots.err, 0, sizeof(int)) != cudaSuccess) ||
      (clear != 0 && cudaDeviceSynchronize() != cudaSuccess)) {
    set_error("avgen_attn_bwd_noalloc_device_error: CUDA error while reading the error word");
    return 3;
  }
  *out = word;
  return 0;
}

}  // extern "C"
