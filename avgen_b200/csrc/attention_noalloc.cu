// Allocation-free C entry point for the attention backward.
//
// This entry point has no counterpart in the reference framework (avgen ships
// no native code). It exists for callers that must not allocate device memory
// per call (a runtime that captures calls into CUDA graphs or budgets memory
// up front): it runs the two-pass attention backward, whose only scratch is the
// per-row statistic delta = rowsum(dO * O), with that scratch held in a
// file-scope device array instead of a fresh allocation.
//
// Contract:
//  * scratch limit: B * H * lse_ld floats <= kNoAllocScratchFloats (4 MiB of
//    fp32, e.g. 20 heads x 52,428 queries); larger problems are rejected with
//    status 2 and nothing is launched;
//  * the scratch is one array per device shared by every call: calls whose
//    work overlaps on the GPU (two streams, two host threads) race on it, so
//    serialise them on one stream;
//  * its contents persist between calls (they hold the last call's delta);
//  * nothing here allocates: the scratch and the kernel error word are static
//    device arrays whose addresses are fetched once per device with
//    cudaGetSymbolAddress.
//
// Status codes: 0 ok, 1 invalid argument, 2 scratch limit exceeded, 3 CUDA
// error while resolving the scratch address, 4 launch error (message kept for
// avgen_attn_bwd_noalloc_last_error).

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <exception>
#include <mutex>

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

// Attention backward without device allocation (two-pass kernels, delta scratch
// in a static device array). q [B, H, Lq, 128], k / v [B, Hk, Lk, 128], o / dout
// [B, Lq, H, 128] dense bf16; lse fp32 [B, H, Lq] with row stride lse_ld (a
// multiple of 4, >= Lq); dq / dk / dv bf16 outputs shaped like q / k / v; kmask
// packed key-valid bits [B, kmask_words] or null; stream is a cudaStream_t.
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

// Message of the last failing call on this host thread ("" if none).
__attribute__((visibility("default"))) const char* avgen_attn_bwd_noalloc_last_error() { return g_last_error; }

}  // extern "C"
