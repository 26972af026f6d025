// Optimizer kernels over flat fp32 parameter buffers (sm_100a).
//
//   * fused AdamW (decoupled weight decay, bias correction) that also writes the
//     bf16 compute copy of the parameters, replacing torch's fused AdamW
//     (avgen/train/optimizer.py:198-205) plus the separate cast the forward
//     would otherwise need. The clip coefficient and the non-finite skip flag
//     are read from device memory, so clipping needs no host sync.
//   * squared L2 norm partials of a gradient range (grad clipping,
//     avgen/parallel/comm.py:128-180).
//   * EMA shadow update shadow += (1 - decay) * (param - shadow)
//     (avgen/train/ema.py:168-204), bf16 or fp32 shadow.
#include "include/host_utils.h"
#include "include/launchers.h"
#include "include/sm100.cuh"

namespace avgen {
namespace {

__global__ void adamw_kernel(AdamWDesc d) {
  // A non-finite step treats every gradient as zero (moments still decay).
  const bool zero_grads = d.skip != nullptr && *d.skip != 0;
  const float gscale = zero_grads ? 0.f : (d.grad_scale ? *d.grad_scale : 1.f);
  const float step_lr = d.lr / d.bias_correction1;
  const float decay = 1.f - d.lr * d.weight_decay;
  const long n4 = d.n / 4;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 p = reinterpret_cast<float4*>(d.param)[i];
    const float4 g = reinterpret_cast<const float4*>(d.grad)[i];
    float4 m = reinterpret_cast<float4*>(d.exp_avg)[i];
    float4 v = reinterpret_cast<float4*>(d.exp_avg_sq)[i];
    float pv[4] = {p.x, p.y, p.z, p.w}, gv[4] = {g.x, g.y, g.z, g.w};
    float mv[4] = {m.x, m.y, m.z, m.w}, vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float gr = zero_grads ? 0.f : gv[e] * gscale;
      mv[e] = d.beta1 * mv[e] + (1.f - d.beta1) * gr;
      vv[e] = d.beta2 * vv[e] + (1.f - d.beta2) * gr * gr;
      const float denom = sqrtf(vv[e]) / d.bias_correction2_sqrt + d.eps;
      pv[e] = pv[e] * decay - step_lr * mv[e] / denom;
    }
    reinterpret_cast<float4*>(d.param)[i] = make_float4(pv[0], pv[1], pv[2], pv[3]);
    reinterpret_cast<float4*>(d.exp_avg)[i] = make_float4(mv[0], mv[1], mv[2], mv[3]);
    reinterpret_cast<float4*>(d.exp_avg_sq)[i] = make_float4(vv[0], vv[1], vv[2], vv[3]);
    if (d.param_bf16 != nullptr) {
      uint2 w;
      w.x = pack_bf16(pv[0], pv[1]);
      w.y = pack_bf16(pv[2], pv[3]);
      reinterpret_cast<uint2*>(d.param_bf16)[i] = w;
    }
  }
  // scalar tail
  for (long i = n4 * 4 + static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < d.n; i += stride) {
    const float gr = zero_grads ? 0.f : d.grad[i] * gscale;
    const float mv = d.beta1 * d.exp_avg[i] + (1.f - d.beta1) * gr;
    const float vv = d.beta2 * d.exp_avg_sq[i] + (1.f - d.beta2) * gr * gr;
    const float denom = sqrtf(vv) / d.bias_correction2_sqrt + d.eps;
    const float pv = d.param[i] * decay - step_lr * mv / denom;
    d.param[i] = pv;
    d.exp_avg[i] = mv;
    d.exp_avg_sq[i] = vv;
    if (d.param_bf16 != nullptr) reinterpret_cast<__nv_bfloat16*>(d.param_bf16)[i] = __float2bfloat16_rn(pv);
  }
}

__global__ void __launch_bounds__(256) sq_norm_kernel(const float* x, long n, float* out) {
  float s = 0.f;
  const long n4 = n / 4;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (long i = n4 * 4 + static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    s += x[i] * x[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < 8; ++k) t += red[k];
    atomicAdd(out, t);
  }
}

__global__ void ema_kernel(long n, const float* param, void* shadow, bool shadow_bf16, float decay) {
  const float w = 1.f - decay;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    if (shadow_bf16) {
      __nv_bfloat16* s = reinterpret_cast<__nv_bfloat16*>(shadow);
      const float sv = __bfloat162float(s[i]);
      s[i] = __float2bfloat16_rn(sv + w * (param[i] - sv));
    } else {
      float* s = reinterpret_cast<float*>(shadow);
      s[i] = s[i] + w * (param[i] - s[i]);
    }
  }
}

long grid_for(long work, int device) {
  const long want = (work + 255) / 256;
  return std::max<long>(1, std::min<long>(want, 16L * num_sms(device)));
}

}  // namespace

void adamw_launch(const AdamWDesc& d, cudaStream_t stream) {
  if (d.n == 0) return;
  AVGEN_CHECK(reinterpret_cast<uintptr_t>(d.param) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(d.grad) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(d.exp_avg) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(d.exp_avg_sq) % 16 == 0 &&
                  (d.param_bf16 == nullptr || reinterpret_cast<uintptr_t>(d.param_bf16) % 8 == 0),
              "adamw: buffers must be 16-byte aligned");
  adamw_kernel<<<grid_for(d.n / 4 + 1, d.device), 256, 0, stream>>>(d);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

void sq_norm_launch(int device, const float* x, long n, float* out, cudaStream_t stream) {
  if (n == 0) return;
  AVGEN_CHECK(reinterpret_cast<uintptr_t>(x) % 16 == 0, "sq_norm: buffer must be 16-byte aligned");
  sq_norm_kernel<<<grid_for(n / 4 + 1, device), 256, 0, stream>>>(x, n, out);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

void ema_launch(int device, long n, const float* param, void* shadow, bool shadow_bf16, float decay,
                cudaStream_t stream) {
  if (n == 0) return;
  ema_kernel<<<grid_for(n, device), 256, 0, stream>>>(n, param, shadow, shadow_bf16, decay);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

}  // namespace avgen
