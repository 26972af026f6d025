// Sampling-loop kernels for sm_100a (bandwidth-bound, one pass over the latents):
//   * guided Euler step: x' = x + (s' - s) * (u + w (c - u)) with the conditional
//     and unconditional velocities read from one batched [2B, ...] forward output
//     (avgen/infer/sampler.py:357-405, avgen/infer/guidance.py:336-360 behaviour)
//   * Flow-GRPO SDE transition: the marginal-preserving Euler-Maruyama mean
//     mean = x + (v + g^2 / (2 s) * (x + (1 - s) v)) * ds, the sample
//     mean + g sqrt(|ds|) * z (rollout) or a stored sample (update), and the
//     per-sample Gaussian log-density summed over every element
//     (avgen/rl/sde.py:239-349 behaviour). One block reduction and one atomic
//     per block and sample.
#include "include/host_utils.h"
#include "include/launchers.h"
#include "include/sm100.cuh"

namespace avgen {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float ld_any(const void* p, bool f32, long idx) {
  return f32 ? reinterpret_cast<const float*>(p)[idx]
             : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[idx]);
}

__global__ void guided_euler_kernel(GuidedEulerDesc d) {
  const long total = static_cast<long>(d.batch) * d.per_sample;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long b = i / d.per_sample;
    const float c = ld_any(d.cond, d.vel_f32, i);
    float v = c;
    if (d.uncond != nullptr) {
      const float u = ld_any(d.uncond, d.vel_f32, i);
      v = u + d.scale * (c - u);
    }
    const float x = ld_any(d.x, d.x_f32, i);
    const float dt = d.sigma_next[b] - d.sigma[b];
    const float y = x + dt * v;
    if (d.out_f32) reinterpret_cast<float*>(d.out)[i] = y;
    else reinterpret_cast<__nv_bfloat16*>(d.out)[i] = __float2bfloat16(y);
  }
}

// grid: (chunks, batch); each block walks its chunk of one sample.
__global__ void __launch_bounds__(256) sde_step_kernel(SDEStepDesc d) {
  const int b = blockIdx.y;
  const long base = static_cast<long>(b) * d.per_sample;
  const float s = fmaxf(d.sigma[b], d.floor);
  const float ds = d.sigma_next[b] - d.sigma[b];
  const float g = d.g[b];
  const float std = g * sqrtf(fabsf(ds));
  const float coef = g * g / (2.f * s);
  const bool score = std > 0.f;
  const float inv_std = score ? 1.f / fmaxf(std, 1e-12f) : 0.f;
  const float log_norm = score ? -logf(fmaxf(std, 1e-12f)) - 0.91893853320467274f : 0.f;  // 0.5 log(2 pi)
  float acc = 0.f;
  for (long j = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; j < d.per_sample;
       j += static_cast<long>(gridDim.x) * blockDim.x) {
    const long i = base + j;
    const float v = ld_any(d.v, d.v_f32, i);
    const float x = d.x[i];
    const float mean = x + (v + coef * (x + (1.f - s) * v)) * ds;
    d.mean[i] = mean;
    float smp;
    if (d.prev != nullptr) {
      smp = d.prev[i];
    } else {
      smp = mean + std * d.noise[i];
      d.sample[i] = smp;
    }
    if (score && (d.mask == nullptr || d.mask[i])) {
      const float r = (smp - mean) * inv_std;
      acc += -0.5f * r * r + log_norm;
    }
  }
  acc = warp_sum(acc);
  __shared__ float part[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) part[warp] = acc;
  __syncthreads();
  if (warp == 0) {
    float t = lane < static_cast<int>(blockDim.x >> 5) ? part[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) atomicAdd(d.log_prob + b, t);
  }
}

}  // namespace

void guided_euler_launch(const GuidedEulerDesc& d, cudaStream_t stream) {
  const long total = static_cast<long>(d.batch) * d.per_sample;
  if (total == 0) return;
  const long want = (total + 255) / 256;
  const long blocks = std::max<long>(1, std::min<long>(want, 16L * num_sms(d.device)));
  guided_euler_kernel<<<blocks, 256, 0, stream>>>(d);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

void sde_step_launch(const SDEStepDesc& d, cudaStream_t stream) {
  if (d.batch == 0 || d.per_sample == 0) return;
  AVGEN_CHECK(d.batch <= 65535, "sde_step: batch above 65535");
  const long want = (d.per_sample + 255) / 256;
  const long per_sample_blocks = std::max<long>(1, 8L * num_sms(d.device) / std::max(1, d.batch));
  const dim3 grid(static_cast<unsigned>(std::max<long>(1, std::min<long>(want, per_sample_blocks))),
                  static_cast<unsigned>(d.batch));
  sde_step_kernel<<<grid, 256, 0, stream>>>(d);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

}  // namespace avgen
