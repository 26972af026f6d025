// Sharded data-parallel kernels: the FSDP gradient reduce-scatter as a pull over
// NVLink peer memory, and AdamW / gradient norm over the per-parameter shards.
//
// Replaces, for FSDP2 on one NVSwitch node, the NCCL reduce-scatter of the
// reference's sharding (avgen/parallel/fsdp.py:123-135, reduce_dtype fp32) and
// torch's fused AdamW over the sharded DTensor parameters
// (avgen/train/optimizer.py:198-205).
//
//   peer_reduce  out[i] = scale * sum over ranks r of src_r[offset + i]: every
//                rank reads its shard of every peer's gradient buffer (mapped
//                with CUDA IPC) with plain loads over NVLink and sums in fp32;
//                the scale folds the data-parallel average into the same pass,
//                and an optional squared-norm partial of the result feeds
//                gradient clipping.
//   mt_sq_norm / mt_adamw  multi-tensor kernels over a table of shards (one
//                row per parameter: param, grad, both moments) cut into chunks;
//                the clip coefficient and the non-finite skip flag come from
//                device memory, so a step needs no host synchronisation.
#include <algorithm>

#include "include/host_utils.h"
#include "include/launchers.h"
#include "include/sm100.cuh"

namespace avgen {
namespace {

constexpr int kMaxRanks = 16;

struct Sources {
  const void* p[kMaxRanks];
};

__device__ __forceinline__ void block_sum_atomic(float s, float* acc) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float red[32];
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[warp] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) atomicAdd(acc, t);
  }
}

// fp32 sources, 16-byte aligned: four elements per load.
__global__ void __launch_bounds__(256) peer_reduce_f32x4_kernel(Sources src, int world, int first, long offset4,
                                                                long n4, float scale, float* out, float* sq_acc) {
  float s = 0.f;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < world; ++k) {  // start at a different peer on every rank: spread the reads
      const int r = (first + k) % world;
      const float4 v = reinterpret_cast<const float4*>(src.p[r])[offset4 + i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    acc.x *= scale;
    acc.y *= scale;
    acc.z *= scale;
    acc.w *= scale;
    reinterpret_cast<float4*>(out)[i] = acc;
    s += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  if (sq_acc != nullptr) block_sum_atomic(s, sq_acc);
}

// Any alignment, fp32 or bf16 sources: one element per load.
template <bool BF16>
__global__ void __launch_bounds__(256) peer_reduce_scalar_kernel(Sources src, int world, int first, long offset,
                                                                 long n, float scale, float* out, float* sq_acc) {
  float s = 0.f;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    float acc = 0.f;
    for (int k = 0; k < world; ++k) {
      const int r = (first + k) % world;
      if constexpr (BF16)
        acc += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(src.p[r])[offset + i]);
      else
        acc += reinterpret_cast<const float*>(src.p[r])[offset + i];
    }
    acc *= scale;
    out[i] = acc;
    s += acc * acc;
  }
  if (sq_acc != nullptr) block_sum_atomic(s, sq_acc);
}

__global__ void __launch_bounds__(256) mt_sq_norm_kernel(const MTChunk* __restrict__ chunks,
                                                         const MTTensor* __restrict__ tensors, float* acc) {
  const MTChunk c = chunks[blockIdx.x];
  const float* g = tensors[c.tensor].grad + c.start;
  float s = 0.f;
  for (long i = threadIdx.x; i < c.len; i += blockDim.x) {
    const float v = g[i];
    s += v * v;
  }
  block_sum_atomic(s, acc);
}

__global__ void __launch_bounds__(256) mt_adamw_kernel(const MTChunk* __restrict__ chunks,
                                                       const MTTensor* __restrict__ tensors, MTAdamWArgs a) {
  const MTChunk c = chunks[blockIdx.x];
  const MTTensor t = tensors[c.tensor];
  // A non-finite step treats every gradient as zero (the moments still decay).
  const bool zero_grads = a.skip != nullptr && *a.skip != 0;
  const float gscale = zero_grads ? 0.f : (a.grad_scale != nullptr ? *a.grad_scale : 1.f);
  const float step_lr = a.lr / a.bias_correction1;
  const float decay = 1.f - a.lr * a.weight_decay;
  for (long i = c.start + threadIdx.x; i < c.start + c.len; i += blockDim.x) {
    const float gr = zero_grads ? 0.f : t.grad[i] * gscale;
    const float m = a.beta1 * t.exp_avg[i] + (1.f - a.beta1) * gr;
    const float v = a.beta2 * t.exp_avg_sq[i] + (1.f - a.beta2) * gr * gr;
    const float denom = sqrtf(v) / a.bias_correction2_sqrt + a.eps;
    t.param[i] = t.param[i] * decay - step_lr * m / denom;
    t.exp_avg[i] = m;
    t.exp_avg_sq[i] = v;
  }
}

long grid_for(long work, int device) {
  return std::max<long>(1, std::min<long>((work + 255) / 256, 4L * num_sms(device)));
}

}  // namespace

void peer_reduce_launch(const void* const* srcs, int world, int rank, long offset, long n, bool src_bf16, float scale,
                        float* out, float* sq_acc, int device, cudaStream_t stream) {
  AVGEN_CHECK(world >= 1 && world <= kMaxRanks, "peer_reduce: 1..", kMaxRanks, " ranks supported, got ", world);
  AVGEN_CHECK(rank >= 0 && rank < world && offset >= 0 && n >= 0, "peer_reduce: bad rank or range");
  if (n == 0) return;
  Sources s{};
  bool aligned = !src_bf16 && offset % 4 == 0 && n % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  for (int r = 0; r < world; ++r) {
    AVGEN_CHECK(srcs[r] != nullptr, "peer_reduce: null source for rank ", r);
    s.p[r] = srcs[r];
    aligned = aligned && (reinterpret_cast<uintptr_t>(srcs[r]) & 15u) == 0;
  }
  const int first = (rank + 1) % world;
  if (aligned) {
    peer_reduce_f32x4_kernel<<<grid_for(n / 4, device), 256, 0, stream>>>(s, world, first, offset / 4, n / 4, scale,
                                                                          out, sq_acc);
  } else if (src_bf16) {
    peer_reduce_scalar_kernel<true><<<grid_for(n, device), 256, 0, stream>>>(s, world, first, offset, n, scale, out,
                                                                             sq_acc);
  } else {
    peer_reduce_scalar_kernel<false><<<grid_for(n, device), 256, 0, stream>>>(s, world, first, offset, n, scale,
                                                                              out, sq_acc);
  }
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

void mt_sq_norm_launch(const MTChunk* chunks, int nchunks, const MTTensor* tensors, float* acc, cudaStream_t stream) {
  if (nchunks == 0) return;
  mt_sq_norm_kernel<<<nchunks, 256, 0, stream>>>(chunks, tensors, acc);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

void mt_adamw_launch(const MTChunk* chunks, int nchunks, const MTTensor* tensors, const MTAdamWArgs& args,
                     cudaStream_t stream) {
  if (nchunks == 0) return;
  mt_adamw_kernel<<<nchunks, 256, 0, stream>>>(chunks, tensors, args);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

}  // namespace avgen
