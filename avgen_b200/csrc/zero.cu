// Sharded AdamW over NVLink peer memory (ZeRO-style, one node).
//
// Replaces, for the data-parallel gradient path, the reference's NCCL gradient
// all-reduce / reduce-scatter (avgen/parallel/fsdp.py reduce_dtype fp32) followed
// by a replicated optimizer step (avgen/train/optimizer.py:198-205). Each rank
// owns one contiguous shard of the flat fp32 parameter/gradient buffers and
// keeps Adam moments only for it:
//
//   shard_reduce     out[i] = (sum over ranks r of grad_r[lo + i]) / world, read
//                    from every peer's gradient buffer with loads over NVLink
//                    (the reduce-scatter), plus the squared-norm partial of the
//                    reduced shard for global gradient clipping;
//   shard_adamw_push AdamW on the shard (clip coefficient and non-finite skip
//                    read from device memory) that stores each updated
//                    parameter to this rank's buffer and to every peer's (the
//                    parameter all-gather fused into the update).
//
// The host orders the phases with one-word barriers: every rank's backward is
// complete before the pull, the norm all-reduce after it also marks every pull
// done, and a last barrier marks every push landed before the next forward.
#include "include/host_utils.h"
#include "include/launchers.h"
#include "include/sm100.cuh"

namespace avgen {
namespace {

constexpr int kMaxPeers = 16;

struct PeerPtrs {
  float* p[kMaxPeers];
};

__global__ void __launch_bounds__(256) shard_reduce_kernel(PeerPtrs grads, int world, long lo, long n4,
                                                           float inv_world, float* out, float* sq_acc) {
  float s = 0.f;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      const float4 v = reinterpret_cast<const float4*>(grads.p[r] + lo)[i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    acc.x *= inv_world;
    acc.y *= inv_world;
    acc.z *= inv_world;
    acc.w *= inv_world;
    reinterpret_cast<float4*>(out)[i] = acc;
    s += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) atomicAdd(sq_acc, t);
  }
}

__global__ void __launch_bounds__(256) shard_adamw_push_kernel(ShardAdamWDesc d, PeerPtrs params) {
  const bool zero_grads = d.skip != nullptr && *d.skip != 0;
  const float gscale = zero_grads ? 0.f : (d.grad_scale ? *d.grad_scale : 1.f);
  const float step_lr = d.lr / d.bias_correction1;
  const float decay = 1.f - d.lr * d.weight_decay;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < d.n4; i += stride) {
    float4 p = reinterpret_cast<const float4*>(params.p[d.rank] + d.lo)[i];
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
    reinterpret_cast<float4*>(d.exp_avg)[i] = make_float4(mv[0], mv[1], mv[2], mv[3]);
    reinterpret_cast<float4*>(d.exp_avg_sq)[i] = make_float4(vv[0], vv[1], vv[2], vv[3]);
    const float4 out = make_float4(pv[0], pv[1], pv[2], pv[3]);
    for (int r = 0; r < d.world; ++r) {  // this rank first is not needed: stores are independent
      reinterpret_cast<float4*>(params.p[r] + d.lo)[i] = out;
    }
  }
  __threadfence_system();  // the pushes are visible system-wide before the kernel's completion is observed
}

PeerPtrs pack_ptrs(const float* const* ptrs, int world) {
  AVGEN_CHECK(world >= 1 && world <= kMaxPeers, "sharded AdamW: 1..", kMaxPeers, " ranks supported, got ", world);
  PeerPtrs out{};
  for (int r = 0; r < world; ++r) {
    AVGEN_CHECK((reinterpret_cast<uintptr_t>(ptrs[r]) & 15u) == 0, "sharded AdamW: buffers must be 16-byte aligned");
    out.p[r] = const_cast<float*>(ptrs[r]);
  }
  return out;
}

long blocks_for(long n4, int device) {
  return std::max<long>(1, std::min<long>((n4 + 255) / 256, 8L * num_sms(device)));
}

}  // namespace

void shard_reduce_launch(const float* const* grads, int world, long lo, long n, float* out, float* sq_acc, int device,
                         cudaStream_t stream) {
  AVGEN_CHECK(n % 4 == 0 && lo % 4 == 0, "shard_reduce: shard bounds must be multiples of 4 elements");
  if (n == 0) return;
  const PeerPtrs p = pack_ptrs(grads, world);
  shard_reduce_kernel<<<blocks_for(n / 4, device), 256, 0, stream>>>(p, world, lo, n / 4, 1.f / world, out, sq_acc);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

void shard_adamw_push_launch(const ShardAdamWDesc& d, const float* const* params, cudaStream_t stream) {
  AVGEN_CHECK(d.n4 >= 0 && d.lo % 4 == 0, "shard_adamw_push: shard bounds must be multiples of 4 elements");
  if (d.n4 == 0) return;
  const PeerPtrs p = pack_ptrs(params, d.world);
  shard_adamw_push_kernel<<<blocks_for(d.n4, d.device), 256, 0, stream>>>(d, p);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

}  // namespace avgen
