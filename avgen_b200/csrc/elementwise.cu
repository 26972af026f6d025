// Bandwidth-bound elementwise kernels for sm_100a:
//   * SwiGLU / GELU-tanh backward on the GEMM-interleaved activation layout
//     (the forward halves live in the GEMM epilogue, gemm.cu)
//   * flow-matching loss partial sums and gradient
//     (avgen/train/objective.py:600-633, reduction 577-590)
//   * counter-based noise + rectified-flow interpolation for the local sequence
//     shard (avgen/train/objective.py:459-481): the draw for a token depends
//     only on (seed, offset, global token index, feature), so a context-parallel
//     rank producing its shard gets exactly the slice of the unsharded draw and
//     no rank draws the full sequence.
#include "include/host_utils.h"
#include "include/launchers.h"
#include "include/sm100.cuh"

namespace avgen {
namespace {

__device__ __forceinline__ float sigmoidf(float x) { return 1.f / (1.f + __expf(-x)); }

// dgu[:, 2j] = dh_j * up_j * sig(g)(1 + g(1 - sig(g))),  dgu[:, 2j+1] = dh_j * silu(g_j)
__global__ void swiglu_bwd_kernel(long rows, int F, const __nv_bfloat16* dh, long lddh,
                                  const __nv_bfloat16* gu, long ldgu, __nv_bfloat16* dgu,
                                  long lddgu) {
  const long pairs_per_row = F / 2;  // process 2 outputs (4 gu values) per thread
  const long total = rows * pairs_per_row;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long r = i / pairs_per_row;
    const long j = (i - r * pairs_per_row) * 2;
    const uint32_t dv = *reinterpret_cast<const uint32_t*>(dh + r * lddh + j);
    const uint2 gv = *reinterpret_cast<const uint2*>(gu + r * ldgu + 2 * j);
    const float d0 = bf16_lo(dv), d1 = bf16_hi(dv);
    const float g0 = bf16_lo(gv.x), u0 = bf16_hi(gv.x);
    const float g1 = bf16_lo(gv.y), u1 = bf16_hi(gv.y);
    const float s0 = sigmoidf(g0), s1 = sigmoidf(g1);
    uint2 o;
    o.x = pack_bf16(d0 * u0 * s0 * (1.f + g0 * (1.f - s0)), d0 * g0 * s0);
    o.y = pack_bf16(d1 * u1 * s1 * (1.f + g1 * (1.f - s1)), d1 * g1 * s1);
    *reinterpret_cast<uint2*>(dgu + r * lddgu + 2 * j) = o;
  }
}

__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float k0 = 0.7978845608028654f;
  const float k1 = 0.044715f;
  const float u = k0 * (x + k1 * x * x * x);
  const float t = tanhf(u);
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * k0 * (1.f + 3.f * k1 * x * x);
}

__global__ void gelu_bwd_kernel(long rows, int F, const __nv_bfloat16* dh, long lddh,
                                const __nv_bfloat16* pre, long ldpre, __nv_bfloat16* dpre,
                                long lddpre) {
  const long per_row = F / 2;
  const long total = rows * per_row;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long r = i / per_row;
    const long j = (i - r * per_row) * 2;
    const uint32_t dv = *reinterpret_cast<const uint32_t*>(dh + r * lddh + j);
    const uint32_t pv = *reinterpret_cast<const uint32_t*>(pre + r * ldpre + j);
    *reinterpret_cast<uint32_t*>(dpre + r * lddpre + j) =
        pack_bf16(bf16_lo(dv) * gelu_tanh_grad(bf16_lo(pv)), bf16_hi(dv) * gelu_tanh_grad(bf16_hi(pv)));
  }
}

__device__ __forceinline__ float load_elem(const void* p, bool f32, long idx) {
  return f32 ? reinterpret_cast<const float*>(p)[idx]
             : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[idx]);
}

// One warp per row: mse over P features, then block reduction and 3 atomics.
__global__ void __launch_bounds__(256) flow_loss_fwd_kernel(FlowLossDesc d) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float acc_w = 0.f, acc_r = 0.f, acc_m = 0.f;
  for (long row = static_cast<long>(blockIdx.x) * 8 + warp; row < d.rows;
       row += static_cast<long>(gridDim.x) * 8) {
    const float m = d.mask[row] ? 1.f : 0.f;
    float se = 0.f;
    for (int c = lane; c < d.P; c += 32) {
      const float diff = load_elem(d.pred, d.pred_f32, row * d.P + c) -
                         load_elem(d.target, d.target_f32, row * d.P + c);
      se += diff * diff;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
    const float mse = se / static_cast<float>(d.P);
    const float w = d.weight ? d.weight[row / d.rows_per_batch] : 1.f;
    acc_w += w * mse * m;
    acc_r += mse * m;
    acc_m += m;
  }
  __shared__ float red[3][8];
  if (lane == 0) {
    red[0][warp] = acc_w;
    red[1][warp] = acc_r;
    red[2][warp] = acc_m;
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[threadIdx.x][k];
    atomicAdd(d.stats + threadIdx.x, s);
  }
}

__global__ void flow_loss_bwd_kernel(FlowLossDesc d) {
  const float scale = d.scale[0] * 2.f / static_cast<float>(d.P);
  const long total = d.rows * d.P;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long row = i / d.P;
    const float m = d.mask[row] ? 1.f : 0.f;
    const float w = d.weight ? d.weight[row / d.rows_per_batch] : 1.f;
    const float g = scale * w * m * (load_elem(d.pred, d.pred_f32, i) - load_elem(d.target, d.target_f32, i));
    if (d.dpred_f32) reinterpret_cast<float*>(d.dpred)[i] = g;
    else reinterpret_cast<__nv_bfloat16*>(d.dpred)[i] = __float2bfloat16_rn(g);
  }
}

// Philox-4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy
// as 1, 2, 3", SC'11): ten rounds of two 32x32->64 multiplies with the Weyl key
// schedule, constants from that paper.
struct Philox {
  static constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;
  static constexpr uint32_t kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
  __device__ __forceinline__ static uint4 run(uint4 c, uint2 k) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
      const uint32_t lo0 = kM0 * c.x, hi0 = __umulhi(kM0, c.x);
      const uint32_t lo1 = kM1 * c.z, hi1 = __umulhi(kM1, c.z);
      c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
      k.x += kW0;
      k.y += kW1;
    }
    return c;
  }
};

__device__ __forceinline__ float u32_to_unit_open(uint32_t x) {
  // (0, 1]: never 0 so log() stays finite.
  return (static_cast<float>(x >> 8) + 1.0f) * (1.0f / 16777216.0f);
}

// Each thread produces 4 normals for 4 consecutive features of one row.
__global__ void noise_interp_kernel(NoiseDesc d) {
  const long quads_per_row = (d.P + 3) / 4;
  const long total = d.rows * quads_per_row;
  const uint2 key = make_uint2(static_cast<uint32_t>(d.seed), static_cast<uint32_t>(d.seed >> 32));
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long row = i / quads_per_row;
    const int q = static_cast<int>(i - row * quads_per_row);
    const long sample = row / d.rows_per_sample;
    const long grow = sample * d.global_rows_per_sample + d.row_base + (row - sample * d.rows_per_sample);
    const uint64_t ctr = d.offset + static_cast<uint64_t>(grow) * quads_per_row + q;
    const uint4 rnd = Philox::run(make_uint4(static_cast<uint32_t>(ctr), static_cast<uint32_t>(ctr >> 32), 0u, 0u), key);
    float z[4];
    {
      const float r0 = sqrtf(-2.f * logf(u32_to_unit_open(rnd.x)));
      float s0, c0;
      sincospif(2.f * u32_to_unit_open(rnd.y), &s0, &c0);
      const float r1 = sqrtf(-2.f * logf(u32_to_unit_open(rnd.z)));
      float s1, c1;
      sincospif(2.f * u32_to_unit_open(rnd.w), &s1, &c1);
      z[0] = r0 * c0; z[1] = r0 * s0; z[2] = r1 * c1; z[3] = r1 * s1;
    }
    const float t = d.t[row];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = q * 4 + e;
      if (c < d.P) {
        const long idx = row * d.P + c;
        const float x = load_elem(d.clean, d.clean_f32, idx);
        reinterpret_cast<float*>(d.noisy)[idx] = x + t * (z[e] - x);
        reinterpret_cast<float*>(d.target)[idx] = z[e] - x;
        if (d.noise) reinterpret_cast<float*>(d.noise)[idx] = z[e];
      }
    }
  }
}

long grid_for(long work, int device, int threads = 256) {
  const long want = (work + threads - 1) / threads;
  return std::max<long>(1, std::min<long>(want, 32L * num_sms(device)));
}

}  // namespace

void swiglu_bwd_launch(int device, long rows, int F, const void* dh, long lddh, const void* gu,
                       long ldgu, void* dgu, long lddgu, cudaStream_t stream) {
  AVGEN_CHECK(F % 2 == 0, "swiglu_bwd: hidden must be even");
  if (rows == 0) return;
  swiglu_bwd_kernel<<<grid_for(rows * F / 2, device), 256, 0, stream>>>(
      rows, F, reinterpret_cast<const __nv_bfloat16*>(dh), lddh,
      reinterpret_cast<const __nv_bfloat16*>(gu), ldgu, reinterpret_cast<__nv_bfloat16*>(dgu), lddgu);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

void gelu_bwd_launch(int device, long rows, int F, const void* dh, long lddh, const void* pre,
                     long ldpre, void* dpre, long lddpre, cudaStream_t stream) {
  AVGEN_CHECK(F % 2 == 0, "gelu_bwd: hidden must be even");
  if (rows == 0) return;
  gelu_bwd_kernel<<<grid_for(rows * F / 2, device), 256, 0, stream>>>(
      rows, F, reinterpret_cast<const __nv_bfloat16*>(dh), lddh,
      reinterpret_cast<const __nv_bfloat16*>(pre), ldpre, reinterpret_cast<__nv_bfloat16*>(dpre), lddpre);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

void flow_loss_fwd_launch(const FlowLossDesc& d, cudaStream_t stream) {
  if (d.rows == 0) return;
  const long blocks = std::max<long>(1, std::min<long>((d.rows + 7) / 8, 8L * num_sms(d.device)));
  flow_loss_fwd_kernel<<<blocks, 256, 0, stream>>>(d);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

void flow_loss_bwd_launch(const FlowLossDesc& d, cudaStream_t stream) {
  if (d.rows == 0) return;
  flow_loss_bwd_kernel<<<grid_for(d.rows * d.P, d.device), 256, 0, stream>>>(d);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

void noise_interp_launch(const NoiseDesc& d, cudaStream_t stream) {
  if (d.rows == 0) return;
  noise_interp_kernel<<<grid_for(d.rows * ((d.P + 3) / 4), d.device), 256, 0, stream>>>(d);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

}  // namespace avgen
