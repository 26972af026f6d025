// QK-RMSNorm + 3-D axial RoPE on the fused QKV projection (forward / backward).
//
// Replaces, for the self-attention of every DiT block, the sequence
//   q_norm / k_norm  (avgen/models/layers.py:530-536)
//   build_rotary_tables + apply_rotary (avgen/models/rope.py:218-338)
//   the (B, L, H, D) -> (B, H, L, D) transpose before SDPA
// with one pass: one warp per token reads the token's q, k and v heads from the
// QKV GEMM output, normalises q and k per head in fp32, rotates interleaved
// (even, odd) channel pairs by angles computed in-kernel from the token's
// physical coordinates (angle_j = coords[axis_j] * freq_j; the per-pair
// frequencies carry theta, time scaling and linear/NTK scaling), and writes
// head-major q, k, v for the attention kernels.
//
// Backward reverses it: inverse rotation, RMSNorm backward, norm-weight
// gradients reduced per warp and flushed with atomics, dQKV written in the GEMM
// layout so the QKV weight/input gradients are plain GEMMs.
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

// EPL = elements per lane = D / 32 (2 or 4), i.e. EPL/2 rotary pairs per lane.
template <int EPL>
__device__ __forceinline__ void load_vec(const __nv_bfloat16* p, float (&f)[EPL]) {
  if constexpr (EPL == 4) {
    const uint2 w = *reinterpret_cast<const uint2*>(p);
    f[0] = bf16_lo(w.x); f[1] = bf16_hi(w.x); f[2] = bf16_lo(w.y); f[3] = bf16_hi(w.y);
  } else {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
    f[0] = bf16_lo(w); f[1] = bf16_hi(w);
  }
}

template <int EPL>
__device__ __forceinline__ void store_vec(__nv_bfloat16* p, const float (&f)[EPL]) {
  if constexpr (EPL == 4) {
    uint2 w;
    w.x = pack_bf16(f[0], f[1]);
    w.y = pack_bf16(f[2], f[3]);
    *reinterpret_cast<uint2*>(p) = w;
  } else {
    *reinterpret_cast<uint32_t*>(p) = pack_bf16(f[0], f[1]);
  }
}

template <int EPL>
__global__ void __launch_bounds__(256) qkv_rope_fwd_kernel(QkvRopeDesc d) {
  constexpr int PPL = EPL / 2;
  const int lane = threadIdx.x & 31;
  const long warps_total = static_cast<long>(gridDim.x) * (blockDim.x >> 5);
  const long tokens = static_cast<long>(d.B) * d.L;
  float qw[EPL], kw[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    qw[e] = d.q_w ? d.q_w[lane * EPL + e] : 1.f;
    kw[e] = d.k_w ? d.k_w[lane * EPL + e] : 1.f;
  }
  float freq[PPL];
  int axis[PPL];
#pragma unroll
  for (int p = 0; p < PPL; ++p) {
    freq[p] = d.coords ? d.freq[lane * PPL + p] : 0.f;
    axis[p] = d.coords ? d.axis[lane * PPL + p] : 0;
  }
  for (long tok = static_cast<long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); tok < tokens;
       tok += warps_total) {
    const long b = tok / d.L;
    const long l = tok - b * d.L;
    float cs[PPL], sn[PPL];
#pragma unroll
    for (int p = 0; p < PPL; ++p) {
      if (d.coords) {
        const float ang = d.coords[tok * 3 + axis[p]] * freq[p];
        sincosf(ang, &sn[p], &cs[p]);
      } else {
        cs[p] = 1.f;
        sn[p] = 0.f;
      }
    }
    const __nv_bfloat16* row = reinterpret_cast<const __nv_bfloat16*>(d.qkv) + tok * d.ldqkv;
    const int heads_total = d.H + 2 * d.Hk;
    for (int h = 0; h < heads_total; ++h) {
      float x[EPL];
      load_vec<EPL>(row + static_cast<long>(h) * d.D + lane * EPL, x);
      const bool is_q = h < d.H;
      const bool is_k = !is_q && h < d.H + d.Hk;
      __nv_bfloat16* dst;
      if (is_q) {
        dst = reinterpret_cast<__nv_bfloat16*>(d.q) + ((b * d.H + h) * d.L + l) * d.D;
      } else if (is_k) {
        dst = reinterpret_cast<__nv_bfloat16*>(d.k) + ((b * d.Hk + (h - d.H)) * d.L + l) * d.D;
      } else {
        dst = reinterpret_cast<__nv_bfloat16*>(d.v) +
              ((b * d.Hk + (h - d.H - d.Hk)) * d.L + l) * d.D;
      }
      if (is_q || is_k) {
        const bool norm = is_q ? (d.q_w != nullptr) : (d.k_w != nullptr);
        if (norm) {
          float ss = 0.f;
#pragma unroll
          for (int e = 0; e < EPL; ++e) ss += x[e] * x[e];
          ss = warp_sum(ss);
          const float r = rsqrtf(ss / static_cast<float>(d.D) + d.eps);
#pragma unroll
          for (int e = 0; e < EPL; ++e) x[e] = x[e] * r * (is_q ? qw[e] : kw[e]);
        }
#pragma unroll
        for (int p = 0; p < PPL; ++p) {
          const float e0 = x[2 * p], e1 = x[2 * p + 1];
          x[2 * p] = e0 * cs[p] - e1 * sn[p];
          x[2 * p + 1] = e0 * sn[p] + e1 * cs[p];
        }
      }
      store_vec<EPL>(dst + lane * EPL, x);
    }
  }
}

template <int EPL>
__global__ void __launch_bounds__(256) qkv_rope_bwd_kernel(QkvRopeDesc d) {
  constexpr int PPL = EPL / 2;
  const int lane = threadIdx.x & 31;
  const long warps_total = static_cast<long>(gridDim.x) * (blockDim.x >> 5);
  const long tokens = static_cast<long>(d.B) * d.L;
  float qw[EPL], kw[EPL], dqw[EPL], dkw[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    qw[e] = d.q_w ? d.q_w[lane * EPL + e] : 1.f;
    kw[e] = d.k_w ? d.k_w[lane * EPL + e] : 1.f;
    dqw[e] = 0.f;
    dkw[e] = 0.f;
  }
  float freq[PPL];
  int axis[PPL];
#pragma unroll
  for (int p = 0; p < PPL; ++p) {
    freq[p] = d.coords ? d.freq[lane * PPL + p] : 0.f;
    axis[p] = d.coords ? d.axis[lane * PPL + p] : 0;
  }
  for (long tok = static_cast<long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); tok < tokens;
       tok += warps_total) {
    const long b = tok / d.L;
    const long l = tok - b * d.L;
    float cs[PPL], sn[PPL];
#pragma unroll
    for (int p = 0; p < PPL; ++p) {
      if (d.coords) {
        const float ang = d.coords[tok * 3 + axis[p]] * freq[p];
        sincosf(ang, &sn[p], &cs[p]);
      } else {
        cs[p] = 1.f;
        sn[p] = 0.f;
      }
    }
    const __nv_bfloat16* row = reinterpret_cast<const __nv_bfloat16*>(d.qkv) + tok * d.ldqkv;
    __nv_bfloat16* drow = reinterpret_cast<__nv_bfloat16*>(d.dqkv) + tok * d.lddqkv;
    const int heads_total = d.H + 2 * d.Hk;
    for (int h = 0; h < heads_total; ++h) {
      const bool is_q = h < d.H;
      const bool is_k = !is_q && h < d.H + d.Hk;
      const __nv_bfloat16* src;
      if (is_q) {
        src = reinterpret_cast<const __nv_bfloat16*>(d.dq) + ((b * d.H + h) * d.L + l) * d.D;
      } else if (is_k) {
        src = reinterpret_cast<const __nv_bfloat16*>(d.dk) + ((b * d.Hk + (h - d.H)) * d.L + l) * d.D;
      } else {
        src = reinterpret_cast<const __nv_bfloat16*>(d.dv) +
              ((b * d.Hk + (h - d.H - d.Hk)) * d.L + l) * d.D;
      }
      float g[EPL];
      load_vec<EPL>(src + lane * EPL, g);
      if (is_q || is_k) {
        // inverse rotation
#pragma unroll
        for (int p = 0; p < PPL; ++p) {
          const float g0 = g[2 * p], g1 = g[2 * p + 1];
          g[2 * p] = g0 * cs[p] + g1 * sn[p];
          g[2 * p + 1] = -g0 * sn[p] + g1 * cs[p];
        }
        const bool norm = is_q ? (d.q_w != nullptr) : (d.k_w != nullptr);
        if (norm) {
          float x[EPL];
          load_vec<EPL>(row + static_cast<long>(h) * d.D + lane * EPL, x);
          float ss = 0.f;
#pragma unroll
          for (int e = 0; e < EPL; ++e) ss += x[e] * x[e];
          ss = warp_sum(ss);
          const float r = rsqrtf(ss / static_cast<float>(d.D) + d.eps);
          float dot = 0.f;
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            const float n = x[e] * r;
            if (is_q) dqw[e] += g[e] * n; else dkw[e] += g[e] * n;
            g[e] *= is_q ? qw[e] : kw[e];
            x[e] = n;
            dot += g[e] * n;
          }
          dot = warp_sum(dot) / static_cast<float>(d.D);
#pragma unroll
          for (int e = 0; e < EPL; ++e) g[e] = r * (g[e] - x[e] * dot);
        }
      }
      store_vec<EPL>(drow + static_cast<long>(h) * d.D + lane * EPL, g);
    }
  }
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    if (d.dq_w) atomicAdd(d.dq_w + lane * EPL + e, dqw[e]);
    if (d.dk_w) atomicAdd(d.dk_w + lane * EPL + e, dkw[e]);
  }
}

}  // namespace

void qkv_rope_fwd_launch(const QkvRopeDesc& d, cudaStream_t stream) {
  AVGEN_CHECK(d.D == 64 || d.D == 128, "qkv_rope: head_dim must be 64 or 128, got ", d.D);
  const long tokens = static_cast<long>(d.B) * d.L;
  if (tokens == 0) return;
  const long blocks = std::min<long>((tokens + 7) / 8, 16L * num_sms(d.device));
  if (d.D == 128) qkv_rope_fwd_kernel<4><<<blocks, 256, 0, stream>>>(d);
  else qkv_rope_fwd_kernel<2><<<blocks, 256, 0, stream>>>(d);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

void qkv_rope_bwd_launch(const QkvRopeDesc& d, cudaStream_t stream) {
  AVGEN_CHECK(d.D == 64 || d.D == 128, "qkv_rope: head_dim must be 64 or 128, got ", d.D);
  const long tokens = static_cast<long>(d.B) * d.L;
  if (tokens == 0) return;
  const long blocks = std::min<long>((tokens + 7) / 8, 8L * num_sms(d.device));
  if (d.D == 128) qkv_rope_bwd_kernel<4><<<blocks, 256, 0, stream>>>(d);
  else qkv_rope_bwd_kernel<2><<<blocks, 256, 0, stream>>>(d);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

}  // namespace avgen
