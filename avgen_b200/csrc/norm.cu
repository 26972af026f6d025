// adaLN RMSNorm kernels (forward / backward) for sm_100a.
//
// Forward, one warp per row (fp32 statistics, one rounding to bf16 at the end):
//   y = rmsnorm(x) * w * (1 + scale[b]) + shift[b]
// which fuses FusedRMSNorm (avgen/models/layers.py:106-118) with `modulate`
// (avgen/models/layers.py:210-229) as DiTBlock.forward applies them
// (avgen/models/blocks.py:207-216). With scale/shift absent it is a plain
// RMSNorm (cross_norm, final_norm, SP-local norms).
//
// Backward is split in two bandwidth-bound passes:
//   * rows:    dx = rstd * (g - n * mean(g * n)),  g = dy * w * (1 + scale)
//              (optionally added to an incoming residual gradient)
//   * columns: dw, dscale[b], dshift[b] as column sums over each batch's rows,
//              reduced in shared memory and flushed with fp32 atomics.
// The same column pass computes the gated-residual backward
//   da = dx * gate[b];  dgate[b] += sum_rows dx * a
// of `hidden + gate * f(...)` (avgen/models/blocks.py:216,227).
#include <algorithm>

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

__device__ __forceinline__ void unpack8(const uint4& w, float* f) {
  f[0] = bf16_lo(w.x); f[1] = bf16_hi(w.x);
  f[2] = bf16_lo(w.y); f[3] = bf16_hi(w.y);
  f[4] = bf16_lo(w.z); f[5] = bf16_hi(w.z);
  f[6] = bf16_lo(w.w); f[7] = bf16_hi(w.w);
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 w;
  w.x = pack_bf16(f[0], f[1]);
  w.y = pack_bf16(f[2], f[3]);
  w.z = pack_bf16(f[4], f[5]);
  w.w = pack_bf16(f[6], f[7]);
  return w;
}

__device__ __forceinline__ void load8f(const float* p, float* f) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

template <int VPL>
__global__ void __launch_bounds__(256) rmsnorm_mod_fwd_kernel(NormDesc d) {
  const int warps = blockDim.x >> 5;
  const long row = static_cast<long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= d.rows) return;
  const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(d.x) + row * d.ldx;
  float v[VPL][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d.W) {
      unpack8(*reinterpret_cast<const uint4*>(xr + c), v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(d.W) + d.eps);
  const long b = mod_row(d.groups, d.num_groups, row, d.rows_per_batch);
  __nv_bfloat16* yr = reinterpret_cast<__nv_bfloat16*>(d.y) + row * d.ldy;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d.W) {
      float o[8], t[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[i][e] * r;
      if (d.w != nullptr) {
        load8f(d.w + c, t);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] *= t[e];
      }
      if (d.scale != nullptr) {
        load8f(d.scale + b * d.mod_stride + c, t);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] *= 1.f + t[e];
      }
      if (d.shift != nullptr) {
        load8f(d.shift + b * d.mod_stride + c, t);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] += t[e];
      }
      *reinterpret_cast<uint4*>(yr + c) = pack8(o);
    }
  }
  if (lane == 0 && d.rstd != nullptr) d.rstd[row] = r;
}

template <int VPL>
__global__ void __launch_bounds__(256) rmsnorm_mod_bwd_rows_kernel(NormDesc d) {
  const int warps = blockDim.x >> 5;
  const long row = static_cast<long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= d.rows) return;
  const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(d.x) + row * d.ldx;
  const __nv_bfloat16* dyr = reinterpret_cast<const __nv_bfloat16*>(d.dy) + row * d.lddy;
  const float r = d.rstd[row];
  const long b = mod_row(d.groups, d.num_groups, row, d.rows_per_batch);
  float n[VPL][8], g[VPL][8];
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d.W) {
      unpack8(*reinterpret_cast<const uint4*>(xr + c), n[i]);
      unpack8(*reinterpret_cast<const uint4*>(dyr + c), g[i]);
      float t[8];
      if (d.w != nullptr) {
        load8f(d.w + c, t);
#pragma unroll
        for (int e = 0; e < 8; ++e) g[i][e] *= t[e];
      }
      if (d.scale != nullptr) {
        load8f(d.scale + b * d.mod_stride + c, t);
#pragma unroll
        for (int e = 0; e < 8; ++e) g[i][e] *= 1.f + t[e];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        n[i][e] *= r;
        dot += g[i][e] * n[i][e];
      }
    }
  }
  dot = warp_sum(dot) / static_cast<float>(d.W);
  __nv_bfloat16* dxr = reinterpret_cast<__nv_bfloat16*>(d.dx) + row * d.lddx;
  const __nv_bfloat16* resr =
      d.dres != nullptr ? reinterpret_cast<const __nv_bfloat16*>(d.dres) + row * d.lddres : nullptr;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d.W) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = r * (g[i][e] - n[i][e] * dot);
      if (resr != nullptr) {
        float t[8];
        unpack8(*reinterpret_cast<const uint4*>(resr + c), t);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] += t[e];
      }
      *reinterpret_cast<uint4*>(dxr + c) = pack8(o);
    }
  }
}

// Column pass. Block: 256 threads = 32 column pairs x 8 row lanes, covering 64
// columns; grid = (ceil(W/64), batches, row splits).
__global__ void __launch_bounds__(256) rmsnorm_mod_bwd_cols_kernel(NormDesc d, int splits) {
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 64 + tx * 2;
  const long b = blockIdx.y;
  const long rows_b = d.rows_per_batch;
  const long chunk = (rows_b + splits - 1) / splits;
  const long r0 = b * rows_b + blockIdx.z * chunk;
  const long r1 = min(b * rows_b + rows_b, min(r0 + chunk, static_cast<long>(d.rows)));
  float acc_w[2] = {0.f, 0.f}, acc_s[2] = {0.f, 0.f}, acc_t[2] = {0.f, 0.f};
  const bool col_ok = c < d.W;
  float w0 = 1.f, w1 = 1.f, s0 = 0.f, s1 = 0.f;
  if (col_ok) {
    if (d.w != nullptr) { w0 = d.w[c]; w1 = d.w[c + 1]; }
    if (d.scale != nullptr) { s0 = d.scale[b * d.mod_stride + c]; s1 = d.scale[b * d.mod_stride + c + 1]; }
  }
  if (col_ok) {
    for (long row = r0 + ty; row < r1; row += 8) {
      const uint32_t xv = *reinterpret_cast<const uint32_t*>(
          reinterpret_cast<const __nv_bfloat16*>(d.x) + row * d.ldx + c);
      const uint32_t gv = *reinterpret_cast<const uint32_t*>(
          reinterpret_cast<const __nv_bfloat16*>(d.dy) + row * d.lddy + c);
      const float r = d.rstd[row];
      const float n0 = bf16_lo(xv) * r, n1 = bf16_hi(xv) * r;
      const float g0 = bf16_lo(gv), g1 = bf16_hi(gv);
      acc_t[0] += g0; acc_t[1] += g1;
      acc_s[0] += g0 * n0 * w0; acc_s[1] += g1 * n1 * w1;
      acc_w[0] += g0 * n0 * (1.f + s0); acc_w[1] += g1 * n1 * (1.f + s1);
    }
  }
  __shared__ float red[3][8][64];
  red[0][ty][tx * 2] = acc_w[0]; red[0][ty][tx * 2 + 1] = acc_w[1];
  red[1][ty][tx * 2] = acc_s[0]; red[1][ty][tx * 2 + 1] = acc_s[1];
  red[2][ty][tx * 2] = acc_t[0]; red[2][ty][tx * 2 + 1] = acc_t[1];
  __syncthreads();
  if (threadIdx.x < 192) {
    const int which = threadIdx.x / 64;
    const int col = threadIdx.x % 64;
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[which][k][col];
    const int cc = blockIdx.x * 64 + col;
    if (cc < d.W) {
      if (which == 0 && d.dw != nullptr) atomicAdd(d.dw + cc, s);
      if (which == 1 && d.dscale != nullptr) atomicAdd(d.dscale + b * d.dmod_stride + cc, s);
      if (which == 2 && d.dshift != nullptr) atomicAdd(d.dshift + b * d.dmod_stride + cc, s);
    }
  }
}

// Column pass when rows map to modulation rows by `groups` (or by row /
// rows_per_batch with small batches). A CTA's row range may then cross several groups: every thread keeps running sums for the
// group of its current row and adds them to global memory when the group changes
// or the range ends. Groups are piecewise constant along rows (a sample's clean
// and noisy frames), so flushes are rare. Grid = (ceil(W/64), 1, row splits).
__global__ void __launch_bounds__(256) rmsnorm_mod_bwd_cols_grouped_kernel(NormDesc d, int splits) {
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 64 + tx * 2;
  if (c >= d.W) return;  // no block-wide barrier below
  const long chunk = (d.rows + splits - 1) / splits;
  const long r0 = blockIdx.z * chunk;
  const long r1 = min(r0 + chunk, static_cast<long>(d.rows));
  float w0 = 1.f, w1 = 1.f;
  if (d.w != nullptr) { w0 = d.w[c]; w1 = d.w[c + 1]; }
  float acc_w[2] = {0.f, 0.f}, acc_s[2] = {0.f, 0.f}, acc_t[2] = {0.f, 0.f};
  long g = -1;
  float s0 = 0.f, s1 = 0.f;
  auto flush = [&]() {
    if (g < 0) return;
    if (d.dscale != nullptr) {
      atomicAdd(d.dscale + g * d.dmod_stride + c, acc_s[0]);
      atomicAdd(d.dscale + g * d.dmod_stride + c + 1, acc_s[1]);
    }
    if (d.dshift != nullptr) {
      atomicAdd(d.dshift + g * d.dmod_stride + c, acc_t[0]);
      atomicAdd(d.dshift + g * d.dmod_stride + c + 1, acc_t[1]);
    }
    acc_s[0] = acc_s[1] = acc_t[0] = acc_t[1] = 0.f;
  };
  for (long row = r0 + ty; row < r1; row += 8) {
    const long gr = mod_row(d.groups, d.num_groups, row, d.rows_per_batch);
    if (gr != g) {
      flush();
      g = gr;
      if (d.scale != nullptr) { s0 = d.scale[g * d.mod_stride + c]; s1 = d.scale[g * d.mod_stride + c + 1]; }
    }
    const uint32_t xv = *reinterpret_cast<const uint32_t*>(
        reinterpret_cast<const __nv_bfloat16*>(d.x) + row * d.ldx + c);
    const uint32_t gv = *reinterpret_cast<const uint32_t*>(
        reinterpret_cast<const __nv_bfloat16*>(d.dy) + row * d.lddy + c);
    const float r = d.rstd[row];
    const float n0 = bf16_lo(xv) * r, n1 = bf16_hi(xv) * r;
    const float g0 = bf16_lo(gv), g1 = bf16_hi(gv);
    acc_t[0] += g0; acc_t[1] += g1;
    acc_s[0] += g0 * n0 * w0; acc_s[1] += g1 * n1 * w1;
    acc_w[0] += g0 * n0 * (1.f + s0); acc_w[1] += g1 * n1 * (1.f + s1);
  }
  flush();
  if (d.dw != nullptr) {
    atomicAdd(d.dw + c, acc_w[0]);
    atomicAdd(d.dw + c + 1, acc_w[1]);
  }
}

// da = dx * gate[b];  dgate[b] += sum_rows dx * a.   Same tiling as above.
__global__ void __launch_bounds__(256) gate_bwd_kernel(GateBwdDesc d, int splits) {
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 64 + tx * 2;
  const long b = blockIdx.y;
  const long rows_b = d.rows_per_batch;
  const long chunk = (rows_b + splits - 1) / splits;
  const long r0 = b * rows_b + blockIdx.z * chunk;
  const long r1 = min(b * rows_b + rows_b, min(r0 + chunk, static_cast<long>(d.rows)));
  float acc[2] = {0.f, 0.f};
  if (c < d.W) {
    const float g0 = d.gate[b * d.gate_stride + c], g1 = d.gate[b * d.gate_stride + c + 1];
    for (long row = r0 + ty; row < r1; row += 8) {
      const uint32_t dv = *reinterpret_cast<const uint32_t*>(
          reinterpret_cast<const __nv_bfloat16*>(d.dx) + row * d.lddx + c);
      const uint32_t av = *reinterpret_cast<const uint32_t*>(
          reinterpret_cast<const __nv_bfloat16*>(d.a) + row * d.lda + c);
      const float d0 = bf16_lo(dv), d1 = bf16_hi(dv);
      acc[0] += d0 * bf16_lo(av);
      acc[1] += d1 * bf16_hi(av);
      *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(d.da) + row * d.ldda + c) =
          pack_bf16(d0 * g0, d1 * g1);
    }
  }
  __shared__ float red[8][64];
  red[ty][tx * 2] = acc[0];
  red[ty][tx * 2 + 1] = acc[1];
  __syncthreads();
  if (threadIdx.x < 64) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[k][threadIdx.x];
    const int cc = blockIdx.x * 64 + threadIdx.x;
    if (cc < d.W) atomicAdd(d.dgate + b * d.dgate_stride + cc, s);
  }
}

// Grouped variant of gate_bwd_kernel (see rmsnorm_mod_bwd_cols_grouped_kernel).
__global__ void __launch_bounds__(256) gate_bwd_grouped_kernel(GateBwdDesc d, int splits) {
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 64 + tx * 2;
  if (c >= d.W) return;
  const long chunk = (d.rows + splits - 1) / splits;
  const long r0 = blockIdx.z * chunk;
  const long r1 = min(r0 + chunk, static_cast<long>(d.rows));
  float acc[2] = {0.f, 0.f};
  long g = -1;
  float g0 = 0.f, g1 = 0.f;
  for (long row = r0 + ty; row < r1; row += 8) {
    const long gr = mod_row(d.groups, d.num_groups, row, d.rows_per_batch);
    if (gr != g) {
      if (g >= 0) {
        atomicAdd(d.dgate + g * d.dgate_stride + c, acc[0]);
        atomicAdd(d.dgate + g * d.dgate_stride + c + 1, acc[1]);
      }
      acc[0] = acc[1] = 0.f;
      g = gr;
      g0 = d.gate[g * d.gate_stride + c];
      g1 = d.gate[g * d.gate_stride + c + 1];
    }
    const uint32_t dv = *reinterpret_cast<const uint32_t*>(
        reinterpret_cast<const __nv_bfloat16*>(d.dx) + row * d.lddx + c);
    const uint32_t av = *reinterpret_cast<const uint32_t*>(
        reinterpret_cast<const __nv_bfloat16*>(d.a) + row * d.lda + c);
    const float d0 = bf16_lo(dv), d1 = bf16_hi(dv);
    acc[0] += d0 * bf16_lo(av);
    acc[1] += d1 * bf16_hi(av);
    *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(d.da) + row * d.ldda + c) =
        pack_bf16(d0 * g0, d1 * g1);
  }
  if (g >= 0) {
    atomicAdd(d.dgate + g * d.dgate_stride + c, acc[0]);
    atomicAdd(d.dgate + g * d.dgate_stride + c + 1, acc[1]);
  }
}

int grouped_splits(long rows, int col_tiles, int sms) {
  long s = (4L * sms) / std::max(1, col_tiles);
  return static_cast<int>(std::max(1L, std::min(s, (rows + 63) / 64)));
}

int pick_vpl(int W) {
  const int need = (W + 255) / 256;
  const int opts[] = {1, 2, 4, 8, 12, 16, 20, 24};
  for (int o : opts)
    if (o >= need) return o;
  return -1;
}

int column_splits(long rows_per_batch, int col_tiles, int batches, int sms) {
  const long target_blocks = 4L * sms;
  long s = target_blocks / std::max(1, col_tiles * batches);
  s = std::max(1L, std::min(s, (rows_per_batch + 63) / 64));
  return static_cast<int>(s);
}

}  // namespace

#define AVGEN_VPL_SWITCH(VPL, ...)                \
  switch (VPL) {                                  \
    case 1: { constexpr int V = 1; __VA_ARGS__; break; }   \
    case 2: { constexpr int V = 2; __VA_ARGS__; break; }   \
    case 4: { constexpr int V = 4; __VA_ARGS__; break; }   \
    case 8: { constexpr int V = 8; __VA_ARGS__; break; }   \
    case 12: { constexpr int V = 12; __VA_ARGS__; break; } \
    case 16: { constexpr int V = 16; __VA_ARGS__; break; } \
    case 20: { constexpr int V = 20; __VA_ARGS__; break; } \
    case 24: { constexpr int V = 24; __VA_ARGS__; break; } \
    default: AVGEN_CHECK(false, "norm: width too large"); \
  }

void rmsnorm_mod_fwd_launch(const NormDesc& d, cudaStream_t stream) {
  AVGEN_CHECK(d.W % 8 == 0, "norm: width must be a multiple of 8");
  if (d.rows == 0) return;
  const int vpl = pick_vpl(d.W);
  const int threads = 256;
  const long blocks = (d.rows + 7) / 8;
  AVGEN_VPL_SWITCH(vpl, rmsnorm_mod_fwd_kernel<V><<<blocks, threads, 0, stream>>>(d));
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

// The per-batch column kernels put one batch per grid row (y <= 65535) and want
// many rows per batch; otherwise the run-flushing kernels take over.
constexpr long kMinRowsPerBatch = 256;

void rmsnorm_mod_bwd_launch(const NormDesc& d_in, cudaStream_t stream) {
  NormDesc d = d_in;
  // without modulation only dw is reduced: one batch spanning every row
  if (d.scale == nullptr && d.shift == nullptr && d.groups == nullptr) d.rows_per_batch = d.rows;
  AVGEN_CHECK(d.W % 8 == 0, "norm: width must be a multiple of 8");
  if (d.rows == 0) return;
  const int vpl = pick_vpl(d.W);
  const long blocks = (d.rows + 7) / 8;
  if (d.dx != nullptr) {
    AVGEN_VPL_SWITCH(vpl, rmsnorm_mod_bwd_rows_kernel<V><<<blocks, 256, 0, stream>>>(d));
    AVGEN_CUDA_CHECK(cudaGetLastError());
  }
  const bool irregular = d.groups != nullptr || d.rows_per_batch < kMinRowsPerBatch;
  if (irregular && (d.dw != nullptr || d.dscale != nullptr || d.dshift != nullptr)) {
    const int col_tiles = (d.W + 63) / 64;
    const int splits = grouped_splits(d.rows, col_tiles, num_sms(d.device));
    rmsnorm_mod_bwd_cols_grouped_kernel<<<dim3(col_tiles, 1, splits), 256, 0, stream>>>(d, splits);
    AVGEN_CUDA_CHECK(cudaGetLastError());
  } else if (d.dw != nullptr || d.dscale != nullptr || d.dshift != nullptr) {
    const int col_tiles = (d.W + 63) / 64;
    const int batches = static_cast<int>((d.rows + d.rows_per_batch - 1) / d.rows_per_batch);
    const int splits = column_splits(d.rows_per_batch, col_tiles, batches, num_sms(d.device));
    dim3 grid(col_tiles, batches, splits);
    rmsnorm_mod_bwd_cols_kernel<<<grid, 256, 0, stream>>>(d, splits);
    AVGEN_CUDA_CHECK(cudaGetLastError());
  }
}

void gate_bwd_launch(const GateBwdDesc& d, cudaStream_t stream) {
  AVGEN_CHECK(d.W % 2 == 0, "gate_bwd: width must be even");
  if (d.rows == 0) return;
  const int col_tiles = (d.W + 63) / 64;
  if (d.groups != nullptr || d.rows_per_batch < kMinRowsPerBatch) {
    const int splits = grouped_splits(d.rows, col_tiles, num_sms(d.device));
    gate_bwd_grouped_kernel<<<dim3(col_tiles, 1, splits), 256, 0, stream>>>(d, splits);
    AVGEN_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int batches = static_cast<int>((d.rows + d.rows_per_batch - 1) / d.rows_per_batch);
  const int splits = column_splits(d.rows_per_batch, col_tiles, batches, num_sms(d.device));
  dim3 grid(col_tiles, batches, splits);
  gate_bwd_kernel<<<grid, 256, 0, stream>>>(d, splits);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

}  // namespace avgen
