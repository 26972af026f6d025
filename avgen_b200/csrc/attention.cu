// Flash attention for sm_100a on tcgen05 tensor cores (head_dim 128, bf16).
//
// Replaces the SDPA call of avgen/models/attention.py:227-273 (self-attention of
// every DiT block and cross-attention to the text tokens) with hand-written
// Blackwell kernels. Bidirectional, optional key-padding mask (packed bits),
// grouped-query attention (H query heads over Hk key/value heads).
//
// Forward (one CTA = one (batch, head) and 256 query rows = two 128-row tiles):
//   warp 0      TMA: Q tiles once, then K/V blocks of 128 keys into a 2-stage ring
//   warp 1      MMA: S_g = Q_g K^T into TMEM; O_g += P_g V with P read from TMEM
//   warps 4..11 two softmax warpgroups, one per query tile; thread = query row
// The two tiles ping-pong on the tensor core (S of one tile is computed while
// the other tile's softmax runs). P overwrites S in place (bf16 packed two per
// 32-bit column). The running max is only moved when it grows by more than 8
// (log2 units); O in TMEM is rescaled only then, after the pending PV finished.
// Scores use the base-2 domain: s2 = (q.k) * scale * log2(e), lse2 = m + log2(l).
//
// Backward (one CTA = one (batch, kv head) and 128 keys, looping over query
// blocks of every query head that reads this kv head):
//   S^T = K Q^T and dP^T = V dO^T into TMEM; one warpgroup (thread = key row)
//   forms P^T = exp2(s2 - lse2) and dS^T = P^T (dP^T - delta); dV += P^T dO and
//   dK += dS^T Q read P^T / dS^T from TMEM; dQ = dS K reads dS from shared
//   memory and is flushed to an fp32 accumulator with vector atomics.
#include <algorithm>
#include <cfloat>

#include "include/host_utils.h"
#include "include/launchers.h"
#include "include/sm100.cuh"

namespace avgen {
namespace {

constexpr int kHD = 128;
constexpr int kTile = 128;
constexpr float kNegBig = -1.0e30f;
constexpr float kRescaleThreshold = 8.0f;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

// K-major SW128 descriptor for a 128-row x 128-element tile stored as two
// 64-element column chunks of 16 KB; k-step kk (16 elements) of 8.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, int kk) {
  return umma_desc_sw128(tile + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
}
// The same tile read MN-major (rows are the reduction axis): k-step kk covers
// rows 16kk..16kk+15; the two 64-element MN chunks are 16 KB apart.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile, int kk) {
  return umma_desc_sw128(tile + kk * 2048, 16384, 1024);
}

// =========================================================================== forward
struct FwdSmem {
  static constexpr int Q = 0;            // 2 tiles x 32 KB
  static constexpr int KV = 65536;       // 2 stages x (K 32 KB + V 32 KB)
  static constexpr int BARS = 65536 + 131072;
  static constexpr int BYTES = BARS + 256 + 1024;
};

// kTrace compiles the diagnostic clock stamps in; the production instance has none of them.
template <bool kTrace>
__global__ void __launch_bounds__(384, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnFwdDesc p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FwdSmem::BARS);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 3;
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 7;
  uint64_t* o_done = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int qt = blockIdx.x % p.q_tiles;
  const int bh = blockIdx.x / p.q_tiles;
  const int h = bh % p.H;
  const int b = bh / p.H;
  const int hk = h / (p.H / p.Hk);
  const int q0 = qt * 256;
  const int nkv = (p.Lk + kTile - 1) / kTile;
  const bool ring = p.ring_world > 1;
  const int ring_tiles = ring ? p.ring_len / kTile : nkv;  // key tiles per rank's chunk
  const int ring_start = ring ? p.ring_rank * ring_tiles : 0;
  // diagnostics: SM clock stamps of CTA 0, 24 per key tile, first 64 tiles. Slots: 0/1/2 MMA
  // thread passes p_full[0] / kv_full(j+1) / p_full[1]; 3-8 softmax group 0 (S seen, loaded,
  // max, rescaled, exponentials, arrive), 9-14 the same for group 1; 15/16 S/PV of group 0
  // complete, 17/18 of group 1 (the tracer waits in order, so 15 can lag).
  long long* trace = (kTrace && blockIdx.x == 0) ? p.trace : nullptr;
  auto stamp = [&](int j, int slot) {
    if (trace != nullptr && j < 64) trace[j * 24 + slot] = clock64();
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 128);
      mbar_init(&o_done[s], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, 65536);
      for (int g = 0; g < 2; ++g)
        for (int c = 0; c < 2; ++c)
          tma_load_3d(smem + FwdSmem::Q + g * 32768 + c * 16384, &tmQ, q_full, c * 64, q0 + g * 128,
                      b * p.H + h);
      for (int j = 0; j < nkv; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, p.err, kErrTimeoutProducer)) break;
        int row = j * kTile, slab = b * p.Hk + hk;
        if (ring) {
          const int g = (j + ring_start) % nkv;  // global key tile
          const int r = g / ring_tiles;
          row = (g - r * ring_tiles) * kTile;
          slab += r * p.B * p.Hk;
          if (r != p.ring_rank && row == 0) {
            const long long t0 = clock64();
            if (!flag_wait_geq(p.ring_flags + r, p.ring_epoch, abort_flag, p.err, kErrTimeoutPeer)) break;
            if (p.wait_cycles != nullptr)
              atomicAdd(p.wait_cycles, static_cast<unsigned long long>(clock64() - t0));
          }
        }
        mbar_arrive_expect_tx(&kv_full[s], 65536);
        uint8_t* st = smem + FwdSmem::KV + s * 65536;
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(st + c * 16384, &tmK, &kv_full[s], c * 64, row, slab);
          tma_load_3d(st + 32768 + c * 16384, &tmV, &kv_full[s], c * 64, row, slab);
        }
      }
    }
  } else if (warp == 1) {
    const uint32_t idS = idesc_bf16_f32(128, 128, false, false);
    const uint32_t idO = idesc_bf16_f32(128, 128, false, true);
    const uint32_t sQ = smem_u32(smem + FwdSmem::Q);
    const uint32_t sKV = smem_u32(smem + FwdSmem::KV);
    auto issue_S = [&](int g, int s) {
      const uint32_t qa = sQ + g * 32768;
      const uint32_t ka = sKV + s * 65536;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_bf16_ss(tmem + g * 128, kmajor_desc(qa, kk), kmajor_desc(ka, kk), idS, kk > 0 ? 1u : 0u);
    };
    auto issue_PV = [&](int g, int s, bool acc) {
      const uint32_t va = sKV + s * 65536 + 32768;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_bf16_ts(tmem + 256 + g * 128, tmem + g * 128 + kk * 8, mnmajor_desc(va, kk), idO,
                    (acc || kk > 0) ? 1u : 0u);
    };
    bool ok = mbar_wait(q_full, 0, abort_flag, p.err, kErrTimeoutMma) &&
              mbar_wait(&kv_full[0], 0, abort_flag, p.err, kErrTimeoutMma);
    if (ok) {
      tc_fence_after();
      if (elect_one()) {
        issue_S(0, 0);
        mma_commit(&s_full[0]);
        issue_S(1, 0);
        mma_commit(&s_full[1]);
      }
      __syncwarp();
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j & 1;
        const int s2 = (j + 1) & 1;
        if (!mbar_wait(&p_full[0], j & 1, abort_flag, p.err, kErrTimeoutMma)) break;
        tc_fence_after();
        if (lane == 0) stamp(j, 0);
        if (elect_one()) {
          issue_PV(0, s, j > 0);
          mma_commit(&o_done[0]);
        }
        __syncwarp();
        const bool more = j + 1 < nkv;
        if (more) {
          if (!mbar_wait(&kv_full[s2], ((j + 1) >> 1) & 1, abort_flag, p.err, kErrTimeoutMma)) break;
          tc_fence_after();
          if (lane == 0) stamp(j, 1);
          if (elect_one()) {
            issue_S(0, s2);
            mma_commit(&s_full[0]);
          }
          __syncwarp();
        }
        if (!mbar_wait(&p_full[1], j & 1, abort_flag, p.err, kErrTimeoutMma)) break;
        tc_fence_after();
        if (lane == 0) stamp(j, 2);
        if (elect_one()) {
          issue_PV(1, s, j > 0);
          mma_commit(&o_done[1]);
          mma_commit(&kv_empty[s]);
          if (more) {
            issue_S(1, s2);
            mma_commit(&s_full[1]);
          }
        }
        __syncwarp();
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ diagnostics: MMA completion stamps
    if (trace != nullptr && lane == 0) {
      for (int j = 0; j < nkv && j < 64; ++j) {
        const uint32_t ph = j & 1;
        if (!mbar_wait(&s_full[0], ph, abort_flag, p.err, kErrTimeoutEpilogue)) break;
        stamp(j, 15);
        if (!mbar_wait(&s_full[1], ph, abort_flag, p.err, kErrTimeoutEpilogue)) break;
        stamp(j, 17);
        if (!mbar_wait(&o_done[0], ph, abort_flag, p.err, kErrTimeoutEpilogue)) break;
        stamp(j, 16);
        if (!mbar_wait(&o_done[1], ph, abort_flag, p.err, kErrTimeoutEpilogue)) break;
        stamp(j, 18);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    const int g = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int q = q0 + g * 128 + row;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_base + g * 128;
    const uint32_t tO = tmem + lane_base + 256 + g * 128;
    const float sl = p.scale_log2;
    float m = kNegBig;
    float l = 0.f;
    bool ok = true;
    const bool tr = kTrace && (warp & 3) == 0 && lane == 0;  // warps 4 and 8 stamp for their group
    const int ts = 3 + 6 * g;
    for (int j = 0; j < nkv; ++j) {
      if (!mbar_wait(&s_full[g], j & 1, abort_flag, p.err, kErrTimeoutSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (tr) stamp(j, ts);
      // key-validity words of this tile, loaded before the TMEM read so their latency overlaps it
      const int kbase = (ring ? (j + ring_start) % nkv : j) * kTile;
      const bool check_keys = kbase + kTile > p.Lk || p.kmask != nullptr;
      uint32_t words[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
      if (check_keys) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int key0 = kbase + 32 * w;
          uint32_t bits = 0xffffffffu;
          if (p.kmask != nullptr && key0 < p.Lk) bits = p.kmask[static_cast<long>(b) * p.kmask_words + (key0 >> 5)];
          const int left = p.Lk - key0;
          if (left < 32) bits &= (left <= 0) ? 0u : ((1u << left) - 1u);
          words[w] = bits;
        }
      }
      uint32_t sr[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t (&chunk)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[32 * c]);
        tmem_ld32(tS + 32 * c, chunk);
      }
      tmem_wait_ld();
      if (tr) stamp(j, ts + 1);
      // a tile whose keys are all valid (a dense mask) skips the per-element selects
      if (check_keys && (words[0] & words[1] & words[2] & words[3]) != 0xffffffffu) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (!((words[c >> 5] >> (c & 31)) & 1u)) sr[c] = __float_as_uint(-INFINITY);
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) mx = fmaxf(mx, __uint_as_float(sr[c]));
      const float m_new = fmaxf(m, mx * sl);
      if (tr) stamp(j, ts + 2);
      if (j == 0) {
        m = m_new;
      } else {
        const bool need = m_new > m + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          if (!mbar_wait(&o_done[g], (j - 1) & 1, abort_flag, p.err, kErrTimeoutSoftmax)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float f = need ? fast_exp2(m - m_new) : 1.f;
          if (need) {
            l *= f;
            m = m_new;
          }
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + 32 * c, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
            tmem_st32(tO + 32 * c, o);
          }
          tmem_wait_st();
        }
      }
      if (tr) stamp(j, ts + 3);
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float p0 = fast_exp2(fmaf(__uint_as_float(sr[2 * c]), sl, -m));
        const float p1 = fast_exp2(fmaf(__uint_as_float(sr[2 * c + 1]), sl, -m));
        sum += p0 + p1;
        sr[c] = pack_bf16(p0, p1);
      }
      l += sum;
      if (tr) stamp(j, ts + 4);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t (&chunk)[16] = *reinterpret_cast<const uint32_t(*)[16]>(&sr[16 * c]);
        tmem_st16(tS + 16 * c, chunk);
      }
      tmem_wait_st();
      tc_fence_before();
      if (tr) stamp(j, ts + 5);
      mbar_arrive(&p_full[g]);
    }
    if (ok && mbar_wait(&o_done[g], (nkv - 1) & 1, abort_flag, p.err, kErrTimeoutSoftmax)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = p.out + static_cast<long>(b) * p.o_sb + static_cast<long>(q) * p.o_sl +
                           static_cast<long>(h) * p.o_sh;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + 32 * c, o);
        tmem_wait_ld();
        if (q < p.Lq) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
            w.y = pack_bf16(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
            w.z = pack_bf16(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
            w.w = pack_bf16(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
            d4[v] = w;
          }
        }
      }
      if (q < p.Lq && p.lse != nullptr)
        p.lse[(static_cast<long>(b) * p.H + h) * p.stat_ld + q] = l > 0.f ? m + __log2f(l) : INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// =========================================================================== backward
// delta[b, h, q] = sum_d dO[b, q, h, d] * O[b, q, h, d]; one warp per (b, q, h) row.
__global__ void attn_bwd_delta_kernel(const __nv_bfloat16* o, const __nv_bfloat16* dout, float* delta,
                                      int B, int H, int L, long sb, long sl, long sh, long ld) {
  const long rows = static_cast<long>(B) * H * L;
  const int lane = threadIdx.x & 31;
  for (long r = static_cast<long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += static_cast<long>(gridDim.x) * (blockDim.x >> 5)) {
    const long q = r % L;
    const long bh = r / L;
    const long h = bh % H;
    const long b = bh / H;
    const long off = b * sb + q * sl + h * sh + lane * 4;
    const uint2 a = *reinterpret_cast<const uint2*>(o + off);
    const uint2 c = *reinterpret_cast<const uint2*>(dout + off);
    float s = bf16_lo(a.x) * bf16_lo(c.x) + bf16_hi(a.x) * bf16_hi(c.x) + bf16_lo(a.y) * bf16_lo(c.y) +
              bf16_hi(a.y) * bf16_hi(c.y);
#pragma unroll
    for (int k = 16; k > 0; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
    if (lane == 0) delta[bh * ld + q] = s;
  }
}

// Descriptors for tiles whose 64-element column chunks are `chunk` bytes apart
// (rows x 128 B): K-major k-step kk (16 elements), MN-major k-step kk (16 rows).
__device__ __forceinline__ uint64_t kdesc(uint32_t tile, int kk, uint32_t chunk) {
  return umma_desc_sw128(tile + (kk >> 2) * chunk + (kk & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t mndesc(uint32_t tile, int kk, uint32_t chunk) {
  return umma_desc_sw128(tile + kk * 2048, chunk, 1024);
}

__device__ __forceinline__ void store_row_bf16(__nv_bfloat16* dst, const uint32_t (&v)[32], float scale) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 w;
    w.x = pack_bf16(__uint_as_float(v[8 * j + 0]) * scale, __uint_as_float(v[8 * j + 1]) * scale);
    w.y = pack_bf16(__uint_as_float(v[8 * j + 2]) * scale, __uint_as_float(v[8 * j + 3]) * scale);
    w.z = pack_bf16(__uint_as_float(v[8 * j + 4]) * scale, __uint_as_float(v[8 * j + 5]) * scale);
    w.w = pack_bf16(__uint_as_float(v[8 * j + 6]) * scale, __uint_as_float(v[8 * j + 7]) * scale);
    d4[j] = w;
  }
}

// ------------------------------------------------------------------ dK / dV
// CTA = (batch, kv head, 128 keys); loops over 64-query tiles of every query head
// of the group. S^T = K Q^T and dP^T = V dO^T land in TMEM (double-buffered);
// eight softmax warps (two per TMEM lane quadrant, one per 32-query half) turn
// them into P^T and dS^T in place, which the tensor core then consumes directly
// from TMEM: dV += P^T dO, dK += dS^T Q.
//
// Elementwise work per score is one FFMA, one EX2, one FADD and one FMUL. No
// bounds tests are needed: rows of Q / dO / lse / delta past Lq arrive as TMA
// zero fill, and dP^T = 0, delta = 0 there, so they add nothing to dK or dV.
// Queries whose every key is masked carry lse = +inf (P = 0). Keys that are
// masked or past Lk only touch their own dK / dV rows, which are stored as 0.
//
// TMEM columns: S^T[b] at 64*b, dP^T[b] at 128 + 64*b, dV at 256, dK at 384.
// Half h of a buffer writes its bf16 pairs to columns [32h, 32h + 16), inside
// the 32 columns only it reads, so the two halves never race.
struct DkvSmem {
  static constexpr int K = 0;           // 32 KB (2 chunks x 16 KB)
  static constexpr int V = 32768;       // 32 KB
  static constexpr int STAGES = 4;
  static constexpr int STAGE = 65536;   // per stage: Q 16 KB, dO 16 KB, lse 256 B, delta 256 B
  static constexpr int STAGE_BYTES = 33280;
  static constexpr int BARS = STAGE + STAGES * STAGE_BYTES;
  static constexpr int BYTES = BARS + 256;
};
constexpr int kQT = 64;  // query tile of the dK/dV kernel

// TMEM column of k-step kk (16 queries) of a P^T / dS^T buffer written as above.
__device__ __forceinline__ uint32_t half_packed_col(int kk) { return static_cast<uint32_t>(kk * 8 + (kk >= 2 ? 16 : 0)); }

__global__ void __launch_bounds__(384, 1)
    attn_bwd_dkv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                        const __grid_constant__ CUtensorMap tmLse, const __grid_constant__ CUtensorMap tmDelta,
                        const AttnBwdDesc p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DkvSmem::BARS);
  uint64_t* kv_full = bars;                          // 1
  uint64_t* st_full = bars + 1;                      // STAGES
  uint64_t* st_empty = st_full + DkvSmem::STAGES;    // STAGES
  uint64_t* sdp_full = st_empty + DkvSmem::STAGES;   // 2
  uint64_t* p_full = sdp_full + 2;                   // 2 (256 arrivals)
  uint64_t* acc_done = p_full + 2;                   // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int kt = blockIdx.x % p.k_tiles;
  const int bhk = blockIdx.x / p.k_tiles;
  const int hk = bhk % p.Hk;
  const int b = bhk / p.Hk;
  const int k0 = kt * kTile;
  // ring layout [world][B * Hk][ring_len][D]: this tile's chunk, row within it and slab
  const int ring_tiles = p.ring_world > 1 ? p.ring_len / kTile : p.k_tiles;
  const int chunk = kt / ring_tiles;
  const int kv_row = (kt - chunk * ring_tiles) * kTile;
  const int kv_slab = chunk * p.B * p.Hk + b * p.Hk + hk;
  const long kv_len = p.ring_world > 1 ? p.ring_len : p.Lk;
  const int group = p.H / p.Hk;
  const int nq = (p.Lq + kQT - 1) / kQT;
  const int iters = nq * group;

  if (threadIdx.x == 0) {
    const bool misaligned = (smem_u32(smem) & 1023u) != 0;
    if (misaligned) record_error(p.err, kErrBadArgument);
    mbar_init(kv_full, 1);
    for (int s = 0; s < DkvSmem::STAGES; ++s) {
      mbar_init(&st_full[s], 1);
      mbar_init(&st_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sdp_full[i], 1);
      mbar_init(&p_full[i], 256);
    }
    mbar_init(acc_done, 1);
    *abort_flag = misaligned ? 1 : 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tDV = tmem + 256, tDK = tmem + 384;

  if (warp == 0) {
    if (lane == 0 && !*abort_flag) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmdO);
      mbar_arrive_expect_tx(kv_full, 65536);
      for (int c = 0; c < 2; ++c) {
        tma_load_3d(smem + DkvSmem::K + c * 16384, &tmK, kv_full, c * 64, k0, b * p.Hk + hk);
        tma_load_3d(smem + DkvSmem::V + c * 16384, &tmV, kv_full, c * 64, k0, b * p.Hk + hk);
      }
      for (int i = 0; i < iters; ++i) {
        const int s = i % DkvSmem::STAGES;
        const int h = hk * group + i / nq;
        const int qb = (i % nq) * kQT;
        if (!mbar_wait(&st_empty[s], ((i / DkvSmem::STAGES) & 1) ^ 1, abort_flag, p.err, kErrTimeoutProducer)) break;
        uint8_t* st = smem + DkvSmem::STAGE + s * DkvSmem::STAGE_BYTES;
        mbar_arrive_expect_tx(&st_full[s], DkvSmem::STAGE_BYTES);
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(st + c * 8192, &tmQ, &st_full[s], c * 64, qb, b * p.H + h);
          tma_load_4d(st + 16384 + c * 8192, &tmdO, &st_full[s], c * 64, h, qb, b);
        }
        tma_load_2d(st + 32768, &tmLse, &st_full[s], qb, b * p.H + h);
        tma_load_2d(st + 32768 + 256, &tmDelta, &st_full[s], qb, b * p.H + h);
      }
    }
  } else if (warp == 1) {
    const uint32_t idS = idesc_bf16_f32(128, kQT, false, false);
    const uint32_t idA = idesc_bf16_f32(128, 128, false, true);
    // Descriptors of k-step 0; k-step kk adds (byte offset >> 4) to the start-address field.
    const uint64_t dK0 = kdesc(smem_u32(smem + DkvSmem::K), 0, 16384);
    const uint64_t dV0 = kdesc(smem_u32(smem + DkvSmem::V), 0, 16384);
    auto stage_base = [&](int i) {
      return smem_u32(smem + DkvSmem::STAGE + (i % DkvSmem::STAGES) * DkvSmem::STAGE_BYTES);
    };
    auto kstep = [](int kk, uint32_t chunk) -> uint64_t { return ((kk >> 2) * chunk + (kk & 3) * 32) >> 4; };
    auto issue_sdp = [&](int i) {
      const uint32_t sQ = stage_base(i);
      const uint64_t q0 = kdesc(sQ, 0, 8192), o0 = kdesc(sQ + 16384, 0, 8192);
      const uint32_t bufS = tmem + 64 * (i & 1), bufP = tmem + 128 + 64 * (i & 1);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) mma_bf16_ss(bufS, dK0 + kstep(kk, 16384), q0 + kstep(kk, 8192), idS, kk > 0);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) mma_bf16_ss(bufP, dV0 + kstep(kk, 16384), o0 + kstep(kk, 8192), idS, kk > 0);
      mma_commit(&sdp_full[i & 1]);
    };
    bool ok = mbar_wait(kv_full, 0, abort_flag, p.err, kErrTimeoutMma);
    for (int i = 0; i < 2 && i < iters && ok; ++i) {
      ok = mbar_wait(&st_full[i % DkvSmem::STAGES], (i / DkvSmem::STAGES) & 1, abort_flag, p.err, kErrTimeoutMma);
      if (!ok) break;
      tc_fence_after();
      if (elect_one()) issue_sdp(i);
      __syncwarp();
    }
    for (int i = 0; i < iters && ok; ++i) {
      const int buf = i & 1;
      if (!mbar_wait(&p_full[buf], (i >> 1) & 1, abort_flag, p.err, kErrTimeoutMma)) break;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t sQ = stage_base(i);
        const uint64_t q0 = mndesc(sQ, 0, 8192), o0 = mndesc(sQ + 16384, 0, 8192);
        const uint32_t bufS = tmem + 64 * buf, bufP = tmem + 128 + 64 * buf;
#pragma unroll
        for (int kk = 0; kk < kQT / 16; ++kk)
          mma_bf16_ts(tDV, bufS + half_packed_col(kk), o0 + static_cast<uint64_t>(kk * 128), idA,
                      (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kQT / 16; ++kk)
          mma_bf16_ts(tDK, bufP + half_packed_col(kk), q0 + static_cast<uint64_t>(kk * 128), idA,
                      (i > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&st_empty[i % DkvSmem::STAGES]);
        if (i == iters - 1) mma_commit(acc_done);
      }
      __syncwarp();
      if (i + 2 < iters) {
        if (!mbar_wait(&st_full[(i + 2) % DkvSmem::STAGES], ((i + 2) / DkvSmem::STAGES) & 1, abort_flag, p.err,
                       kErrTimeoutMma))
          break;
        tc_fence_after();
        if (elect_one()) issue_sdp(i + 2);
        __syncwarp();
      }
    }
  } else if (warp >= 4) {
    const int quad = warp & 3;
    const int half = (warp - 4) >> 2;  // which 32 queries of the 64-query tile
    const int row = quad * 32 + lane;  // key row
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const float sl = p.scale_log2;
    const int key = k0 + row;
    bool key_ok = key < p.Lk;
    if (key_ok && p.kmask != nullptr)
      key_ok = (p.kmask[static_cast<long>(b) * p.kmask_words + (key >> 5)] >> (key & 31)) & 1u;
    bool ok = true;
    for (int i = 0; i < iters; ++i) {
      const int buf = i & 1;
      const float* stats = reinterpret_cast<const float*>(smem + DkvSmem::STAGE +
                                                          (i % DkvSmem::STAGES) * DkvSmem::STAGE_BYTES + 32768);
      // lse / delta of this stage were written by TMA: observe its barrier too
      if (!mbar_wait(&st_full[i % DkvSmem::STAGES], (i / DkvSmem::STAGES) & 1, abort_flag, p.err,
                     kErrTimeoutSoftmax) ||
          !mbar_wait(&sdp_full[buf], (i >> 1) & 1, abort_flag, p.err, kErrTimeoutSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tS = tmem + lane_base + 64 * buf + 32 * half;
      const uint32_t tP = tmem + lane_base + 128 + 64 * buf + 32 * half;
      uint32_t sv[32], dv[32];
      tmem_ld32(tS, sv);
      tmem_ld32(tP, dv);
      const float4* l4 = reinterpret_cast<const float4*>(stats + 32 * half);
      const float4* d4 = reinterpret_cast<const float4*>(stats + 64 + 32 * half);
      tmem_wait_ld();
      uint32_t pp[16], dd[16];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float4 l = l4[e], dl = d4[e];
        const float p0 = fast_exp2(fmaf(__uint_as_float(sv[4 * e + 0]), sl, -l.x));
        const float p1 = fast_exp2(fmaf(__uint_as_float(sv[4 * e + 1]), sl, -l.y));
        const float p2 = fast_exp2(fmaf(__uint_as_float(sv[4 * e + 2]), sl, -l.z));
        const float p3 = fast_exp2(fmaf(__uint_as_float(sv[4 * e + 3]), sl, -l.w));
        pp[2 * e] = pack_bf16(p0, p1);
        pp[2 * e + 1] = pack_bf16(p2, p3);
        dd[2 * e] = pack_bf16(p0 * (__uint_as_float(dv[4 * e + 0]) - dl.x), p1 * (__uint_as_float(dv[4 * e + 1]) - dl.y));
        dd[2 * e + 1] =
            pack_bf16(p2 * (__uint_as_float(dv[4 * e + 2]) - dl.z), p3 * (__uint_as_float(dv[4 * e + 3]) - dl.w));
      }
      tmem_st16(tS, pp);
      tmem_st16(tP, dd);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[buf]);
    }
    if (ok && mbar_wait(acc_done, 0, abort_flag, p.err, kErrTimeoutSoftmax)) {
      tc_fence_after();
      const long off = (static_cast<long>(kv_slab) * kv_len + kv_row + row) * kHD;
      // each half stores 64 of the 128 columns of its key row
#pragma unroll 1
      for (int c = 2 * half; c < 2 * half + 2; ++c) {
        uint32_t a[32], v[32];
        tmem_ld32(tDK + lane_base + 32 * c, a);
        tmem_ld32(tDV + lane_base + 32 * c, v);
        tmem_wait_ld();
        if (key < p.Lk) {
          if (!key_ok) {  // a masked key's rows hold unnormalised garbage: write zeros, not 0 * garbage
#pragma unroll
            for (int e = 0; e < 32; ++e) a[e] = v[e] = 0u;
          }
          store_row_bf16(p.dk + off + 32 * c, a, p.scale);
          store_row_bf16(p.dv + off + 32 * c, v, 1.f);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ dQ
// CTA = (batch, head, 256 queries as two 128-row tiles); loops over 64-key blocks.
// TMEM per tile g: S (64 cols) at 128g, dP (64) at 128g + 64, dQ (128) at 256 + 128g.
// Masked keys (HAS_MASK) and keys past Lk in the last block get P = 0: a key row
// of TMA zero fill scores 0, and exp2(0 - lse) can overflow when every valid
// score of the row is very negative.
struct DqSmem {
  static constexpr int Q = 0;          // 2 x 32 KB
  static constexpr int DO = 65536;     // 2 x 32 KB
  static constexpr int STAGES = 3;
  static constexpr int KV = 131072;    // per stage: K 16 KB, V 16 KB
  static constexpr int STAGE_BYTES = 32768;
  static constexpr int BARS = KV + STAGES * STAGE_BYTES;
  static constexpr int BYTES = BARS + 256;
};
constexpr int kKT = 64;  // key block of the dQ kernel

template <bool HAS_MASK>
__global__ void __launch_bounds__(384, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                       const AttnBwdDesc p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DqSmem::BARS);
  uint64_t* q_full = bars;                          // 1
  uint64_t* kv_full = bars + 1;                     // STAGES
  uint64_t* kv_empty = kv_full + DqSmem::STAGES;    // STAGES
  uint64_t* sdp_full = kv_empty + DqSmem::STAGES;   // 2
  uint64_t* ds_full = sdp_full + 2;                 // 2 (128 arrivals)
  uint64_t* dq_done = ds_full + 2;                  // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dq_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int qt = blockIdx.x % p.q_tiles;
  const int bh = blockIdx.x / p.q_tiles;
  const int h = bh % p.H;
  const int b = bh / p.H;
  const int hk = h / (p.H / p.Hk);
  const int q0 = qt * 256;
  const int nkv = (p.Lk + kKT - 1) / kKT;

  if (threadIdx.x == 0) {
    const bool misaligned = (smem_u32(smem) & 1023u) != 0;
    if (misaligned) record_error(p.err, kErrBadArgument);
    mbar_init(q_full, 1);
    for (int s = 0; s < DqSmem::STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&sdp_full[g], 1);
      mbar_init(&ds_full[g], 128);
    }
    mbar_init(dq_done, 1);
    *abort_flag = misaligned ? 1 : 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && !*abort_flag) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, 131072);
      for (int g = 0; g < 2; ++g)
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(smem + DqSmem::Q + g * 32768 + c * 16384, &tmQ, q_full, c * 64, q0 + 128 * g, b * p.H + h);
          tma_load_4d(smem + DqSmem::DO + g * 32768 + c * 16384, &tmdO, q_full, c * 64, h, q0 + 128 * g, b);
        }
      for (int j = 0; j < nkv; ++j) {
        const int s = j % DqSmem::STAGES;
        if (!mbar_wait(&kv_empty[s], ((j / DqSmem::STAGES) & 1) ^ 1, abort_flag, p.err, kErrTimeoutProducer)) break;
        uint8_t* st = smem + DqSmem::KV + s * DqSmem::STAGE_BYTES;
        mbar_arrive_expect_tx(&kv_full[s], DqSmem::STAGE_BYTES);
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(st + c * 8192, &tmK, &kv_full[s], c * 64, j * kKT, b * p.Hk + hk);
          tma_load_3d(st + 16384 + c * 8192, &tmV, &kv_full[s], c * 64, j * kKT, b * p.Hk + hk);
        }
      }
    }
  } else if (warp == 1) {
    const uint32_t idS = idesc_bf16_f32(128, kKT, false, false);
    const uint32_t idQ = idesc_bf16_f32(128, 128, false, true);
    const uint64_t dQ0[2] = {kdesc(smem_u32(smem + DqSmem::Q), 0, 16384),
                             kdesc(smem_u32(smem + DqSmem::Q + 32768), 0, 16384)};
    const uint64_t dO0[2] = {kdesc(smem_u32(smem + DqSmem::DO), 0, 16384),
                             kdesc(smem_u32(smem + DqSmem::DO + 32768), 0, 16384)};
    auto kv_addr = [&](int j) { return smem_u32(smem + DqSmem::KV + (j % DqSmem::STAGES) * DqSmem::STAGE_BYTES); };
    auto kstep = [](int kk, uint32_t chunk) -> uint64_t { return ((kk >> 2) * chunk + (kk & 3) * 32) >> 4; };
    auto issue_sdp = [&](int g, int j) {
      const uint32_t sK = kv_addr(j);
      const uint64_t k0d = kdesc(sK, 0, 8192), v0d = kdesc(sK + 16384, 0, 8192);
      const uint32_t tS = tmem + 128 * g, tP = tS + 64;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) mma_bf16_ss(tS, dQ0[g] + kstep(kk, 16384), k0d + kstep(kk, 8192), idS, kk > 0);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) mma_bf16_ss(tP, dO0[g] + kstep(kk, 16384), v0d + kstep(kk, 8192), idS, kk > 0);
      mma_commit(&sdp_full[g]);
    };
    auto issue_dq = [&](int g, int j) {
      const uint64_t km = mndesc(kv_addr(j), 0, 8192);
#pragma unroll
      for (int kk = 0; kk < kKT / 16; ++kk)
        mma_bf16_ts(tmem + 256 + 128 * g, tmem + 128 * g + kk * 8, km + static_cast<uint64_t>(kk * 128), idQ,
                    (j > 0 || kk > 0) ? 1u : 0u);
    };
    bool ok = mbar_wait(q_full, 0, abort_flag, p.err, kErrTimeoutMma) &&
              mbar_wait(&kv_full[0], 0, abort_flag, p.err, kErrTimeoutMma);
    if (ok) {
      tc_fence_after();
      if (elect_one()) {
        issue_sdp(0, 0);
        issue_sdp(1, 0);
      }
      __syncwarp();
    }
    for (int j = 0; j < nkv && ok; ++j) {
      const bool more = j + 1 < nkv;
      if (!mbar_wait(&ds_full[0], j & 1, abort_flag, p.err, kErrTimeoutMma)) break;
      tc_fence_after();
      if (elect_one()) issue_dq(0, j);
      __syncwarp();
      if (more) {
        if (!mbar_wait(&kv_full[(j + 1) % DqSmem::STAGES], ((j + 1) / DqSmem::STAGES) & 1, abort_flag, p.err,
                       kErrTimeoutMma))
          break;
        tc_fence_after();
        if (elect_one()) issue_sdp(0, j + 1);
        __syncwarp();
      }
      if (!mbar_wait(&ds_full[1], j & 1, abort_flag, p.err, kErrTimeoutMma)) break;
      tc_fence_after();
      if (elect_one()) {
        issue_dq(1, j);
        mma_commit(&kv_empty[j % DqSmem::STAGES]);
        if (more) issue_sdp(1, j + 1);
        if (!more) mma_commit(dq_done);
      }
      __syncwarp();
    }
  } else if (warp >= 4) {
    const int g = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int q = q0 + 128 * g + row;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_base + 128 * g, tP = tS + 64;
    const float sl = p.scale_log2;
    const bool q_ok = q < p.Lq;
    // rows past Lq or with no valid key: lse = +inf makes every P zero
    const float lse_q = q_ok ? p.lse[(static_cast<long>(b) * p.H + h) * p.stat_ld + q] : INFINITY;
    const float dlt_q = q_ok ? p.delta[(static_cast<long>(b) * p.H + h) * p.stat_ld + q] : 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      if (!mbar_wait(&sdp_full[g], j & 1, abort_flag, p.err, kErrTimeoutSoftmax)) { ok = false; break; }
      tc_fence_after();
      uint32_t words[2] = {0xffffffffu, 0xffffffffu};
      const int key0 = j * kKT;
      const bool tail = key0 + kKT > p.Lk;
      if (HAS_MASK || tail) {
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          const int k32 = key0 + 32 * w;
          uint32_t bits = 0xffffffffu;
          if (HAS_MASK && k32 < p.Lk) bits = p.kmask[static_cast<long>(b) * p.kmask_words + (k32 >> 5)];
          const int left = p.Lk - k32;
          if (left < 32) bits &= (left <= 0) ? 0u : ((1u << left) - 1u);
          words[w] = bits;
        }
      }
      const bool masked = HAS_MASK || tail;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t sv[32], dv[32];
        tmem_ld32(tS + 32 * c, sv);
        tmem_ld32(tP + 32 * c, dv);
        tmem_wait_ld();
        uint32_t dd[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float p0 = fast_exp2(fmaf(__uint_as_float(sv[2 * e]), sl, -lse_q));
          float p1 = fast_exp2(fmaf(__uint_as_float(sv[2 * e + 1]), sl, -lse_q));
          if (masked) {
            p0 = ((words[c] >> (2 * e)) & 1u) ? p0 : 0.f;
            p1 = ((words[c] >> (2 * e + 1)) & 1u) ? p1 : 0.f;
          }
          dd[e] = pack_bf16(p0 * (__uint_as_float(dv[2 * e]) - dlt_q), p1 * (__uint_as_float(dv[2 * e + 1]) - dlt_q));
        }
        tmem_st16(tS + 16 * c, dd);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&ds_full[g]);
    }
    if (ok && mbar_wait(dq_done, 0, abort_flag, p.err, kErrTimeoutSoftmax)) {
      tc_fence_after();
      __nv_bfloat16* dst = p.dq + ((static_cast<long>(b) * p.H + h) * p.Lq + q) * kHD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + 256 + 128 * g + 32 * c, v);
        tmem_wait_ld();
        if (q_ok) store_row_bf16(dst + 32 * c, v, p.scale);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ fused backward
// One pass over (query tile, key tile) pairs with five GEMM-shaped products per
// pair (the minimum): S^T = K Q^T, dP^T = V dO^T, dV += P^T dO, dK += dS^T Q and
// dQ^T = K^T dS^T. CTA = (batch, kv head, 128 keys); it walks the 64-query tiles
// of every query head of its group.
//
//  * S^T, dP^T: TMEM, double-buffered. Eight softmax warps (two per TMEM lane
//    quadrant, one per 32-query half) form P^T and dS^T in place in TMEM (bf16
//    pairs) and also write dS^T to shared memory as a 128 x 64 SW128 tile.
//  * dV and dK read P^T / dS^T from TMEM (the TS form: no shared-memory traffic
//    for A); the shared dS^T tile is the MN-major B operand of dQ^T, whose A
//    operand is the K tile read MN-major.
//  * dQ^T of a pair (128 d x 64 q, fp32) lands in the S^T buffer after dV has
//    read P^T from it, so the next pair's dP^T can start while dQ^T drains. Four epilogue warps drain it through shared memory and add it into
//    a global fp32 dQ^T accumulator [B*H, 128, ld] with TMA bulk reduce-add, two
//    32 x 32 swizzled boxes per warp (measured faster than per-thread
//    red.global.add, whose load/store-pipe traffic slows the MMA operand reads).
//    A final kernel scales and transposes it to bf16 dQ.
//
// No bounds tests sit in the elementwise loop: query rows past Lq arrive as TMA
// zero fill (they add nothing and are dropped by the reduce), rows whose every
// key is masked carry lse = +inf (P = 0), and masked keys or keys past Lk get
// P = dS = 0 through a per-thread select (their dS^T would otherwise reach dQ).
//
// TMEM columns: dV [0,128), dK [128,256), S^T / dQ^T[b] at 256 + 64b, dP^T[b] at 384 + 64b.
struct FusedBwdSmem {
  static constexpr int K = 0;            // 2 chunks x 16 KB (128 keys x 64 d, SW128)
  static constexpr int V = 32768;
  static constexpr int STAGES = 3;
  static constexpr int STAGE = 65536;    // per stage: Q 16 KB, dO 16 KB
  static constexpr int STAGE_BYTES = 32768;
  static constexpr int DST = STAGE + STAGES * STAGE_BYTES;   // 2 x 16 KB dS^T (128 keys x 64 q)
  static constexpr int STG = DST + 2 * 16384;                 // 4 x 8 KB fp32 dQ^T slabs
  static constexpr int STATS = STG + 4 * 8192;                // STAGES x (lse 256 B, delta 256 B)
  static constexpr int BARS = STATS + STAGES * 512;
  static constexpr int BYTES = BARS + 256;
};
static_assert(FusedBwdSmem::BYTES <= 232448, "fused attention backward exceeds shared memory");

template <bool kTrace>
__global__ void __launch_bounds__(512, 1)
    attn_bwd_fused_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                          const __grid_constant__ CUtensorMap tmLse, const __grid_constant__ CUtensorMap tmDelta,
                          const __grid_constant__ CUtensorMap tmAcc, const AttnBwdDesc p) {
  using S = FusedBwdSmem;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BARS);
  uint64_t* kv_full = bars;                      // 1
  uint64_t* st_full = bars + 1;                  // STAGES
  uint64_t* st_empty = st_full + S::STAGES;      // STAGES
  uint64_t* sdp_full = st_empty + S::STAGES;     // 2
  uint64_t* p_full = sdp_full + 2;               // 2 (256 arrivals)
  uint64_t* dq_full = p_full + 2;                // 2
  uint64_t* dq_empty = dq_full + 2;              // 2 (128 arrivals)
  uint64_t* acc_done = dq_empty + 2;             // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* trace_bar = bars + 20;               // 5, diagnostics only: per-GEMM completion

  const int warp = warp_id();
  const int lane = lane_id();
  const int kt_span = p.kt_count > 0 ? p.kt_count : p.k_tiles;
  const int kt = p.kt_begin + static_cast<int>(blockIdx.x % kt_span);
  const int bhk = blockIdx.x / kt_span;
  const int hk = bhk % p.Hk;
  const int b = bhk / p.Hk;
  const int k0 = kt * kTile;
  // ring layout [world][B * Hk][ring_len][D]: this tile's chunk, row within it and slab
  const int ring_tiles = p.ring_world > 1 ? p.ring_len / kTile : p.k_tiles;
  const int chunk = kt / ring_tiles;
  const int kv_row = (kt - chunk * ring_tiles) * kTile;
  const int kv_slab = chunk * p.B * p.Hk + b * p.Hk + hk;
  const long kv_len = p.ring_world > 1 ? p.ring_len : p.Lk;
  const int group = p.H / p.Hk;
  const int nq = (p.Lq + kQT - 1) / kQT;
  const int iters = nq * group;
  // diagnostics: SM clock stamps of CTA 0, 24 per iteration, first 64 iterations. Slots:
  // 0 MMA thread passes p_full(i), 1 it passes dq_empty, 2 softmax starts, 3 warp 4 arrives,
  // 4 drain sees dq_full, 5/6/7 dV/dK/dQ^T(i) complete, 8-15 softmax warps arrive,
  // 16-19 drain warps release dQ^T, 20/21 dP^T/S^T(i+2) complete.
  long long* trace = (kTrace && blockIdx.x == 0) ? p.trace : nullptr;
  auto stamp = [&](int i, int slot) {
    if (trace != nullptr && i < 64) trace[i * 24 + slot] = clock64();
  };

  if (threadIdx.x == 0) {
    const bool misaligned = (smem_u32(smem) & 1023u) != 0;
    if (misaligned) record_error(p.err, kErrBadArgument);
    mbar_init(kv_full, 1);
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(&st_full[s], 1);
      mbar_init(&st_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sdp_full[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_empty[i], 128);
    }
    mbar_init(acc_done, 1);
    for (int j = 0; j < 5; ++j) mbar_init(&trace_bar[j], 1);
    *abort_flag = misaligned ? 1 : 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tDV = tmem, tDK = tmem + 128;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && !*abort_flag) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmdO);
      mbar_arrive_expect_tx(kv_full, 65536);
      for (int c = 0; c < 2; ++c) {
        tma_load_3d(smem + S::K + c * 16384, &tmK, kv_full, c * 64, kv_row, kv_slab);
        tma_load_3d(smem + S::V + c * 16384, &tmV, kv_full, c * 64, kv_row, kv_slab);
      }
      for (int i = 0; i < iters; ++i) {
        const int s = i % S::STAGES;
        const int h = hk * group + i / nq;
        const int qb = (i % nq) * kQT;
        if (!mbar_wait(&st_empty[s], ((i / S::STAGES) & 1) ^ 1, abort_flag, p.err, kErrTimeoutProducer)) break;
        uint8_t* st = smem + S::STAGE + s * S::STAGE_BYTES;
        mbar_arrive_expect_tx(&st_full[s], S::STAGE_BYTES + 512);
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(st + c * 8192, &tmQ, &st_full[s], c * 64, qb, b * p.H + h);
          tma_load_4d(st + 16384 + c * 8192, &tmdO, &st_full[s], c * 64, h, qb, b);
        }
        tma_load_2d(smem + S::STATS + s * 512, &tmLse, &st_full[s], qb, b * p.H + h);
        tma_load_2d(smem + S::STATS + s * 512 + 256, &tmDelta, &st_full[s], qb, b * p.H + h);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idS = idesc_bf16_f32(128, kQT, false, false);  // S^T, dP^T: 128 keys x 64 q
    const uint32_t idA = idesc_bf16_f32(128, 128, false, true);   // dV, dK: 128 keys x 128 d
    const uint32_t idQ = idesc_bf16_f32(128, kQT, true, true);    // dQ^T: 128 d x 64 q
    const uint64_t dK0 = kdesc(smem_u32(smem + S::K), 0, 16384);
    const uint64_t dV0 = kdesc(smem_u32(smem + S::V), 0, 16384);
    const uint64_t dKt = mndesc(smem_u32(smem + S::K), 0, 16384);  // K as the MN-major A of dQ^T
    auto stage_base = [&](int i) { return smem_u32(smem + S::STAGE + (i % S::STAGES) * S::STAGE_BYTES); };
    auto kstep = [](int kk, uint32_t chunk) -> uint64_t { return ((kk >> 2) * chunk + (kk & 3) * 32) >> 4; };
    auto issue_s = [&](int i) {
      const uint64_t q0 = kdesc(stage_base(i), 0, 8192);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_bf16_ss(tmem + 256 + 64 * (i & 1), dK0 + kstep(kk, 16384), q0 + kstep(kk, 8192), idS, kk > 0);
    };
    auto issue_dp = [&](int i) {
      const uint64_t o0 = kdesc(stage_base(i) + 16384, 0, 8192);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_bf16_ss(tmem + 384 + 64 * (i & 1), dV0 + kstep(kk, 16384), o0 + kstep(kk, 8192), idS, kk > 0);
    };
    bool ok = mbar_wait(kv_full, 0, abort_flag, p.err, kErrTimeoutMma);
    for (int i = 0; i < 2 && i < iters && ok; ++i) {
      ok = mbar_wait(&st_full[i % S::STAGES], (i / S::STAGES) & 1, abort_flag, p.err, kErrTimeoutMma);
      if (!ok) break;
      tc_fence_after();
      if (elect_one()) {
        issue_s(i);
        issue_dp(i);
        mma_commit(&sdp_full[i & 1]);
      }
      __syncwarp();
    }
    for (int i = 0; i < iters && ok; ++i) {
      const int buf = i & 1;
      if (!mbar_wait(&p_full[buf], (i >> 1) & 1, abort_flag, p.err, kErrTimeoutMma)) break;
      tc_fence_after();
      if (elect_one()) {
        stamp(i, 0);
        const uint32_t sQ = stage_base(i);
        const uint64_t qmn = mndesc(sQ, 0, 8192), omn = mndesc(sQ + 16384, 0, 8192);
        const uint32_t dst = smem_u32(smem + S::DST + buf * 16384);
        const uint64_t dsM = mndesc(dst, 0, 16384);  // dS^T as MN-major B (k = keys, n = queries)
#pragma unroll
        for (int kk = 0; kk < kQT / 16; ++kk)
          mma_bf16_ts(tDV, tmem + 256 + 64 * buf + half_packed_col(kk), omn + static_cast<uint64_t>(kk * 128), idA,
                      (i > 0 || kk > 0) ? 1u : 0u);
        if (trace != nullptr) mma_commit(&trace_bar[0]);
#pragma unroll
        for (int kk = 0; kk < kQT / 16; ++kk)
          mma_bf16_ts(tDK, tmem + 384 + 64 * buf + half_packed_col(kk), qmn + static_cast<uint64_t>(kk * 128), idA,
                      (i > 0 || kk > 0) ? 1u : 0u);
        if (trace != nullptr) mma_commit(&trace_bar[1]);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)  // into the S^T buffer: dV(i) has read P^T(i) (in order)
          mma_bf16_ss(tmem + 256 + 64 * buf, dKt + static_cast<uint64_t>(kk * 128),
                      dsM + static_cast<uint64_t>(kk * 128), idQ, kk > 0 ? 1u : 0u);
        mma_commit(&dq_full[buf]);
        if (trace != nullptr) mma_commit(&trace_bar[2]);
        mma_commit(&st_empty[i % S::STAGES]);
        if (i == iters - 1) mma_commit(acc_done);
      }
      __syncwarp();
      if (i + 2 < iters) {
        if (!mbar_wait(&st_full[(i + 2) % S::STAGES], ((i + 2) / S::STAGES) & 1, abort_flag, p.err, kErrTimeoutMma))
          break;
        tc_fence_after();
        if (elect_one()) {
          issue_dp(i + 2);  // dP^T buffer: in order after dK(i) read dS^T(i); runs while dQ^T(i) drains
          if (trace != nullptr) mma_commit(&trace_bar[3]);
        }
        __syncwarp();
        // the S^T buffer holds dQ^T(i) until the epilogue has read it
        if (!mbar_wait(&dq_empty[buf], (i >> 1) & 1, abort_flag, p.err, kErrTimeoutMma)) break;
        tc_fence_after();
        if (elect_one()) {
          stamp(i, 1);
          issue_s(i + 2);
          mma_commit(&sdp_full[buf]);
          if (trace != nullptr) mma_commit(&trace_bar[4]);
        }
        __syncwarp();
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ diagnostics: GEMM completion stamps
    if (trace != nullptr && lane == 0) {
      for (int i = 0; i < iters && i < 64; ++i) {
        const uint32_t ph = i & 1;
        if (!mbar_wait(&trace_bar[0], ph, abort_flag, p.err, kErrTimeoutEpilogue)) break;
        stamp(i, 5);
        if (!mbar_wait(&trace_bar[1], ph, abort_flag, p.err, kErrTimeoutEpilogue)) break;
        stamp(i, 6);
        if (!mbar_wait(&trace_bar[2], ph, abort_flag, p.err, kErrTimeoutEpilogue)) break;
        stamp(i, 7);
        if (i + 2 >= iters) continue;
        if (!mbar_wait(&trace_bar[3], ph, abort_flag, p.err, kErrTimeoutEpilogue)) break;
        stamp(i, 20);
        if (!mbar_wait(&trace_bar[4], ph, abort_flag, p.err, kErrTimeoutEpilogue)) break;
        stamp(i, 21);
      }
    }
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------------ softmax: P^T, dS^T
    const int quad = warp & 3;
    const int half = (warp - 4) >> 2;
    const int row = quad * 32 + lane;  // key row
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const float sl = p.scale_log2;
    const int key = k0 + row;
    bool key_ok = key < p.Lk;
    if (key_ok && p.kmask != nullptr)
      key_ok = (p.kmask[static_cast<long>(b) * p.kmask_words + (key >> 5)] >> (key & 31)) & 1u;
    bool ok = true;
    for (int i = 0; i < iters; ++i) {
      const int buf = i & 1;
      const float* stats = reinterpret_cast<const float*>(smem + S::STATS + (i % S::STAGES) * 512);
      if (!mbar_wait(&st_full[i % S::STAGES], (i / S::STAGES) & 1, abort_flag, p.err, kErrTimeoutSoftmax) ||
          !mbar_wait(&sdp_full[buf], (i >> 1) & 1, abort_flag, p.err, kErrTimeoutSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (warp == 4 && lane == 0) stamp(i, 2);
      const uint32_t tS = tmem + lane_base + 256 + 64 * buf + 32 * half;
      const uint32_t tP = tmem + lane_base + 384 + 64 * buf + 32 * half;
      uint32_t sv[32], dv[32];
      tmem_ld32(tS, sv);
      tmem_ld32(tP, dv);
      const float4* l4 = reinterpret_cast<const float4*>(stats + 32 * half);
      const float4* d4 = reinterpret_cast<const float4*>(stats + 64 + 32 * half);
      tmem_wait_ld();
      uint32_t pp[16], dd[16];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float4 l = l4[e], dl = d4[e];
        // select, not multiply: a masked key's score may overflow exp2 and 0 * inf is NaN
        const float p0 = key_ok ? fast_exp2(fmaf(__uint_as_float(sv[4 * e + 0]), sl, -l.x)) : 0.f;
        const float p1 = key_ok ? fast_exp2(fmaf(__uint_as_float(sv[4 * e + 1]), sl, -l.y)) : 0.f;
        const float p2 = key_ok ? fast_exp2(fmaf(__uint_as_float(sv[4 * e + 2]), sl, -l.z)) : 0.f;
        const float p3 = key_ok ? fast_exp2(fmaf(__uint_as_float(sv[4 * e + 3]), sl, -l.w)) : 0.f;
        pp[2 * e] = pack_bf16(p0, p1);
        pp[2 * e + 1] = pack_bf16(p2, p3);
        dd[2 * e] = pack_bf16(p0 * (__uint_as_float(dv[4 * e + 0]) - dl.x), p1 * (__uint_as_float(dv[4 * e + 1]) - dl.y));
        dd[2 * e + 1] =
            pack_bf16(p2 * (__uint_as_float(dv[4 * e + 2]) - dl.z), p3 * (__uint_as_float(dv[4 * e + 3]) - dl.w));
      }
      tmem_st16(tS, pp);
      tmem_st16(tP, dd);
      // dS^T row `row`, queries [32 half, 32 half + 32): 16-byte chunks 4 half .. 4 half + 3 of
      // the 128-byte row, XOR-swizzled by row & 7 (SW128).
      uint8_t* drow = smem + S::DST + buf * 16384 + row * 128;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int chunk = (4 * half + j) ^ (row & 7);
        *reinterpret_cast<uint4*>(drow + chunk * 16) = make_uint4(dd[4 * j], dd[4 * j + 1], dd[4 * j + 2], dd[4 * j + 3]);
      }
      tmem_wait_st();
      fence_proxy_async();
      tc_fence_before();
      if (warp == 4 && lane == 0) stamp(i, 3);
      if (lane == 0) stamp(i, 8 + (warp - 4));
      mbar_arrive(&p_full[buf]);
    }
    if (ok && mbar_wait(acc_done, 0, abort_flag, p.err, kErrTimeoutSoftmax)) {
      tc_fence_after();
      const long off = (static_cast<long>(kv_slab) * kv_len + kv_row + row) * kHD;
#pragma unroll 1
      for (int c = 2 * half; c < 2 * half + 2; ++c) {
        uint32_t a[32], v[32];
        tmem_ld32(tDK + lane_base + 32 * c, a);
        tmem_ld32(tDV + lane_base + 32 * c, v);
        tmem_wait_ld();
        if (key < p.Lk) {
          store_row_bf16(p.dk + off + 32 * c, a, p.scale);
          store_row_bf16(p.dv + off + 32 * c, v, 1.f);
        }
      }
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------ dQ^T drain + TMA reduce-add
    const int quad = warp & 3;  // d rows [32 quad, 32 quad + 32)
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    // two SW128 sub-tiles of 32 d x 32 q (4 KB each) per warp: queries [0,32) and [32,64)
    uint8_t* slab = smem + S::STG + quad * 8192;
    for (int i = 0; i < iters; ++i) {
      const int buf = i & 1;
      const int h = hk * group + i / nq;
      const int qb = (i % nq) * kQT;
      if (!mbar_wait(&dq_full[buf], (i >> 1) & 1, abort_flag, p.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      if (warp == 12 && lane == 0) stamp(i, 4);
      uint32_t v0[32], v1[32];
      tmem_ld32(tmem + lane_base + 256 + 64 * buf, v0);
      tmem_ld32(tmem + lane_base + 256 + 64 * buf + 32, v1);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&dq_empty[buf]);
      if (lane == 0) stamp(i, 16 + (warp - 12));
      if (lane == 0 && i > 0) bulk_wait_group_read0();  // the previous reduce has read the slab
      __syncwarp();
      // row `lane` of each sub-tile: 16-byte chunk j at j ^ (lane & 7) (SW128), so the
      // eight lanes of a store phase hit eight different bank groups
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = (j ^ (lane & 7)) * 16 + lane * 128;
        *reinterpret_cast<uint4*>(slab + c) = make_uint4(v0[4 * j], v0[4 * j + 1], v0[4 * j + 2], v0[4 * j + 3]);
        *reinterpret_cast<uint4*>(slab + 4096 + c) =
            make_uint4(v1[4 * j], v1[4 * j + 1], v1[4 * j + 2], v1[4 * j + 3]);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_3d(&tmAcc, slab, qb, 32 * quad, b * p.H + h);
        tma_reduce_add_3d(&tmAcc, slab + 4096, qb + 32, 32 * quad, b * p.H + h);
        bulk_commit_group();
      }
    }
    if (lane == 0) bulk_wait_group0();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dq[b, h, q, :] = scale * acc[b*H + h, :, q] (fp32 [B*H, 128, ld] -> bf16 [B, H, Lq, 128]).
// CTA = 64 queries of one (b, h): coalesced row reads, a shared-memory transpose, 256-byte row writes.
__global__ void __launch_bounds__(256) attn_dq_convert_kernel(const float* __restrict__ acc, long ld, int Lq,
                                                              float scale, __nv_bfloat16* __restrict__ dq) {
  __shared__ float tile[128][65];
  const long bh = blockIdx.y;
  const int q0 = blockIdx.x * 64;
  const float* src = acc + bh * 128 * ld;
  for (int idx = threadIdx.x; idx < 128 * 64; idx += 256) {
    const int d = idx >> 6, q = idx & 63;
    tile[d][q] = (q0 + q < Lq) ? src[d * ld + q0 + q] : 0.f;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 64 * 16; idx += 256) {
    const int q = idx >> 4, d0 = (idx & 15) * 8;
    if (q0 + q >= Lq) continue;
    uint4 w;
    w.x = pack_bf16(tile[d0 + 0][q] * scale, tile[d0 + 1][q] * scale);
    w.y = pack_bf16(tile[d0 + 2][q] * scale, tile[d0 + 3][q] * scale);
    w.z = pack_bf16(tile[d0 + 4][q] * scale, tile[d0 + 5][q] * scale);
    w.w = pack_bf16(tile[d0 + 6][q] * scale, tile[d0 + 7][q] * scale);
    *reinterpret_cast<uint4*>(dq + (bh * Lq + q0 + q) * kHD + d0) = w;
  }
}

}  // namespace

void attn_fwd_launch(const AttnFwdDesc& d_in, cudaStream_t stream) {
  AttnFwdDesc d = d_in;
  AVGEN_CHECK(d.D == kHD, "attention: head_dim must be 128, got ", d.D);
  AVGEN_CHECK(d.H % d.Hk == 0, "attention: H must be a multiple of Hk");
  if (d.B == 0 || d.Lq == 0) return;
  d.q_tiles = (d.Lq + 255) / 256;
  // Q, K, V head-major [B*H, L, D] with rows of D elements.
  const CUtensorMap tq = make_tmap_3d_bf16(d.q, kHD, d.Lq, static_cast<long>(d.B) * d.H, kHD,
                                           static_cast<long>(d.Lq) * kHD, 64, 128, 1);
  const bool ring = d.ring_world > 1;
  if (ring) {
    AVGEN_CHECK(d.ring_len % kTile == 0 && d.ring_len > 0 && d.Lk == d.ring_world * d.ring_len,
                "attention ring: keys per rank must be a positive multiple of 128 and Lk = world * that");
    AVGEN_CHECK(d.ring_rank >= 0 && d.ring_rank < d.ring_world && d.ring_flags != nullptr,
                "attention ring: bad rank or missing flags");
  }
  // ring: [world * B * Hk, ring_len, D]; else [B * Hk, Lk, D]
  const long kv_len = ring ? d.ring_len : d.Lk;
  const long kv_slabs = static_cast<long>(d.B) * d.Hk * (ring ? d.ring_world : 1);
  const CUtensorMap tk = make_tmap_3d_bf16(d.k, kHD, kv_len, kv_slabs, kHD, kv_len * kHD, 64, 128, 1);
  const CUtensorMap tv = make_tmap_3d_bf16(d.v, kHD, kv_len, kv_slabs, kHD, kv_len * kHD, 64, 128, 1);
  static PerDeviceOnce once_plain, once_trace;
  raise_smem_limit(once_plain, attn_fwd_kernel<false>, FwdSmem::BYTES);
  raise_smem_limit(once_trace, attn_fwd_kernel<true>, FwdSmem::BYTES);
  const long grid = static_cast<long>(d.B) * d.H * d.q_tiles;
  if (d.trace != nullptr)
    attn_fwd_kernel<true><<<grid, 384, FwdSmem::BYTES, stream>>>(tq, tk, tv, d);
  else
    attn_fwd_kernel<false><<<grid, 384, FwdSmem::BYTES, stream>>>(tq, tk, tv, d);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

void attn_bwd_launch(const AttnBwdDesc& d_in, cudaStream_t stream) {
  AttnBwdDesc d = d_in;
  AVGEN_CHECK(d.D == kHD, "attention bwd: head_dim must be 128");
  AVGEN_CHECK(d.H % d.Hk == 0, "attention bwd: H must be a multiple of Hk");
  if (d.B == 0 || d.Lk == 0 || d.Lq == 0) return;
  AVGEN_CHECK(d.o_sh == kHD && d.o_sl == static_cast<long>(d.H) * kHD &&
                  d.o_sb == static_cast<long>(d.Lq) * d.H * kHD,
              "attention bwd: O / dO must be dense [B, Lq, H, 128]");
  AVGEN_CHECK(d.stat_ld >= d.Lq && d.stat_ld % 4 == 0, "attention bwd: lse/delta row stride must be >= Lq and a multiple of 4");
  AVGEN_CHECK(d.ring_world <= 1 || d.dq_acc != nullptr, "attention bwd: the ring layout needs the fused kernel");
  AVGEN_CHECK(d.kt_count == 0 || d.dq_acc != nullptr, "attention bwd: key-tile ranges need the fused kernel");
  // delta = rowsum(dO * O)
  if (!d.skip_prologue) {
    const long rows = static_cast<long>(d.B) * d.H * d.Lq;
    const long blocks = std::min<long>((rows + 7) / 8, 16L * num_sms(d.device));
    attn_bwd_delta_kernel<<<blocks, 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(d.o), reinterpret_cast<const __nv_bfloat16*>(d.dout),
        d.delta, d.B, d.H, d.Lq, d.o_sb, d.o_sl, d.o_sh, d.stat_ld);
    AVGEN_CUDA_CHECK(cudaGetLastError());
  }
  auto head_major = [&](const void* ptr, int heads, int len, int rows) {
    return make_tmap_3d_bf16(ptr, kHD, len, static_cast<long>(d.B) * heads, kHD, static_cast<long>(len) * kHD, 64,
                             rows, 1);
  };
  auto dout_map = [&](int rows) {
    CUtensorMap m;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(kHD), static_cast<cuuint64_t>(d.H),
                          static_cast<cuuint64_t>(d.Lq), static_cast<cuuint64_t>(d.B)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(kHD) * 2, static_cast<cuuint64_t>(d.H) * kHD * 2,
                             static_cast<cuuint64_t>(d.Lq) * d.H * kHD * 2};
    cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(rows), 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(d.dout), dims,
                                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    AVGEN_CHECK(r == CUDA_SUCCESS, "attention bwd: dO tensor map failed (", static_cast<int>(r), ")");
    return m;
  };
  auto f32_rows = [&](const float* ptr, int box_len) {
    CUtensorMap m;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(d.Lq), static_cast<cuuint64_t>(d.B) * d.H};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(d.stat_ld) * 4};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(box_len), 1};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides,
                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    AVGEN_CHECK(r == CUDA_SUCCESS, "attention bwd: row-stat tensor map failed (", static_cast<int>(r), ")");
    return m;
  };
  if (d.dq_acc != nullptr) {
    // ---- fused: dK, dV and dQ^T partials in one pass, then dQ = scale * acc^T
    const long ld = (d.Lq + 3) / 4 * 4;  // 16-byte rows for the TMA reduce
    if (!d.skip_prologue)
      AVGEN_CUDA_CHECK(cudaMemsetAsync(d.dq_acc, 0, sizeof(float) * ld * kHD * d.B * d.H, stream));
    d.k_tiles = (d.Lk + kTile - 1) / kTile;
    AVGEN_CHECK(d.kt_begin >= 0 && d.kt_count >= 0 && d.kt_begin + d.kt_count <= d.k_tiles,
                "attention bwd: key-tile range outside [0, ", d.k_tiles, ")");
    const bool ring = d.ring_world > 1;
    if (ring)
      AVGEN_CHECK(d.ring_len % kTile == 0 && d.ring_len > 0 && d.Lk == d.ring_world * d.ring_len,
                  "attention bwd ring: keys per rank must be a positive multiple of 128 and Lk = world * that");
    const CUtensorMap tq = head_major(d.q, d.H, d.Lq, kQT);
    const CUtensorMap tk = ring ? head_major(d.k, d.Hk * d.ring_world, d.ring_len, kTile)
                                : head_major(d.k, d.Hk, d.Lk, kTile);
    const CUtensorMap tv = ring ? head_major(d.v, d.Hk * d.ring_world, d.ring_len, kTile)
                                : head_major(d.v, d.Hk, d.Lk, kTile);
    const CUtensorMap tdo = dout_map(kQT);
    const CUtensorMap tl = f32_rows(d.lse, kQT);
    const CUtensorMap tdl = f32_rows(d.delta, kQT);
    CUtensorMap tacc;
    {
      cuuint64_t dims[3] = {static_cast<cuuint64_t>(d.Lq), static_cast<cuuint64_t>(kHD),
                            static_cast<cuuint64_t>(d.B) * d.H};
      cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 4, static_cast<cuuint64_t>(ld) * kHD * 4};
      cuuint32_t box[3] = {32, 32, 1};  // 32 q (128 B, the SW128 span) x 32 d
      cuuint32_t estr[3] = {1, 1, 1};
      CUresult r = tensor_map_encoder()(&tacc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, d.dq_acc, dims, strides, box, estr,
                                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      AVGEN_CHECK(r == CUDA_SUCCESS, "attention bwd: dQ accumulator tensor map failed (", static_cast<int>(r), ")");
    }
    static PerDeviceOnce once_plain, once_trace;
    raise_smem_limit(once_plain, attn_bwd_fused_kernel<false>, FusedBwdSmem::BYTES);
    raise_smem_limit(once_trace, attn_bwd_fused_kernel<true>, FusedBwdSmem::BYTES);
    const long grid = static_cast<long>(d.B) * d.Hk * (d.kt_count > 0 ? d.kt_count : d.k_tiles);
    if (d.trace != nullptr)
      attn_bwd_fused_kernel<true><<<grid, 512, FusedBwdSmem::BYTES, stream>>>(tq, tk, tv, tdo, tl, tdl, tacc, d);
    else
      attn_bwd_fused_kernel<false><<<grid, 512, FusedBwdSmem::BYTES, stream>>>(tq, tk, tv, tdo, tl, tdl, tacc, d);
    AVGEN_CUDA_CHECK(cudaGetLastError());
    if (!d.skip_epilogue) {
      dim3 cgrid((d.Lq + 63) / 64, d.B * d.H);
      attn_dq_convert_kernel<<<cgrid, 256, 0, stream>>>(d.dq_acc, ld, d.Lq, d.scale, d.dq);
      AVGEN_CUDA_CHECK(cudaGetLastError());
    }
    return;
  }
  // ---- dK / dV
  {
    d.k_tiles = (d.Lk + kTile - 1) / kTile;
    const CUtensorMap tq = head_major(d.q, d.H, d.Lq, kQT);
    const CUtensorMap tk = head_major(d.k, d.Hk, d.Lk, kTile);
    const CUtensorMap tv = head_major(d.v, d.Hk, d.Lk, kTile);
    const CUtensorMap tdo = dout_map(kQT);
    const CUtensorMap tl = f32_rows(d.lse, kQT);
    const CUtensorMap tdl = f32_rows(d.delta, kQT);
    static PerDeviceOnce once;
    raise_smem_limit(once, attn_bwd_dkv_kernel, DkvSmem::BYTES);
    const long grid = static_cast<long>(d.B) * d.Hk * d.k_tiles;
    attn_bwd_dkv_kernel<<<grid, 384, DkvSmem::BYTES, stream>>>(tq, tk, tv, tdo, tl, tdl, d);
    AVGEN_CUDA_CHECK(cudaGetLastError());
  }
  // ---- dQ
  {
    d.q_tiles = (d.Lq + 255) / 256;
    const CUtensorMap tq = head_major(d.q, d.H, d.Lq, 128);
    const CUtensorMap tk = head_major(d.k, d.Hk, d.Lk, kKT);
    const CUtensorMap tv = head_major(d.v, d.Hk, d.Lk, kKT);
    const CUtensorMap tdo = dout_map(128);
    static PerDeviceOnce once_masked, once_dense;
    raise_smem_limit(once_masked, attn_bwd_dq_kernel<true>, DqSmem::BYTES);
    raise_smem_limit(once_dense, attn_bwd_dq_kernel<false>, DqSmem::BYTES);
    const long grid = static_cast<long>(d.B) * d.H * d.q_tiles;
    if (d.kmask != nullptr) {
      attn_bwd_dq_kernel<true><<<grid, 384, DqSmem::BYTES, stream>>>(tq, tk, tv, tdo, d);
    } else {
      attn_bwd_dq_kernel<false><<<grid, 384, DqSmem::BYTES, stream>>>(tq, tk, tv, tdo, d);
    }
    AVGEN_CUDA_CHECK(cudaGetLastError());
  }
}

}  // namespace avgen
