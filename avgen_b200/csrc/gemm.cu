// tcgen05 GEMM for sm_100a with fused epilogues.
//
//   D[M, N] = A[M, K] . B[N, K]^T        (bf16 operands, fp32 accumulation in TMEM)
//
// This one kernel serves every linear layer of the DiT block, forward and
// backward. It replaces the cuBLAS calls behind `nn.Linear` in the reference
// (avgen/models/layers.py:382-433, 436-686) and fuses the elementwise work that
// follows each of them there:
//   * kEpiStore       D = acc (+ bias)
//   * kEpiGateResid   D = R + gate[b, n] * (acc + bias)        gated residual of
//                     avgen/models/blocks.py:207-227 (aux = un-gated acc)
//   * kEpiSwiGLU      acc columns (2j, 2j+1) hold (gate_j, up_j); D[:, j] =
//                     silu(gate) * up (avgen/models/layers.py:420); aux = acc
//   * kEpiGelu        D = gelu_tanh(acc + bias); aux = pre-activation
//   * kEpiAtomicF32   D += acc with fp32 vector atomics: weight gradients
//                     accumulate straight into fp32 gradient buffers, which also
//                     makes split-K free.
//
// Operand majorness: A and B are each K-major (the reduction axis contiguous,
// like x and W of nn.Linear) or MN-major (used by the backward GEMMs dX = dY.W and
// dW = dY^T.X without materialised transposes).
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128x64 A and BNx64 B tiles into a STAGES-deep ring
//   warp 1      MMA issuer: one thread issues tcgen05.mma 128xBNx16, commits to
//               the ring's empty barriers and to the accumulator-full barrier
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (each thread owns one
//               row), fused math, vector stores to global memory
// The accumulator is double buffered in TMEM (2 x BN fp32 columns) so the
// epilogue of tile i overlaps the MMAs of tile i+1.
//
// Appended reduction pair: an optional second operand pair (A2[M, K2], B2[N, K2],
// same majorness as A and B) extends the reduction, D = [A | A2] . [B | B2]^T,
// so a low-rank update accumulates into the same TMEM tile as the dense product.
// This is how LoRA runs without a second pass over the output: forward
// y = x W^T + (x A^T s) B^T and input gradient dx = dy W + (dy B) (s A), the
// rank-r factors riding as K2 = r extra reduction columns (the reference adds
// the two products in eager PyTorch, avgen/finetune/lora.py:692-715).
//
// Gated operand (all-gather fused into the GEMM): the rows of A (M) or of B (N)
// are split into equal chunks, chunk r arriving from rank r over NVLink while the
// kernel runs. Before its first k-block of a tile, the producer waits (bounded,
// acquire at system scope) until every chunk the tile touches has its flag at the
// call's epoch; the copy stream writes that flag after the chunk's copy lands.
// Tiles are rotated so this rank's own chunk is computed first, and peer chunks
// follow in the order they are pulled, so each transfer hides behind the MMAs of
// the chunks before it. This replaces the NCCL all-gather that precedes the
// FSDP weight GEMM (avgen/parallel/fsdp.py:75-124) and the sequence-parallel
// activation GEMM of tensor parallelism (avgen/parallel/tensor.py:112-128) in the
// reference.
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "include/host_utils.h"
#include "include/launchers.h"
#include "include/sm100.cuh"

namespace avgen {

struct GemmArgs {
  int M, N, K;
  int k_splits;
  int kb_per_split;
  int kb2;  // k-blocks of the appended pair, issued by the last split only
  const unsigned* gate_flags;  // arrival word per chunk (nullptr: no gating)
  unsigned gate_epoch;
  int gate_operand;  // 1: chunks of A's rows (M), 2: chunks of B's rows (N)
  int gate_chunk;    // rows per chunk
  int gate_rank;     // this rank's chunk (never waited on)
  int rot_m, rot_n;  // tile rotation that puts the own chunk first
  void* out;
  long ldo;
  const float* bias;
  const __nv_bfloat16* resid;
  long ldr;
  const float* gate;
  long gate_stride;
  int rows_per_batch;
  const int* groups;
  int num_groups;
  __nv_bfloat16* aux;
  long ldaux;
  int* err;
};

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
// Epilogue warps per CTA: 4 (one per TMEM lane quadrant) or 8 (two per quadrant,
// each taking half of a tile's columns); see epi_warps_setting.
constexpr int threads_for(int epi_warps) { return 64 + 32 * epi_warps; }

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

// Grouped raster over (m, n) tiles: 16 M-tiles share each sweep over N so B
// tiles stay resident in L2.
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& tm, int& tn) {
  constexpr int G = 16;
  const int per_group = G * num_n;
  const int group = t / per_group;
  const int first_m = group * G;
  const int gsize = min(num_m - first_m, G);
  const int r = t - group * per_group;
  tm = first_m + r % gsize;
  tn = r / gsize;
}

__device__ __forceinline__ void rotated_coords(const GemmArgs& a, int t, int num_m, int num_n, int& tm, int& tn) {
  tile_coords(t, num_m, num_n, tm, tn);
  tm = (tm + a.rot_m) % num_m;
  tn = (tn + a.rot_n) % num_n;
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float u = k0 * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanhf(u));
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float* v, int valid) {
  if (valid >= 32) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 w;
      w.x = pack_bf16(v[8 * j + 0], v[8 * j + 1]);
      w.y = pack_bf16(v[8 * j + 2], v[8 * j + 3]);
      w.z = pack_bf16(v[8 * j + 4], v[8 * j + 5]);
      w.w = pack_bf16(v[8 * j + 6], v[8 * j + 7]);
      d4[j] = w;
    }
  } else {
    for (int i = 0; i < valid; ++i) dst[i] = __float2bfloat16_rn(v[i]);
  }
}

__device__ __forceinline__ void store_f32x32(float* dst, const float* v, int valid) {
  if (valid >= 32) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int j = 0; j < 8; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
    for (int i = 0; i < valid; ++i) dst[i] = v[i];
  }
}

template <int EPI, bool OUT_F32>
__device__ __forceinline__ void epilogue_row(const GemmArgs& a, int row, int col0,
                                             const uint32_t (&r)[32]) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  const int valid = min(32, a.N - col0);
  if (valid <= 0) return;
  if (a.bias != nullptr && EPI != kEpiAtomicF32) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += (i < valid) ? a.bias[col0 + i] : 0.0f;
  }
  if constexpr (EPI == kEpiStore) {
    if constexpr (OUT_F32) {
      store_f32x32(reinterpret_cast<float*>(a.out) + row * a.ldo + col0, v, valid);
    } else {
      store_bf16x32(reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.ldo + col0, v, valid);
    }
  } else if constexpr (EPI == kEpiAtomicF32) {
    float* dst = reinterpret_cast<float*>(a.out) + row * a.ldo + col0;
    if (valid >= 32) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        atomicAdd(reinterpret_cast<float4*>(dst) + j,
                  make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
      }
    } else {
      for (int i = 0; i < valid; ++i) atomicAdd(dst + i, v[i]);
    }
  } else if constexpr (EPI == kEpiGateResid) {
    if (a.aux != nullptr) store_bf16x32(a.aux + row * a.ldaux + col0, v, valid);
    const float* g = (a.gate != nullptr)
                         ? a.gate + mod_row(a.groups, a.num_groups, row, a.rows_per_batch) * a.gate_stride + col0
                         : nullptr;
    const __nv_bfloat16* res = a.resid + row * a.ldr + col0;
    float o[32];
    if (valid >= 32) {
      const uint4* r4 = reinterpret_cast<const uint4*>(res);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 w = r4[j];
        o[8 * j + 0] = bf16_lo(w.x); o[8 * j + 1] = bf16_hi(w.x);
        o[8 * j + 2] = bf16_lo(w.y); o[8 * j + 3] = bf16_hi(w.y);
        o[8 * j + 4] = bf16_lo(w.z); o[8 * j + 5] = bf16_hi(w.z);
        o[8 * j + 6] = bf16_lo(w.w); o[8 * j + 7] = bf16_hi(w.w);
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] += (g ? g[i] : 1.0f) * v[i];
    } else {
      for (int i = 0; i < valid; ++i) o[i] = __bfloat162float(res[i]) + (g ? g[i] : 1.0f) * v[i];
    }
    store_bf16x32(reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.ldo + col0, o, valid);
  } else if constexpr (EPI == kEpiSwiGLU) {
    if (a.aux != nullptr) store_bf16x32(a.aux + row * a.ldaux + col0, v, valid);
    float h[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) h[j] = silu(v[2 * j]) * v[2 * j + 1];
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.ldo + col0 / 2;
    const int hv = valid / 2;
    if (hv >= 16) {
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint4 w;
        w.x = pack_bf16(h[8 * j + 0], h[8 * j + 1]);
        w.y = pack_bf16(h[8 * j + 2], h[8 * j + 3]);
        w.z = pack_bf16(h[8 * j + 4], h[8 * j + 5]);
        w.w = pack_bf16(h[8 * j + 6], h[8 * j + 7]);
        d4[j] = w;
      }
    } else {
      for (int i = 0; i < hv; ++i) dst[i] = __float2bfloat16_rn(h[i]);
    }
  } else if constexpr (EPI == kEpiGelu) {
    if (a.aux != nullptr) store_bf16x32(a.aux + row * a.ldaux + col0, v, valid);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
    store_bf16x32(reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.ldo + col0, v, valid);
  }
}

// Bounded wait used only on the abort path (ignores the abort flag).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(a, parity)) {
    if (globaltimer() - t0 > kWaitTimeoutNs) return;
  }
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool OUT_F32, int EW>
__global__ void __launch_bounds__(threads_for(EW), 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmA2,
                      const __grid_constant__ CUtensorMap tmB2, const GemmArgs args) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int num_m = (args.M + kBM - 1) / kBM;
  const int num_n = (args.N + BN - 1) / BN;
  const int tiles_mn = num_m * num_n;
  const int num_tiles = tiles_mn * args.k_splits;
  const int num_kb = (args.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 32 * EW);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (args.kb2 > 0) {
      prefetch_tmap(&tmA2);
      prefetch_tmap(&tmB2);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool aborted = false;
      uint32_t ready = 0;  // chunks already seen at the epoch
      for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x) {
        const int split = t / tiles_mn;
        int tm, tn;
        rotated_coords(args, t - split * tiles_mn, num_m, num_n, tm, tn);
        if (args.gate_flags != nullptr) {
          // Wait for every chunk this tile reads (at most two for chunk >= tile).
          const bool on_m = args.gate_operand == 1;
          const int lo = on_m ? tm * kBM : tn * BN;
          const int hi = min(on_m ? args.M : args.N, lo + (on_m ? kBM : BN)) - 1;
          for (int c = lo / args.gate_chunk; c <= hi / args.gate_chunk && !aborted; ++c) {
            if (c == args.gate_rank || ((ready >> c) & 1u)) continue;
            if (!flag_wait_geq(args.gate_flags + c, args.gate_epoch, abort_flag, args.err, kErrTimeoutPeer)) {
              aborted = true;
            } else {
              ready |= 1u << c;
            }
          }
          if (aborted) break;
        }
        const int kb0 = split * args.kb_per_split;
        const int kb1 = min(num_kb, kb0 + args.kb_per_split);
        const int kend = kb1 + (split == args.k_splits - 1 ? args.kb2 : 0);
        for (int kb = kb0; kb < kend; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, args.err, kErrTimeoutProducer)) {
            aborted = true;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          // Blocks past the first pair's reduction come from the appended pair
          // (out-of-range K2 columns are zero-filled by TMA and count in full).
          const bool second = kb >= num_kb;
          const CUtensorMap* mapA = second ? &tmA2 : &tmA;
          const CUtensorMap* mapB = second ? &tmB2 : &tmB;
          const int k0 = (second ? kb - num_kb : kb) * kBK;
          if constexpr (!A_MN) {
            tma_load_2d(sa, mapA, &full[stage], k0, tm * kBM);
          } else {
            tma_load_2d(sa, mapA, &full[stage], tm * kBM, k0);
            tma_load_2d(sa + 8192, mapA, &full[stage], tm * kBM + 64, k0);
          }
          if constexpr (!B_MN) {
            tma_load_2d(sb, mapB, &full[stage], k0, tn * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) {
              tma_load_2d(sb + j * 8192, mapB, &full[stage], tn * BN + 64 * j, k0);
            }
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (aborted) {
        // Let the copies already in flight land before the CTA's shared memory
        // goes away.
        const int inflight = min(issued, STAGES);
        for (int i = 0; i < inflight; ++i) {
          if (--stage < 0) {
            stage = STAGES - 1;
            phase ^= 1;
          }
          drain_wait(&full[stage], phase);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_bf16_f32(kBM, BN, A_MN, B_MN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool aborted = false;
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x) {
      const int split = t / tiles_mn;
      const int kb0 = split * args.kb_per_split;
      const int kb1 = min(num_kb, kb0 + args.kb_per_split);
      const int kend = kb1 + (split == args.k_splits - 1 ? args.kb2 : 0);
      if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, args.err, kErrTimeoutMma)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
      for (int kb = kb0; kb < kend; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag, args.err, kErrTimeoutMma)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        if (elect_one()) {
          const uint32_t a_base = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t b_base = a_base + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = A_MN ? umma_desc_sw128(a_base + k * 2048, 8192, 1024)
                                     : umma_desc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? umma_desc_sw128(b_base + k * 2048, 8192, 1024)
                                     : umma_desc_sw128(b_base + k * 32, 16, 1024);
            mma_bf16_ss(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (aborted) break;
      if (elect_one()) mma_commit(&tfull[acc]);
      __syncwarp();
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warps 2..: warp w reads TMEM lane quadrant w % 4 (the only lanes it may
    // access) and the part (w - 2) / 4 of the tile's columns. The next 32-column
    // chunk is loaded from TMEM while the current one is converted and stored.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    constexpr int HALF = BN / (EW / 4);
    const int row_in_tile = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      const int split = t / tiles_mn;
      int tm, tn;
      rotated_coords(args, t - split * tiles_mn, num_m, num_n, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, args.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const int row = tm * kBM + row_in_tile;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(acc * BN + half * HALF);
      const int col_base = tn * BN + half * HALF;
      uint32_t r[2][32];
      tmem_ld32(t_row, r[0]);
#pragma unroll
      for (int c = 0; c < HALF / 32; ++c) {
        tmem_wait_ld();
        if (c + 1 < HALF / 32) tmem_ld32(t_row + 32 * (c + 1), r[(c + 1) & 1]);
        if (row < args.M) epilogue_row<EPI, OUT_F32>(args, row, col_base + 32 * c, r[c & 1]);
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// Epilogue warps. In isolation on B200 (65536-row GEMMs) eight warps cut the
// SwiGLU-epilogue GEMM from 9.17 to 7.02 ms (N=20480, K=2560) and the fp32
// atomic weight-gradient epilogue by ~5%, while the gated-residual epilogue
// (per-row residual loads) ran 12% slower (0.894 -> 1.005 ms, N=2560, K=2560).
// Inside the full training step, which runs at the 1 kW power cap, eight warps
// measured 1-2% slower per step at equal clocks, so four is the default;
// AVGEN_GEMM_EPI_WARPS=8 selects eight.
inline int epi_warps_setting(int /*epi*/) {
  static const int forced = [] {
    const char* e = std::getenv("AVGEN_GEMM_EPI_WARPS");
    return e == nullptr ? 0 : std::atoi(e);
  }();
  return forced == 8 ? 8 : 4;
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool OUT_F32, int EW>
void launch_gemm_ew(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta2,
                    const CUtensorMap& tb2, const GemmArgs& args, cudaStream_t stream, int num_sms) {
  using Cfg = GemmCfg<BN>;
  auto kernel = gemm_sm100_kernel<BN, A_MN, B_MN, EPI, OUT_F32, EW>;
  static PerDeviceOnce once;
  raise_smem_limit(once, kernel, Cfg::SMEM_BYTES);
  const int num_m = (args.M + kBM - 1) / kBM;
  const int num_n = (args.N + BN - 1) / BN;
  const int tiles = num_m * num_n * args.k_splits;
  const int grid = std::max(1, std::min(tiles, num_sms));
  kernel<<<grid, threads_for(EW), Cfg::SMEM_BYTES, stream>>>(ta, tb, ta2, tb2, args);
  AVGEN_CUDA_CHECK(cudaGetLastError());
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool OUT_F32>
void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta2,
                 const CUtensorMap& tb2, const GemmArgs& args, cudaStream_t stream, int num_sms) {
  if (epi_warps_setting(EPI) == 4)
    launch_gemm_ew<BN, A_MN, B_MN, EPI, OUT_F32, 4>(ta, tb, ta2, tb2, args, stream, num_sms);
  else
    launch_gemm_ew<BN, A_MN, B_MN, EPI, OUT_F32, 8>(ta, tb, ta2, tb2, args, stream, num_sms);
}

}  // namespace

// Launcher (torch-free; the Python binding validates tensors and fills `d`).
void gemm_launch(const GemmDesc& d, cudaStream_t stream) {
  const bool a_mn = d.a_mn, b_mn = d.b_mn;
  const int M = d.M, N = d.N, K = d.K;
  AVGEN_CHECK(M > 0 && N > 0 && K > 0, "gemm: empty problem");
  AVGEN_CHECK(N % 8 == 0, "gemm: N must be a multiple of 8, got ", N);
  AVGEN_CHECK((d.lda * 2) % 16 == 0 && (d.ldb * 2) % 16 == 0,
              "gemm: operand row strides must be 16-byte aligned");
  AVGEN_CHECK(reinterpret_cast<uintptr_t>(d.a) % 16 == 0 && reinterpret_cast<uintptr_t>(d.b) % 16 == 0,
              "gemm: operands must be 16-byte aligned");
  GemmArgs args{};
  args.M = M;
  args.N = N;
  args.K = K;
  const int num_kb = (K + kBK - 1) / kBK;
  int splits = std::max(1, d.k_splits);
  if (d.epilogue != kEpiAtomicF32) splits = 1;
  splits = std::min(splits, num_kb);
  args.kb_per_split = (num_kb + splits - 1) / splits;
  args.k_splits = (num_kb + args.kb_per_split - 1) / args.kb_per_split;
  args.out = d.out;
  args.ldo = d.ldo;
  args.bias = d.bias;
  args.resid = reinterpret_cast<const __nv_bfloat16*>(d.resid);
  args.ldr = d.ldr;
  args.gate = d.gate;
  args.gate_stride = d.gate_stride;
  args.rows_per_batch = std::max(1, d.rows_per_batch);
  args.groups = d.groups;
  args.num_groups = d.num_groups;
  args.aux = reinterpret_cast<__nv_bfloat16*>(d.aux);
  args.ldaux = d.ldaux;
  args.err = d.err;

  constexpr int BN = 256;
  CUtensorMap ta, tb;
  if (!a_mn) {
    ta = make_tmap_2d_bf16(d.a, K, M, d.lda, kBK, kBM);
  } else {
    ta = make_tmap_2d_bf16(d.a, M, K, d.lda, 64, kBK);
  }
  if (!b_mn) {
    tb = make_tmap_2d_bf16(d.b, K, N, d.ldb, kBK, BN);
  } else {
    tb = make_tmap_2d_bf16(d.b, N, K, d.ldb, 64, kBK);
  }
  // Appended pair: same majorness as (A, B), reduction length K2.
  CUtensorMap ta2 = ta, tb2 = tb;
  args.kb2 = 0;
  if (d.a2 != nullptr || d.b2 != nullptr) {
    const int K2 = d.K2;
    AVGEN_CHECK(d.a2 != nullptr && d.b2 != nullptr && K2 > 0, "gemm: the appended pair needs a2, b2 and K2 > 0");
    AVGEN_CHECK((d.lda2 * 2) % 16 == 0 && (d.ldb2 * 2) % 16 == 0,
                "gemm: appended operand row strides must be 16-byte aligned");
    AVGEN_CHECK(reinterpret_cast<uintptr_t>(d.a2) % 16 == 0 && reinterpret_cast<uintptr_t>(d.b2) % 16 == 0,
                "gemm: appended operands must be 16-byte aligned");
    AVGEN_CHECK(a_mn || K2 % 8 == 0, "gemm: K2 of a K-major appended A must be a multiple of 8");
    ta2 = !a_mn ? make_tmap_2d_bf16(d.a2, K2, M, d.lda2, kBK, kBM) : make_tmap_2d_bf16(d.a2, M, K2, d.lda2, 64, kBK);
    tb2 = !b_mn ? make_tmap_2d_bf16(d.b2, K2, N, d.ldb2, kBK, BN) : make_tmap_2d_bf16(d.b2, N, K2, d.ldb2, 64, kBK);
    args.kb2 = (K2 + kBK - 1) / kBK;
  }
  args.gate_flags = nullptr;
  args.rot_m = args.rot_n = 0;
  if (d.gate_flags != nullptr) {
    AVGEN_CHECK(d.gate_operand == 1 || d.gate_operand == 2, "gemm: gate_operand must be 1 (A rows) or 2 (B rows)");
    const int extent = d.gate_operand == 1 ? M : N;
    AVGEN_CHECK(d.gate_chunk > 0 && (extent + d.gate_chunk - 1) / d.gate_chunk <= 32,
                "gemm: gated operand needs 1..32 chunks, got chunk ", d.gate_chunk, " of ", extent, " rows");
    AVGEN_CHECK(d.gate_rank >= 0 && d.gate_rank * d.gate_chunk < extent, "gemm: gate_rank out of range");
    args.gate_flags = d.gate_flags;
    args.gate_epoch = d.gate_epoch;
    args.gate_operand = d.gate_operand;
    args.gate_chunk = d.gate_chunk;
    args.gate_rank = d.gate_rank;
    if (d.gate_operand == 1) args.rot_m = d.gate_rank * d.gate_chunk / kBM;
    else args.rot_n = d.gate_rank * d.gate_chunk / BN;
  }
  const int sms = num_sms(d.device);
  const int epilogue = d.epilogue;
  const bool out_f32 = d.out_f32;

#define AVGEN_GEMM_CASE(AMN, BMN, EPI, F32)                                  \
  if (a_mn == AMN && b_mn == BMN && epilogue == EPI && out_f32 == F32) {    \
    launch_gemm<BN, AMN, BMN, EPI, F32>(ta, tb, ta2, tb2, args, stream, sms); \
    return;                                                                  \
  }
  AVGEN_GEMM_CASE(false, false, kEpiStore, false)
  AVGEN_GEMM_CASE(false, false, kEpiStore, true)
  AVGEN_GEMM_CASE(false, false, kEpiGateResid, false)
  AVGEN_GEMM_CASE(false, false, kEpiSwiGLU, false)
  AVGEN_GEMM_CASE(false, false, kEpiGelu, false)
  AVGEN_GEMM_CASE(false, false, kEpiAtomicF32, true)
  AVGEN_GEMM_CASE(false, true, kEpiStore, false)
  AVGEN_GEMM_CASE(false, true, kEpiStore, true)
  AVGEN_GEMM_CASE(true, true, kEpiStore, true)
  AVGEN_GEMM_CASE(true, true, kEpiAtomicF32, true)
#undef AVGEN_GEMM_CASE
  AVGEN_CHECK(false, "gemm: unsupported combination a_mn=", a_mn, " b_mn=", b_mn,
              " epilogue=", epilogue, " out_f32=", out_f32);
}

}  // namespace avgen
