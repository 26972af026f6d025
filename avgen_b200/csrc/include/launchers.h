// Torch-free launcher interfaces of the avgen_b200 kernels. The .cu files
// implement them; bindings.cpp validates torch tensors and calls them.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace avgen {

enum GemmEpilogue : int {
  kEpiStore = 0,
  kEpiGateResid = 1,
  kEpiSwiGLU = 2,
  kEpiGelu = 3,
  kEpiAtomicF32 = 4,
};

struct GemmDesc {
  int device = 0;
  int M = 0, N = 0, K = 0;
  const void* a = nullptr;  // bf16, [M, K] (a_mn=false) or [K, M] (a_mn=true)
  long lda = 0;
  bool a_mn = false;
  const void* b = nullptr;  // bf16, [N, K] (b_mn=false) or [K, N] (b_mn=true)
  long ldb = 0;
  bool b_mn = false;
  void* out = nullptr;
  long ldo = 0;
  bool out_f32 = false;
  int epilogue = kEpiStore;
  const float* bias = nullptr;
  const void* resid = nullptr;  // bf16 [M, N]
  long ldr = 0;
  const float* gate = nullptr;  // fp32 [B, gate_stride]
  long gate_stride = 0;
  int rows_per_batch = 1;
  const int* groups = nullptr;  // int32 [M]: gate row of each output row (overrides rows_per_batch)
  int num_groups = 0;           // gate rows; group indices are clamped to [0, num_groups)
  void* aux = nullptr;  // bf16 [M, N]
  long ldaux = 0;
  int k_splits = 1;
  int* err = nullptr;
  // Optional appended reduction pair: D = [A | a2] . [B | b2]^T, a2 [M, K2] and
  // b2 [N, K2] with the majorness of a and b (K2 columns, row strides lda2/ldb2).
  const void* a2 = nullptr;
  long lda2 = 0;
  const void* b2 = nullptr;
  long ldb2 = 0;
  int K2 = 0;
  // Optional gated operand: rows of A (gate_operand 1) or of B (2) in chunks of
  // gate_chunk; a tile touching chunk c != gate_rank waits for gate_flags[c] >= gate_epoch.
  const unsigned* gate_flags = nullptr;
  unsigned gate_epoch = 0;
  int gate_operand = 0;
  int gate_chunk = 0;
  int gate_rank = 0;
};

void gemm_launch(const GemmDesc& d, cudaStream_t stream);

// adaLN RMSNorm. y = rmsnorm(x) * w * (1 + scale[b]) + shift[b] (each optional).
struct NormDesc {
  int device = 0;
  long rows = 0;
  int W = 0;
  long rows_per_batch = 1;
  const int* groups = nullptr;  // int32 [rows]: modulation row of each row (overrides rows_per_batch)
  int num_groups = 0;           // modulation rows; indices are clamped to [0, num_groups)
  float eps = 1e-6f;
  const void* x = nullptr;  // bf16 [rows, W]
  long ldx = 0;
  void* y = nullptr;  // bf16 [rows, W]
  long ldy = 0;
  float* rstd = nullptr;  // fp32 [rows]
  const float* w = nullptr;
  const float* scale = nullptr;  // fp32 [B, mod_stride]
  const float* shift = nullptr;
  long mod_stride = 0;
  // backward
  const void* dy = nullptr;
  long lddy = 0;
  void* dx = nullptr;
  long lddx = 0;
  const void* dres = nullptr;  // optional incoming residual gradient added to dx
  long lddres = 0;
  float* dw = nullptr;
  float* dscale = nullptr;
  float* dshift = nullptr;
  long dmod_stride = 0;
};
void rmsnorm_mod_fwd_launch(const NormDesc& d, cudaStream_t stream);
void rmsnorm_mod_bwd_launch(const NormDesc& d, cudaStream_t stream);

struct GateBwdDesc {
  int device = 0;
  long rows = 0;
  int W = 0;
  long rows_per_batch = 1;
  const int* groups = nullptr;  // int32 [rows]: gate row of each row (overrides rows_per_batch)
  int num_groups = 0;
  const void* dx = nullptr;  // bf16 [rows, W]
  long lddx = 0;
  const void* a = nullptr;  // bf16 [rows, W], the un-gated branch output
  long lda = 0;
  const float* gate = nullptr;  // fp32 [B, gate_stride]
  long gate_stride = 0;
  void* da = nullptr;  // bf16 [rows, W]
  long ldda = 0;
  float* dgate = nullptr;  // fp32 [B, dgate_stride], accumulated
  long dgate_stride = 0;
};
void gate_bwd_launch(const GateBwdDesc& d, cudaStream_t stream);

// QK-RMSNorm + 3-D RoPE + head-major relayout of a fused QKV projection.
struct QkvRopeDesc {
  int device = 0;
  int B = 0, L = 0, H = 0, Hk = 0, D = 0;
  float eps = 1e-6f;
  const void* qkv = nullptr;  // bf16 [B*L, (H + 2Hk) * D]
  long ldqkv = 0;
  const float* q_w = nullptr;  // fp32 [D] or null (no QK norm)
  const float* k_w = nullptr;
  const float* coords = nullptr;  // fp32 [B*L, 3] or null (no rotary)
  const float* freq = nullptr;    // fp32 [D/2]
  const int* axis = nullptr;      // int32 [D/2]
  void* q = nullptr;  // bf16 [B, H, L, D]
  void* k = nullptr;  // bf16 [B, Hk, L, D]
  void* v = nullptr;  // bf16 [B, Hk, L, D]
  // backward
  const void* dq = nullptr;
  const void* dk = nullptr;
  const void* dv = nullptr;
  void* dqkv = nullptr;  // bf16 [B*L, (H + 2Hk) * D]
  long lddqkv = 0;
  float* dq_w = nullptr;
  float* dk_w = nullptr;
};
void qkv_rope_fwd_launch(const QkvRopeDesc& d, cudaStream_t stream);
void qkv_rope_bwd_launch(const QkvRopeDesc& d, cudaStream_t stream);

// Elementwise activations.
void swiglu_bwd_launch(int device, long rows, int F, const void* dh, long lddh, const void* gu,
                       long ldgu, void* dgu, long lddgu, cudaStream_t stream);
void gelu_bwd_launch(int device, long rows, int F, const void* dh, long lddh, const void* pre,
                     long ldpre, void* dpre, long lddpre, cudaStream_t stream);

// Flow-matching loss partials: stats[0] += sum(w_b * mse_tok * m), stats[1] += sum(mse_tok * m),
// stats[2] += sum(m) with mse_tok the mean over the P features of (pred - target)^2.
struct FlowLossDesc {
  int device = 0;
  long rows = 0;
  int P = 0;
  long rows_per_batch = 1;
  const void* pred = nullptr;
  bool pred_f32 = false;
  const void* target = nullptr;
  bool target_f32 = true;
  const uint8_t* mask = nullptr;  // [rows] loss mask
  const float* weight = nullptr;  // [B]
  float* stats = nullptr;         // [3]
  // backward: dpred = scale[0] * 2 (pred - target) / P * w_b * m
  const float* scale = nullptr;
  void* dpred = nullptr;
  bool dpred_f32 = false;
};
void flow_loss_fwd_launch(const FlowLossDesc& d, cudaStream_t stream);
void flow_loss_bwd_launch(const FlowLossDesc& d, cudaStream_t stream);

// Counter-based Gaussian noise (Philox-4x32-10 + Box-Muller) keyed by the global
// element index, and the rectified-flow interpolation
//   noisy = x + t (eps - x),  target = eps - x.
struct NoiseDesc {
  int device = 0;
  long rows = 0;
  int P = 0;
  uint64_t seed = 0;
  uint64_t offset = 0;
  long row_base = 0;        // global index of local row 0 (CP shard start)
  long rows_per_sample = 1; // local rows per sample
  long global_rows_per_sample = 1;
  const void* clean = nullptr;
  bool clean_f32 = true;
  const float* t = nullptr;  // [rows] per-token noise level
  void* noisy = nullptr;     // fp32 [rows, P]
  void* target = nullptr;    // fp32 [rows, P]
  void* noise = nullptr;     // optional fp32 [rows, P]
};
void noise_interp_launch(const NoiseDesc& d, cudaStream_t stream);

// Fused AdamW over a flat fp32 parameter range, with optional bf16 copy-out.
struct AdamWDesc {
  int device = 0;
  long n = 0;
  float* param = nullptr;
  const float* grad = nullptr;
  float* exp_avg = nullptr;
  float* exp_avg_sq = nullptr;
  void* param_bf16 = nullptr;  // optional bf16 compute copy
  float lr = 1e-4f, beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f, weight_decay = 0.f;
  float bias_correction1 = 1.f, bias_correction2_sqrt = 1.f;
  const float* grad_scale = nullptr;  // device scalar multiplying grads (clip); may be null
  const int* skip = nullptr;          // device flag: non-zero treats all gradients as zero
};
// Flash attention (head_dim 128). q: [B, H, Lq, D]; k, v: [B, Hk, Lk, D] (dense,
// head-major); out: token-major with strides (o_sb, o_sl, o_sh); lse: fp32
// [B, H, Lq] in the base-2 domain of the scaled scores.
struct AttnFwdDesc {
  int device = 0;
  int B = 0, H = 0, Hk = 0, Lq = 0, Lk = 0, D = 128;
  int q_tiles = 0;
  float scale_log2 = 0.f;
  const void* q = nullptr;
  const void* k = nullptr;
  const void* v = nullptr;
  const uint32_t* kmask = nullptr;  // packed key-valid bits [B, kmask_words] or null
  int kmask_words = 0;
  __nv_bfloat16* out = nullptr;
  long o_sb = 0, o_sl = 0, o_sh = 0;
  float* lse = nullptr;  // [B, H, Lq] with row stride stat_ld
  long stat_ld = 0;      // floats between (b, h) rows of lse; a multiple of 4
  int* err = nullptr;
  long long* trace = nullptr;  // diagnostics: SM clock stamps of CTA 0 (64 iterations x 24 slots)
  // Context-parallel ring (ring_world > 1): k and v are [ring_world][B * Hk][ring_len][D]
  // with Lk = ring_world * ring_len (ring_len a multiple of 128). Each CTA visits key
  // tiles starting at this rank's own chunk; the first tile of chunk r != ring_rank is
  // loaded only after ring_flags[r] has reached ring_epoch (bounded wait).
  int ring_world = 0;
  int ring_rank = 0;
  int ring_len = 0;
  const unsigned* ring_flags = nullptr;
  unsigned ring_epoch = 0;
  // Optional: SM clock cycles the TMA producers spent waiting on ring_flags, summed
  // over CTAs (exposed-communication accounting).
  unsigned long long* wait_cycles = nullptr;
};
void attn_fwd_launch(const AttnFwdDesc& d, cudaStream_t stream);

struct AttnBwdDesc {
  int device = 0;
  int B = 0, H = 0, Hk = 0, Lq = 0, Lk = 0, D = 128;
  int k_tiles = 0;
  float scale = 0.f;       // softmax scale (dK and dQ are multiplied by it)
  float scale_log2 = 0.f;  // scale * log2(e)
  const void* q = nullptr;
  const void* k = nullptr;
  const void* v = nullptr;
  const void* o = nullptr;     // forward output, token-major dense [B, Lq, H, D]
  const void* dout = nullptr;  // same layout
  long o_sb = 0, o_sl = 0, o_sh = 0;
  const float* lse = nullptr;  // [B, H, Lq], row stride stat_ld
  float* delta = nullptr;      // scratch [B, H, Lq], row stride stat_ld
  long stat_ld = 0;            // floats between (b, h) rows; a multiple of 4 (16-byte TMA rows)
  const uint32_t* kmask = nullptr;
  int kmask_words = 0;
  __nv_bfloat16* dq = nullptr; // [B, H, Lq, D]
  int q_tiles = 0;
  __nv_bfloat16* dk = nullptr; // [B, Hk, Lk, D]
  __nv_bfloat16* dv = nullptr;
  float* dq_acc = nullptr;     // optional fp32 scratch of B*H*128*ld floats, ld = Lq rounded up to 4: selects the fused one-pass kernel
  // Context-parallel ring (ring_world > 1, fused kernel only): k, v, dk and dv are
  // [ring_world][B * Hk][ring_len][D] with Lk = ring_world * ring_len; dk/dv hold this
  // rank's partial gradients for every rank's keys, chunk r contiguous.
  int ring_world = 0;
  int ring_len = 0;
  // Key-tile range of one launch of the fused kernel (kt_count 0 = every tile). A
  // backward split over several launches runs the prologue (delta, dQ scratch
  // reset) only in the first (skip_prologue false) and the dQ conversion only in
  // the last (skip_epilogue false).
  int kt_begin = 0;
  int kt_count = 0;
  bool skip_prologue = false;
  bool skip_epilogue = false;
  long long* trace = nullptr;  // optional int64 [64 * 24]: per-warp SM clock stamps of CTA 0 (diagnostics)
  int* err = nullptr;
};
void attn_bwd_launch(const AttnBwdDesc& d, cudaStream_t stream);

void adamw_launch(const AdamWDesc& d, cudaStream_t stream);
void sq_norm_launch(int device, const float* x, long n, float* out, cudaStream_t stream);
void ema_launch(int device, long n, const float* param, void* shadow, bool shadow_bf16, float decay,
                cudaStream_t stream);

// Guided Euler step over [batch, per_sample] latents: out = x + (sigma_next - sigma) *
// (uncond + scale (cond - uncond)); uncond may be null (plain Euler).
struct GuidedEulerDesc {
  int device = 0;
  int batch = 0;
  long per_sample = 0;
  const void* cond = nullptr;
  const void* uncond = nullptr;
  bool vel_f32 = true;
  const void* x = nullptr;
  bool x_f32 = true;
  void* out = nullptr;
  bool out_f32 = true;
  const float* sigma = nullptr;       // [batch]
  const float* sigma_next = nullptr;  // [batch]
  float scale = 1.f;
};
void guided_euler_launch(const GuidedEulerDesc& d, cudaStream_t stream);

// Flow-GRPO SDE transition over fp32 [batch, per_sample] states; log_prob [batch]
// is accumulated into (zero it first).
struct SDEStepDesc {
  int device = 0;
  int batch = 0;
  long per_sample = 0;
  const void* v = nullptr;
  bool v_f32 = true;
  const float* x = nullptr;
  const float* sigma = nullptr;
  const float* sigma_next = nullptr;
  const float* g = nullptr;      // diffusion coefficient per sample
  float floor = 1e-3f;
  const float* noise = nullptr;  // rollout: standard normal draw
  const float* prev = nullptr;   // update: stored next state
  const bool* mask = nullptr;    // optional element validity
  float* mean = nullptr;
  float* sample = nullptr;       // rollout output
  float* log_prob = nullptr;
};
void sde_step_launch(const SDEStepDesc& d, cudaStream_t stream);

// Peer-memory runtime (p2p.cu).
void* p2p_alloc(size_t bytes, int device);
void p2p_free(void* ptr);
void p2p_export(void* ptr, char* handle64);
void* p2p_open(const char* handle64, int device);
void p2p_close(void* ptr);
void stream_write(cudaStream_t stream, void* flag, unsigned value);
void p2p_copy(void* dst, const void* src, size_t bytes, cudaStream_t stream);
void slab_sum_launch(const void* const* srcs_dev, int nsrc, void* dst, long n, int device, cudaStream_t stream);

// Sharded AdamW over NVLink (zero.cu). grads / params: one flat fp32 buffer
// address per rank (this rank's own included), valid on this device.
void shard_reduce_launch(const float* const* grads, int world, long lo, long n, float* out, float* sq_acc, int device,
                         cudaStream_t stream);
struct ShardAdamWDesc {
  int device = 0;
  int rank = 0, world = 1;
  long lo = 0;    // shard start (elements, multiple of 4)
  long n4 = 0;    // shard length / 4
  const float* grad = nullptr;  // reduced shard gradient [n]
  float* exp_avg = nullptr;     // shard moments [n]
  float* exp_avg_sq = nullptr;
  float lr = 1e-4f, beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f, weight_decay = 0.f;
  float bias_correction1 = 1.f, bias_correction2_sqrt = 1.f;
  const float* grad_scale = nullptr;
  const int* skip = nullptr;
};
void shard_adamw_push_launch(const ShardAdamWDesc& d, const float* const* params, cudaStream_t stream);

// Sharded data parallelism (fsdp.cu). peer_reduce: out[i] = scale * sum over the
// `world` sources (one address per rank, valid on this device) of src[offset + i];
// fp32 or bf16 sources, fp32 out; sq_acc (nullable) accumulates sum(out^2).
void peer_reduce_launch(const void* const* srcs, int world, int rank, long offset, long n, bool src_bf16, float scale,
                        float* out, float* sq_acc, int device, cudaStream_t stream);
// Multi-tensor optimizer kernels: one block per chunk of one tensor row.
struct MTTensor {
  float* param = nullptr;
  const float* grad = nullptr;
  float* exp_avg = nullptr;
  float* exp_avg_sq = nullptr;
};
struct MTChunk {
  int tensor = 0;
  int pad = 0;
  long start = 0;
  long len = 0;
};
struct MTAdamWArgs {
  float lr = 1e-4f, beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f, weight_decay = 0.f;
  float bias_correction1 = 1.f, bias_correction2_sqrt = 1.f;
  const float* grad_scale = nullptr;
  const int* skip = nullptr;
};
void mt_sq_norm_launch(const MTChunk* chunks, int nchunks, const MTTensor* tensors, float* acc, cudaStream_t stream);
void mt_adamw_launch(const MTChunk* chunks, int nchunks, const MTTensor* tensors, const MTAdamWArgs& args,
                     cudaStream_t stream);

}  // namespace avgen
