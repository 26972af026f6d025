// C interface of the allocation-free attention backward (attention_noalloc.cu).
//
// This entry point has no counterpart in the reference framework, which ships
// no native code. It serves callers that cannot allocate device memory per
// call: a runtime that captures its work into CUDA graphs, or a host process
// that budgets device memory once at start-up. It runs the two-pass attention
// backward with its only scratch (delta = rowsum(dO * O), one fp32 per query
// row) in a file-scope device array.
//
// Contract
//  * Scratch limit: B * H * lse_ld fp32 values <= 1,048,576 (4 MiB per device,
//    e.g. 20 heads x 52,428 query rows); larger calls return status 2 and launch
//    nothing.
//  * One scratch array per device, shared by every call and kept until the
//    process exits. Calls whose work overlaps on the GPU (two streams, two host
//    threads) race on it: serialise them on one stream. Its contents persist
//    between calls (the last call's delta).
//  * The first call on a device resolves the array's device address with
//    cudaGetSymbolAddress (once per device); make that first call outside any
//    stream capture.
//  * `stream` must belong to the current device (status 1 otherwise).
//  * Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
//
// Status codes: 0 ok, 1 invalid argument, 2 scratch limit exceeded, 3 CUDA error
// while resolving the device arrays, 4 launch error. The message of the last
// failing call on the calling host thread is avgen_attn_bwd_noalloc_last_error().
//
// Kernels that give up a bounded wait record a non-zero code in a device error
// word of this entry point (codes 1-6 of the kernels' error enumeration; 0 means
// none). The launch status cannot report it, since the kernels run after the
// call returns: read it with avgen_attn_bwd_noalloc_device_error.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

// q [B, H, Lq, 128], k / v [B, Hk, Lk, 128], o / dout [B, Lq, H, 128], dense
// bf16; lse fp32 [B, H, Lq] with row stride lse_ld (a multiple of 4, >= Lq);
// dq / dk / dv bf16 outputs shaped like q / k / v; kmask packed key-valid bits
// [B, kmask_words] or null; stream is a cudaStream_t (null: the legacy stream).
int avgen_attn_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                           const float* lse, long lse_ld, void* dq, void* dk, void* dv, const unsigned int* kmask,
                           int kmask_words, int B, int H, int Hk, int Lq, int Lk, float scale, void* stream);

// Message of the last failing call on this host thread ("" if none).
const char* avgen_attn_bwd_noalloc_last_error(void);

// Waits for all work on the current device, stores this entry point's device
// error word into *out and, when `clear` is non-zero, resets it to 0. Returns
// 0, or 3 on a CUDA error (with *out untouched).
int avgen_attn_bwd_noalloc_device_error(int* out, int clear);

#ifdef __cplusplus
}
#endif
