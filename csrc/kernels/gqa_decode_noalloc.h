// Allocation-free gated-GQA decode step: C ABI.
//
// This entry point has no counterpart in the reference.  It serves callers that
// cannot allocate device memory: host runtimes that reserve all GPU memory for
// their own pool at start-up (serving engines, embedded runtimes), plugin
// interfaces whose contract forbids allocation after initialisation, and
// latency-critical paths that must not risk the implicit device synchronisation
// of cudaMalloc / cudaFree.  The caller passes every input and output; the
// split-KV partials, the merge tickets and the status word live in fixed-size
// file-scope device arrays of csrc/kernels/gqa_decode.cu (4 MiB of partials,
// 4096 tickets), held by every GPU that loads the library until the process
// exits.  Nothing here calls cudaMalloc, cudaFree or an allocating library
// routine.
//
// Sharing rules: every call on a device shares the arrays, and they keep the
// last call's contents.  Calls that overlap on the GPU (different streams with
// no ordering between them) race on the arrays and give wrong results.  The
// first call on a device, with that device current, resolves the arrays' device
// addresses with cudaGetSymbolAddress; make that first call before any stream
// capture that includes this entry point.
//
// Rows whose position lies outside [0, s_max) are inactive: no cache row is
// written or read for them and their output row is zero.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  BWN_NOALLOC_OK = 0,
  BWN_NOALLOC_BAD_ARGUMENT = 1,
  BWN_NOALLOC_SCRATCH_TOO_SMALL = 2,  // batch * q_heads * (4 + 256) floats > 1 Mi, or batch * kv_heads > 4096
  BWN_NOALLOC_CUDA_ERROR = 3,         // symbol lookup, memset, copy or launch failed
  BWN_NOALLOC_INTERNAL_ERROR = 4,
};

// One decode step of gated GQA attention (q RMSNorm + partial RoPE, the new K
// row's RMSNorm + RoPE, K/V append at positions[b], softmax over keys
// 0..positions[b], sigmoid output gate).  bf16 tensors: qg [batch, q_heads, 512]
// (query || gate, row stride qg_stride), k_new / v_new [batch, kv_heads, 256]
// (row stride kv_new_stride), k_cache / v_cache [batch, kv_heads, s_max, 256],
// out [batch, q_heads * 256] (row stride out_stride).  fp32: q_norm_w / k_norm_w
// [256], cos / sin [s_max, rope_dim].  positions: int32 [batch].  splits <= 0
// picks 8; the split count is lowered to what the scratch holds.
int bwn_gqa_decode_noalloc(const void* qg, long qg_stride, const void* k_new, const void* v_new,
                           long kv_new_stride, const float* q_norm_w, const float* k_norm_w, const float* cos,
                           const float* sin, void* k_cache, void* v_cache, const int* positions, void* out,
                           long out_stride, int batch, int q_heads, int kv_heads, int s_max, int rope_dim,
                           float eps, int splits, cudaStream_t stream);

// The device status word of the last bwn_gqa_decode_noalloc call on the current
// device, read after `stream`'s queued work finishes (this call synchronises the
// stream).  *status_out = 0: the kernels completed; non-zero: a bounded
// device-side wait gave up (bit 1: a shared-memory barrier wait), and the output
// of that call must not be used.  Every decode call clears the word when it
// starts.  Returns BWN_NOALLOC_OK, BWN_NOALLOC_BAD_ARGUMENT (null pointer) or
// BWN_NOALLOC_CUDA_ERROR.
int bwn_gqa_decode_noalloc_status(int* status_out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
