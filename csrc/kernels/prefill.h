// Launch descriptors for the prefill kernels (csrc/kernels/prefill.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace bwn {

#ifdef __CUDACC__
// The chunk's start position: the device scalar when given (so one captured
// graph serves every chunk offset of a bucketed prefill), else the host value.
template <class Args>
__device__ __forceinline__ int prefill_start(const Args& p) {
  return p.start_dev ? __ldg(p.start_dev) : p.start;
}
#endif

struct GqaPrefillArgs {
  const __nv_bfloat16* qg;   // [B, S, QH, 512] rows of stride qg_row (query || gate per head)
  long qg_row;
  const __nv_bfloat16* k;    // [B, S, KVH, 256] rows of stride kv_row
  const __nv_bfloat16* v;
  long kv_row;
  const float* q_norm_w;
  const float* k_norm_w;
  const float* cos;          // [S_max, rope_dim]
  const float* sin;
  __nv_bfloat16* k_cache;    // [B, KVH, s_max, 256]
  __nv_bfloat16* v_cache;
  __nv_bfloat16* q_rot;      // scratch [B, QH, S_pad, 256]
  __nv_bfloat16* out;        // [B, S, QH*256] rows of stride out_row
  long out_row;
  int* status;
  const int* start_dev;      // optional device copy of the start position (read at run time; overrides start)
  int batch, S, S_pad, start, q_heads, kv_heads, s_max, rope_dim;
  float eps, scale;
};
void gqa_prefill(const GqaPrefillArgs& p, cudaStream_t stream);

struct DnPrefillArgs {
  const __nv_bfloat16* qkv;  // [B, S, C] rows of stride qkv_row
  long qkv_row;
  const __nv_bfloat16* z;    // [B, S, VH*128] rows of stride z_row
  long z_row;
  const __nv_bfloat16* a;    // [B, S, VH] rows of stride ab_row
  const __nv_bfloat16* b;
  long ab_row;
  __nv_bfloat16* conv_ring;  // [B, R, C], slot = position & (R - 1)
  int ring_slots;            // R (4 or 8)
  void* state;               // [B, VH, 128, 128]
  bool state_bf16;
  const int* valid_len;      // [B]
  const float* conv_w;       // [C, 4]
  const float* A_log;
  const float* dt_bias;
  const float* norm_w;       // [128]
  // scratch
  __nv_bfloat16* q_out;      // [B, KH, S_pad, 128]
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;      // [B, VH, S_pad, 128]
  float* g_out;              // [B, VH, S_pad]
  float* beta_out;
  __nv_bfloat16* out;        // [B, S, VH*128] rows of stride out_row
  long out_row;
  const int* start_dev;      // optional device copy of the start position (read at run time; overrides start)
  int batch, S, S_pad, start, k_heads, v_heads;
  float l2_eps, norm_eps;
  int* status = nullptr;     // device status word (bounded waits of the tensor-core kernel)
};
void deltanet_prefill(const DnPrefillArgs& p, cudaStream_t stream);
// the chunked recurrence on tcgen05 (csrc/kernels/dn_chunk_tc.cu)
bool deltanet_chunk_tc_supported(const DnPrefillArgs& p);
void deltanet_chunk_tc(const DnPrefillArgs& p, int* status, cudaStream_t stream);

}  // namespace bwn
