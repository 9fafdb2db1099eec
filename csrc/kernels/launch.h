// Launch descriptors and host entry points of the bwn CUDA kernels.  The torch
// bindings (csrc/ops.cpp) validate tensors and fill these structs; kernels see
// raw pointers only, so the .cu files compile without torch headers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace bwn {

// ---- DeltaNet recurrent decode (deltanet_decode.cu) -------------------------
struct DeltaNetDecodeArgs {
  const __nv_bfloat16* qkv;  // [B, C] (row stride qkv_stride), pre-conv
  long qkv_stride;
  const __nv_bfloat16* z;    // [B, VH*128]
  long z_stride;
  const __nv_bfloat16* a;    // [B, VH]  (row stride ab_stride)
  const __nv_bfloat16* b;
  long ab_stride;
  __nv_bfloat16* conv_ring;  // [B, 4, C]
  void* state;               // [B, VH, 128, 128] fp32 or bf16
  bool state_bf16;
  const int* positions;      // [B]; < 0 = inactive row
  const float* conv_w;       // [C, 4]
  const float* A_log;        // [VH]
  const float* dt_bias;      // [VH]
  const float* norm_w;       // [128]
  __nv_bfloat16* out;        // [B, VH*128]
  long out_stride;
  int batch, k_heads, v_heads;
  float l2_eps, norm_eps;
};
void deltanet_decode(const DeltaNetDecodeArgs& p, cudaStream_t stream);

// ---- gated GQA decode (gqa_decode.cu) ---------------------------------------
struct GqaDecodeArgs {
  const __nv_bfloat16* qg;   // [B, QH, 512] query||gate per head (pre-norm)
  long qg_stride;            // row stride (elements) between sequences
  const __nv_bfloat16* k_new;  // [B, KVH, 256] pre-norm
  const __nv_bfloat16* v_new;  // [B, KVH, 256]
  long kv_new_stride;
  const float* q_norm_w;     // [256]
  const float* k_norm_w;     // [256]
  const float* cos;          // [S_max, rope_dim]
  const float* sin;
  __nv_bfloat16* k_cache;    // [B, KVH, S_max, 256]
  __nv_bfloat16* v_cache;
  const int* positions;      // [B]
  __nv_bfloat16* out;        // [B, QH*256]
  long out_stride;
  float* workspace;          // [B, KVH, splits, G, 2 + 256]
  int* tickets;              // [B * KVH]
  int* status;
  int batch, q_heads, kv_heads, s_max, rope_dim, splits;
  float eps;
};
void gqa_decode(const GqaDecodeArgs& p, cudaStream_t stream);
int gqa_decode_workspace_floats(int batch, int q_heads, int kv_heads, int splits);

// ---- norms / elementwise (norm.cu) ------------------------------------------
// out = rmsnorm(x) * (1 + w)    (one_plus) or * w
void rms_norm(const __nv_bfloat16* x, long ldx, const float* w, __nv_bfloat16* out, long ldo, int rows, int cols,
              float eps, bool one_plus, cudaStream_t stream);
// residual += x ; out = rmsnorm(residual) * (1 + w)
void add_rms_norm(const __nv_bfloat16* x, long ldx, __nv_bfloat16* residual, long ldr, const float* w,
                  __nv_bfloat16* out, long ldo, int rows, int cols, float eps, cudaStream_t stream);
// out[t] = table[ids[t] - offset] if in [0, rows) else 0
void embedding(const int* ids, int n, const __nv_bfloat16* table, long rows, int cols, long offset,
               __nv_bfloat16* out, cudaStream_t stream);
// per row: packed key = (orderable(max value) << 32) | (0xFFFFFFFF - global id)
// so that an int64 max-reduction picks the largest value, lowest id on ties.
void argmax_packed(const float* logits, long ld, int rows, int cols, long id_offset, int64_t* out,
                   cudaStream_t stream);
void argmax_packed_bf16(const __nv_bfloat16* logits, long ld, int rows, int cols, long id_offset, int64_t* out,
                        cudaStream_t stream);
void unpack_argmax(const int64_t* packed, int rows, int* ids_out, cudaStream_t stream);

}  // namespace bwn
