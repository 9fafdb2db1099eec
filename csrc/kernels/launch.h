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
  __nv_bfloat16* conv_ring;  // [B, R, C], slot = position & (R - 1)
  int ring_slots;            // R: 4, or 8 when multi-token verify is used
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

// ---- DeltaNet multi-token verify with deferred commit (deltanet_verify.cu) --
struct DnVerifyArgs {
  const __nv_bfloat16* qkv;  // [B*N, C] new tokens, pre-conv (row stride qkv_row)
  long qkv_row;
  const __nv_bfloat16* z;    // [B*N, VH*128]
  long z_row;
  const __nv_bfloat16* a;    // [B*N, VH] (row stride ab_row)
  const __nv_bfloat16* b;
  long ab_row;
  __nv_bfloat16* stash_qkv;  // [2, B, SN, C]     raw rows of the last verify, by step parity
  __nv_bfloat16* stash_ab;   // [2, B, SN, 2*VH]  their a then b
  int stash_n;               // SN >= n_tok (n_tok = 0: commit only)
  const int* vstep;          // verify step counter: read parity vstep&1, write the other
  __nv_bfloat16* conv_ring;  // [B, R, C], R >= N + 3
  int ring_slots;
  void* state;               // [B, VH, 128, 128] committed state
  bool state_bf16;
  const int* positions;      // [B] committed length = position of the first new token; < 0 inactive
  const int* pending;        // [B] accepted tokens of the last verify not yet committed (0..N)
  const float* conv_w;
  const float* A_log;
  const float* dt_bias;
  const float* norm_w;
  __nv_bfloat16* out;        // [B*N, VH*128]
  long out_row;
  int* status;
  int batch, n_tok, k_heads, v_heads;
  float l2_eps, norm_eps;
};
void deltanet_verify(const DnVerifyArgs& p, cudaStream_t stream);
constexpr int kDnVerifyMaxTok = 8;

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
  // multi-token verify: `batch` query rows, n_tok consecutive rows per cache
  // sequence (row r -> cache sequence r / n_tok, position positions[r]).  With
  // n_tok > 1 the new K/V rows are appended by a separate launch first, so
  // every row's attention reads them from the cache; 0 or 1 = decode.
  int n_tok;
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


// ---- ESM-2 rotary embedding + transpose (esm.cu) -----------------------------
struct RopeHalfArgs {
  const __nv_bfloat16* in;   // element (b, s, h, d) at b * in_b + s * in_s + h * in_h + d
  __nv_bfloat16* out;        // element (b, s, h, d) at b * out_b + s * out_s + h * out_h + d
  long in_b, in_s, in_h, out_b, out_s, out_h;
  const float* cos;          // [S, D/2]
  const float* sin;
  int B, S, H, D;
  float sign;                // +1 forward rotation, -1 its transpose (backward)
  float scale;
};
void rope_half(const RopeHalfArgs& a, cudaStream_t stream);

}  // namespace bwn
