// Launch descriptors for the DeepSeek V4 kernels (csrc/kernels/deepseek.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace bwn {

struct HcPreArgs {
  const __nv_bfloat16* x;  // [T, hc, dim]
  const float* fn;         // [mix_out, hc*dim]
  const float* scale;      // [3] (pre, post, comb) or [1] for the head
  const float* base;       // [mix_out]
  int tokens, hc, dim, mix_out, sinkhorn_iters;
  float eps, norm_eps;
  __nv_bfloat16* y;        // [T, dim]
  float* post;             // [T, hc]       (mix_out == (2+hc)*hc)
  float* comb;             // [T, hc, hc]
  const float* mix_in = nullptr;  // optional [T, ld_mix]: x . fn^T already computed (one GEMM over
  int ld_mix = 0;                 // all tokens); the kernel then only adds the rms scale
};
void hc_pre(const HcPreArgs& a, cudaStream_t st);
void hc_post(const __nv_bfloat16* x, const __nv_bfloat16* resid, const float* post, const float* comb, int tokens,
             int hc, int dim, __nv_bfloat16* out, cudaStream_t st);

struct MqaArgs {
  const __nv_bfloat16* q;   // [rows, H, D] (normalised, roped)
  const __nv_bfloat16* kv;  // [B, T, D] shared key/value rows
  long kv_seq_stride;       // elements between sequences of kv
  const int* visible;       // [rows] number of visible keys of each query row
  int rows, q_per_seq, H, D, splits;
  float scale;
  float* workspace;         // [rows, splits, H, 2 + D]
  int* tickets;             // [rows]
  __nv_bfloat16* out;       // [rows, H, D]
};
void mqa_attn(const MqaArgs& a, cudaStream_t st);
// prefill-sized MQA on tcgen05 (csrc/kernels/mqa_tc.cu): head dim 512, 128 % H == 0,
// (rows * H) % 128 == 0, whole row tiles per sequence, kv rows per sequence % 32 == 0
bool mqa_prefill_tc_supported(const MqaArgs& a, int kv_rows_per_seq);
void mqa_prefill_tc(const MqaArgs& a, int kv_rows_per_seq, long kv_total_rows, int* status, cudaStream_t st);
void rope_interleaved(__nv_bfloat16* x, int rows, int H, int D, int half, const float* cos, const float* sin,
                      const int* pos, cudaStream_t st);

}  // namespace bwn
