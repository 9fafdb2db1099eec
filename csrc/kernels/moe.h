// Launch descriptors for the MoE kernels (csrc/kernels/moe.cu).
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace bwn {

struct MoeTopkArgs {
  const float* logits;  // [T, E]
  const float* bias;    // [E] (DeepSeek selection bias) or null
  int T, E, k;
  bool renorm;          // Qwen: renormalise the top-k probabilities
  bool deepseek;        // DeepSeek scoring (sqrt-softplus / sigmoid, route_scale)
  int sqrt_softplus;
  float route_scale;
  float* w;             // [T, k]
  int* ids;             // [T, k]
};
void moe_topk(const MoeTopkArgs& a, cudaStream_t st);

struct MoeRouteArgs {
  const int* ids;       // [T, k] global expert ids
  int T, k, e0, E_local;
  int* counts;          // [E_local]
  int* offsets;         // [E_local + 1]
  int* pos_of;          // [T*k] packed row or -1
  int* row_src;         // [T*k] pair index of each packed row
  const __nv_bfloat16* x;  // [T, H] rows (stride ldx) to gather, or null
  long ldx;
  int H;
  __nv_bfloat16* x_perm;   // [T*k, H]
};
void moe_route(const MoeRouteArgs& a, cudaStream_t st);

struct MoeCombineArgs {
  const __nv_bfloat16* y;  // [T*k, H] packed expert outputs
  const float* w;          // [T, k]
  const int* pos_of;       // [T, k]
  int T, k, H;
  const __nv_bfloat16* shared_y;  // [T, H] or null
  long ld_shared;
  const float* shared_gate;       // [T] pre-sigmoid or null
  __nv_bfloat16* out;
  long ldo;
};
void moe_combine(const MoeCombineArgs& a, cudaStream_t st);

struct GroupedArgs {
  const int* counts;
  const int* offsets;
  int groups, N, K, tiles_m, max_tiles_n;
  __nv_bfloat16* out;
  long ldo;
  int* status;
  float swiglu_limit;  // > 0: gate <= limit, |up| <= limit before silu(gate) * up
};
struct GroupedProblem {
  const void* W;    // [groups * N, K] bf16 (expert-major)
  const void* X;    // [rows_total, K] bf16, expert-major rows
  int rows_total;
  const int* counts;
  const int* offsets;
  int groups, N, K, max_rows_per_group;
  bool swiglu;      // W rows are gate/up interleaved in 16s; out has N/2 columns
  __nv_bfloat16* out;
  long ldo;
  int* status;
  float swiglu_limit = 0.f;
};
void grouped_gemm(const GroupedProblem& p, cudaStream_t st);

// Grouped GEMM with block-scaled E4M3FN expert weights (csrc/kernels/moe_w8.cu).
// ``scales16[e][r / 16][k / 128]``: one fp32 scale per 16 weight rows and 128
// columns (a 128x128 checkpoint block repeats over its 8 row groups; 16-row
// granularity keeps the gate/up interleave exact), value = fp8 * scale.
struct GroupedW8Problem {
  const uint8_t* W;       // [groups * N, K] E4M3FN bytes (expert-major)
  const float* scales16;  // [groups, N / 16, ceil(K / 128)]
  const void* X;          // [rows_total, K] bf16, expert-major rows
  int rows_total;
  const int* counts;
  const int* offsets;
  int groups, N, K, max_rows_per_group;
  bool swiglu;
  __nv_bfloat16* out;
  long ldo;
  int* status;
  float swiglu_limit = 0.f;
};
void grouped_gemm_w8(const GroupedW8Problem& p, cudaStream_t st);

}  // namespace bwn
