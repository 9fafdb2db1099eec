// Launch descriptors for the MoE kernels (csrc/kernels/moe.cu).
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common/host.h"

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

// ---- decode-sized MoE block (csrc/kernels/moe_decode.cu) ---------------------
constexpr int kMoeDecodeMaxGroups = 320;  // local experts + the shared-expert group

// Router GEMV (+ shared-gate row) -> grid barrier -> softmax / top-k /
// renormalise -> stable expert-major packing (+ the shared expert as group
// E_local over tokens [t_lo, t_hi)) -> gather of the packed rows, one launch.
struct MoeRouteFusedArgs {
  const __nv_bfloat16* x;       // [T, H] normed hidden (row stride ldx)
  long ldx;
  const __nv_bfloat16* router;  // [E (+1), H]: routed experts' rows, then the shared gate row when has_sg
  int T, H, E, k;
  bool renorm, has_sg;
  int e0, E_local;              // this rank's experts [e0, e0 + E_local)
  bool shared_group;            // pack the shared expert as group E_local
  int t_lo, t_hi;               // tokens whose shared-expert rows this rank computes
  float* logits;                // [T, E (+1)] scratch
  unsigned* bar;                // [64] grid barrier: arrivals at [0], generation at [32]; zero before first use
  float* w;                     // [T, k] routing weights
  int* ids;                     // [T, k] expert ids
  float* sg;                    // [T] shared-gate logit (0 without has_sg)
  int* counts;                  // [G] rows per group
  int* offsets;                 // [G + 1]
  int* pos_of;                  // [T * k] packed row of each pair, -1 when its expert is not local
  int* pos_sh;                  // [T] packed row of each token's shared-expert row, -1 if none
  __nv_bfloat16* x_perm;        // [T * k + T, H] packed rows
  int* status;
  unsigned long long limit_ns;
};
void moe_route_fused(const MoeRouteFusedArgs& a, cudaStream_t st);
int moe_route_fused_grid(int T, int E, bool has_sg);

enum { kCombinePartial = 0, kCombineAddNorm = 1, kCombineSymm = 2, kCombineSymmNorm = 3 };
// Per token: sum_slot w * y[pos_of] + sigmoid(sg) * y[pos_sh] (+ sigmoid(shared_gate)
// * shared_y), fp32, rounded to bf16 once; then stored (partial), added to the
// residual and RMSNorm(1+w)'d (add-norm), or stored into this rank's symmetric
// slot with the completion flag published (symm), or that followed, in the same
// launch, by the NVLS sum over ranks + residual add + RMSNorm (symm-norm).
struct MoeCombineExArgs {
  const __nv_bfloat16* y;  // [rows, H] expert outputs, packed
  const float* w;          // [T, k]
  const int* pos_of;       // [T, k]
  int T, k, H;
  const int* pos_sh;       // [T] or null
  const float* sg;         // [T] shared-gate logits (with pos_sh)
  const __nv_bfloat16* shared_y;  // [T, H] separately computed shared expert, or null
  long ld_shared;
  const float* shared_gate;       // [T] its gate logits
  int mode;
  __nv_bfloat16* out;      // partial / normed output
  long ldo;
  __nv_bfloat16* resid;    // add-norm: residual stream (updated)
  long ldr;
  const float* norm_w;
  float eps;
  __nv_bfloat16* symm_base;  // symm: this rank's slot base
  CommSignal sig;
  // symm-norm: the reduction tail (multicast base of the slots, this rank's
  // flag array, mutable selector [2], status word, wait bound)
  const __nv_bfloat16* mc_base;
  const unsigned* flags;
  int* sel_rw;
  int* status;
  unsigned long long limit_ns;
};
void moe_combine_ex(const MoeCombineExArgs& a, cudaStream_t st);

}  // namespace bwn
