// Host entry points of the fused NVLink collective kernels (csrc/comm/fused_ar.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common/host.h"

namespace bwn {

void symm_put_signal(const __nv_bfloat16* x, long ldx, int rows, int cols, __nv_bfloat16* local_base,
                     const CommSignal& sig, cudaStream_t st);

struct ArNormArgs {
  const __nv_bfloat16* mc_base;  // multicast address of the two bf16 partial slots
  long buf_stride;
  int* sel;                // [2]: selector, CTA ticket
  const unsigned* flags;   // this rank's flag array (slot r written by rank r)
  int world;
  const int* epoch;
  __nv_bfloat16* resid;
  long ldr;
  const float* w;
  __nv_bfloat16* out;
  long ldo;
  int rows, cols;
  float eps;
  int* status;
  unsigned long long limit_ns;
};
void ar_add_norm(const ArNormArgs& a, cudaStream_t st);

// The all-reduce of a row-parallel partial [rows, cols] fused with DeepSeek V4's
// hyper-connection post-mix: out[t, j, :] = post[t, j] * x[t, :] +
// sum_i comb[t, i, j] * resid[t, i, :], x = the bf16-rounded sum over ranks.
// Same slots, flags and selector protocol as ar_add_norm.
struct ArHcArgs {
  const __nv_bfloat16* mc_base;
  long buf_stride;
  int* sel;
  const unsigned* flags;
  int world;
  const int* epoch;
  const __nv_bfloat16* resid;  // [rows, hc, cols]
  const float* post;           // [rows, hc]
  const float* comb;           // [rows, hc, hc]
  __nv_bfloat16* out;          // [rows, hc, cols]
  int rows, cols, hc;
  int* status;
  unsigned long long limit_ns;
};
void ar_hc_post(const ArHcArgs& a, cudaStream_t st);

// Sequence-parallel reduce-scatter + residual add + RMSNorm + all-gather of
// one shard of rows (F1 in reduce-scatter mode feeding F2).
struct SpNormArgs {
  const __nv_bfloat16* mc_partial;     // multicast base of the partial slots, or null
  const __nv_bfloat16* local_partial;  // [rows, cols] local addend when mc_partial is null
  long ldp;
  long buf_stride;
  int* sel;                  // slot selector of the partial slots
  const unsigned* flags;     // partial completion flags (this rank's array)
  const int* epoch;          // partial epoch
  int world, rank;
  __nv_bfloat16* x;          // residual shard [rows, cols] (updated)
  long ldx;
  const float* w;            // RMSNorm(1+w)
  __nv_bfloat16* h_mc;       // multicast base of the gathered normed rows [world*rows, cols]
  int rows, cols;
  float eps;
  unsigned* ag_peer_flags[8];
  int* ag_epoch;
  int* ticket;
  int* status;
  unsigned long long limit_ns;
};
void sp_norm_gather(const SpNormArgs& a, cudaStream_t st);

struct GreedyArgs {
  const int64_t* keys;     // [rows] local packed argmax keys
  int rows;
  int64_t* peer_slots[8];       // each rank's slot base ([world][rows] int64)
  unsigned* peer_flags[8];      // each rank's flag array
  const unsigned* flags;
  int world, rank;
  int* epoch;
  int* ids_out;
  int* status;
  unsigned long long limit_ns;
};
void greedy_allmax(const GreedyArgs& a, cudaStream_t st);

}  // namespace bwn
