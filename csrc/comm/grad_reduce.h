// Host entry points of the fused data-parallel gradient reduction (csrc/comm/grad_reduce.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace bwn {

constexpr int kGradFlagSlots = 8;  // per bucket: [phase 1: 8][phase 2: 8] flags

struct GradBucketArgs {
  int world, rank;
  long n;                    // bucket length (elements), multiple of 8 * world
  float* grad;               // fp32 gradients of the bucket (flat)
  __nv_bfloat16* local;      // this rank's bf16 copy in the symmetric buffer
  __nv_bfloat16* mc;         // multicast address of the same copy
  const unsigned* flags;     // this rank's 2*8 flags of the bucket
  unsigned* peer_flags[8];   // every rank's flags of the bucket
  unsigned epoch;            // step number (flags reach it when a phase is done)
  int* ticket;
  float scale;               // 1 / world
  int* status;
  unsigned long long limit_ns;
};

void grad_bucket_reduce(const GradBucketArgs& a, cudaStream_t st);  // pack + reduce-scatter/all-gather
void grad_bucket_unpack(const GradBucketArgs& a, cudaStream_t st);  // wait + bf16 -> fp32 grads

}  // namespace bwn
