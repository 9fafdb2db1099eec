// FP8 W8A16 GEMM launch descriptor (csrc/kernels/gemm_w8.cu).
#pragma once
#include "common/host.h"

namespace bwn {

struct GemmW8Problem {
  const void* A = nullptr;  // fp8 e4m3 weight [M, K] (row stride lda bytes)
  long lda = 0;
  const float* scales = nullptr;  // [ceil(M/128), lds] per 128x128 block
  int lds = 0;
  const void* B = nullptr;  // bf16 tokens [N, K]
  long ldb = 0;
  int M = 0, N = 0, K = 0;
  void* out = nullptr;      // transposed store: out[n, m]
  long ldo = 0;
  int epi = kEpiBF16;
  const __nv_bfloat16* resid = nullptr;
  long ldr = 0;
  float* workspace = nullptr;
  long workspace_floats = 0;
  int* tickets = nullptr;
  int tickets_len = 0;
  int* status = nullptr;
  CommSignal sig;
};
void gemm_w8(const GemmW8Problem& p, cudaStream_t stream);

}  // namespace bwn
