// Shared epilogue of the tcgen05 GEMM kernels (gemm_tc.cu, gemm_w8.cu): the
// argument block and the per-thread store of one 32-column accumulator chunk
// (bf16, bf16 + residual, SwiGLU over 16-interleaved gate/up, fp32, or the
// bf16 partial into a symmetric slot), in normal or transposed (swap-AB)
// orientation.
#pragma once
#include "common/host.h"
#include "common/sm100.cuh"

namespace bwn {

struct GemmArgs {
  int M, N, K;
  int tiles_m, tiles_n, splits, kb_per_split, num_kb;
  void* out;
  long ldo;
  const __nv_bfloat16* resid;  // optional, same indexing as out (bf16 modes)
  long ldr;
  float* workspace;            // splits>1: [tiles * splits * BM * BN] fp32
  int* tickets;                // splits>1: [tiles]
  int* status;
  CommSignal sig;              // kEpiSymm / kEpiSymmNorm: completion signal to peers
  AgWait ag;                   // A rows all-gathered by peers: wait per owner
  ArTail tail;                 // kEpiSymmNorm: reduction + residual + RMSNorm after the signal
};

// Row tile of a work tile; with an all-gathered A this rank's own rows come first.
__device__ __forceinline__ int gemm_tile_m(const GemmArgs& a, int tile, int bm) {
  int tm = tile % a.tiles_m;
  if (a.ag.flags) tm = (tm + a.ag.rank * (a.ag.rows / bm)) % a.tiles_m;
  return tm;
}

template <int BN, int EPI, bool TRANS>
__device__ __forceinline__ void epi_store_chunk(const GemmArgs& a, const float (&v)[32], int ncols, int m, int n0) {
  // m: global row (A row), n0: global column of v[0]; ncols valid in v (16 or 32)
  if (EPI == kEpiSymm || EPI == kEpiSymmNorm) {
    // out is this rank's bf16 [tokens, ldo] symmetric buffer pair; the slot in
    // use alternates under the device-side selector.  Peers read it through the
    // multicast address once the completion flag is published.
    GemmArgs b = a;
    b.out = reinterpret_cast<__nv_bfloat16*>(a.out) + (long)((*a.sig.sel) & 1) * a.sig.buf_stride;
    epi_store_chunk<BN, kEpiBF16, TRANS>(b, v, ncols, m, n0);
    return;
  }
  if (EPI == kEpiF32) {
    float* out = reinterpret_cast<float*>(a.out);
    if (!TRANS) {
      if (m >= a.M) return;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols && n0 + j < a.N) out[(long)m * a.ldo + n0 + j] = v[j];
    } else {
      if (m >= a.M) return;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols && n0 + j < a.N) out[(long)(n0 + j) * a.ldo + m] = v[j];
    }
    return;
  }
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
  if (EPI == kEpiSwiGLU) {
    if (!TRANS) {
      // columns [n0, n0+32) = 16 gate then 16 up features of output block n0/32
      if (m >= a.M) return;
      const int f0 = (n0 >> 5) * 16;
      if (n0 + 32 > a.N) return;
      alignas(16) __nv_bfloat16 o[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = __float2bfloat16(silu_f(v[j]) * v[j + 16]);
      uint4* dst = reinterpret_cast<uint4*>(out + (long)m * a.ldo + f0);
      dst[0] = reinterpret_cast<uint4*>(o)[0];
      dst[1] = reinterpret_cast<uint4*>(o)[1];
    } else {
      // rows: lanes 0-15 gate, 16-31 up (m block of 32 aligned)
      const int lane = threadIdx.x & 31;
      const int f = (m >> 5) * 16 + (lane & 15);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float up = __shfl_down_sync(0xffffffffu, v[j], 16);
        if (lane < 16 && j < ncols && n0 + j < a.N && m < a.M)
          out[(long)(n0 + j) * a.ldo + f] = __float2bfloat16(silu_f(v[j]) * up);
      }
    }
    return;
  }
  // bf16 store (optionally + residual)
  if (!TRANS) {
    if (m >= a.M) return;
    const bool full = (n0 + 32 <= a.N) && ncols == 32 && ((a.ldo & 7) == 0);
    if (full) {
      alignas(16) __nv_bfloat16 o[32];
      if (EPI == kEpiResid) {
        const uint4* rs = reinterpret_cast<const uint4*>(a.resid + (long)m * a.ldr + n0);
        alignas(16) __nv_bfloat16 r[32];
#pragma unroll
        for (int q = 0; q < 4; ++q) reinterpret_cast<uint4*>(r)[q] = rs[q];
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = __float2bfloat16(v[j] + __bfloat162float(r[j]));
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = __float2bfloat16(v[j]);
      }
      uint4* dst = reinterpret_cast<uint4*>(out + (long)m * a.ldo + n0);
#pragma unroll
      for (int q = 0; q < 4; ++q) dst[q] = reinterpret_cast<uint4*>(o)[q];
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < ncols && n0 + j < a.N) {
          float x = v[j];
          if (EPI == kEpiResid) x += __bfloat162float(a.resid[(long)m * a.ldr + n0 + j]);
          out[(long)m * a.ldo + n0 + j] = __float2bfloat16(x);
        }
      }
    }
  } else {
    if (m >= a.M) return;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < ncols && n0 + j < a.N) {
        float x = v[j];
        if (EPI == kEpiResid) x += __bfloat162float(a.resid[(long)(n0 + j) * a.ldr + m]);
        out[(long)(n0 + j) * a.ldo + m] = __float2bfloat16(x);
      }
    }
  }
}


}  // namespace bwn
