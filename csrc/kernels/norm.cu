// Row-wise normalisation and small elementwise kernels: RMSNorm with the
// Qwen3.5 (1+w) scaling (reference nki_rms_norm,
// contrib/qwen3.6-27b/kernels/rms_norm_nki.py:37-108), the fused residual add +
// RMSNorm used between sub-blocks, the (optionally vocab-sharded) embedding
// gather (static_decode_35b.py:1061-1079) and the packed argmax that makes the
// sharded greedy a single int64 max all-reduce (static_decode_35b.py:1534-1564).
#include "common/host.h"
#include "common/sm100.cuh"
#include "common/launch.cuh"
#include "kernels/launch.h"

namespace bwn {

// one CTA per row; 8-element (16-byte) vectors; the row is kept in registers
template <bool ADD, int VPT>
__global__ void __launch_bounds__(256) rms_norm_kernel(const __nv_bfloat16* __restrict__ x, long ldx,
                                                       __nv_bfloat16* __restrict__ resid, long ldr,
                                                       const float* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                                       long ldo, int cols, float eps, bool one_plus) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const int t = threadIdx.x;
  const int nvec = cols >> 3;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = t + i * blockDim.x;
    if (vi < nvec) {
      uint4 xr = reinterpret_cast<const uint4*>(x + (long)row * ldx)[vi];
      const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&xr);
      if (ADD) {
        uint4 rr = reinterpret_cast<const uint4*>(resid + (long)row * ldr)[vi];
        const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&rr);
        alignas(16) __nv_bfloat16 nr[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 a = __bfloat1622float2(xh[e]);
          const float2 b = __bfloat1622float2(rh[e]);
          nr[2 * e] = __float2bfloat16(a.x + b.x);
          nr[2 * e + 1] = __float2bfloat16(a.y + b.y);
        }
        reinterpret_cast<uint4*>(resid + (long)row * ldr)[vi] = *reinterpret_cast<uint4*>(nr);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = __bfloat162float(nr[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 a = __bfloat1622float2(xh[e]);
          v[i][2 * e] = a.x;
          v[i][2 * e + 1] = a.y;
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
    }
  }
  __shared__ float red[8];
  ss = warp_sum(ss);
  if ((t & 31) == 0) red[t >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = rsqrtf(tot / cols + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = t + i * blockDim.x;
    if (vi < nvec) {
      alignas(16) __nv_bfloat16 o[8];
      const float4 w0 = reinterpret_cast<const float4*>(w)[2 * vi];
      const float4 w1 = reinterpret_cast<const float4*>(w)[2 * vi + 1];
      const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = __float2bfloat16(v[i][e] * inv * (one_plus ? 1.f + ww[e] : ww[e]));
      reinterpret_cast<uint4*>(out + (long)row * ldo)[vi] = *reinterpret_cast<uint4*>(o);
    }
  }
}

template <bool ADD>
static void launch_norm(const __nv_bfloat16* x, long ldx, __nv_bfloat16* resid, long ldr, const float* w,
                        __nv_bfloat16* out, long ldo, int rows, int cols, float eps, bool one_plus,
                        cudaStream_t st) {
  BWN_CHECK(cols % 8 == 0 && ldx % 8 == 0 && ldo % 8 == 0 && (!ADD || ldr % 8 == 0),
            "rms_norm: columns/strides must be multiples of 8");
  const int nvec = cols / 8;
  int threads = 256;
  if (nvec <= 128) threads = ((nvec + 31) / 32) * 32;
  const int vpt = (nvec + threads - 1) / threads;
  if (rows == 0) return;
#define BWN_NORM_CASE(V)                                                                              \
  case V:                                                                                             \
    launch_k(rms_norm_kernel<ADD, V>, dim3(rows), dim3(threads), 0, st, x, ldx, resid, ldr, w, out, ldo, cols, eps, \
             one_plus);                                                                                \
    break;
  switch (vpt) {
    BWN_NORM_CASE(1)
    BWN_NORM_CASE(2)
    BWN_NORM_CASE(3)
    BWN_NORM_CASE(4)
    BWN_NORM_CASE(5)
    BWN_NORM_CASE(6)
    BWN_NORM_CASE(7)
    BWN_NORM_CASE(8)
    default: BWN_FAIL("rms_norm: row of %d columns too wide", cols);
  }
#undef BWN_NORM_CASE
  BWN_CUDA_CHECK(cudaGetLastError());
}

void rms_norm(const __nv_bfloat16* x, long ldx, const float* w, __nv_bfloat16* out, long ldo, int rows, int cols,
              float eps, bool one_plus, cudaStream_t stream) {
  launch_norm<false>(x, ldx, nullptr, 0, w, out, ldo, rows, cols, eps, one_plus, stream);
}

void add_rms_norm(const __nv_bfloat16* x, long ldx, __nv_bfloat16* residual, long ldr, const float* w,
                  __nv_bfloat16* out, long ldo, int rows, int cols, float eps, cudaStream_t stream) {
  launch_norm<true>(x, ldx, residual, ldr, w, out, ldo, rows, cols, eps, true, stream);
}

// ---------------------------------------------------------------------------
__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table, long rows,
                                 int cols, long offset, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int tok = blockIdx.x;
  const long id = (long)ids[tok] - offset;
  const bool in = id >= 0 && id < rows;
  const int nvec = cols / 8;
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    uint4 val = make_uint4(0, 0, 0, 0);
    if (in) val = reinterpret_cast<const uint4*>(table + id * cols)[v];
    reinterpret_cast<uint4*>(out + (long)tok * cols)[v] = val;
  }
}

void embedding(const int* ids, int n, const __nv_bfloat16* table, long rows, int cols, long offset,
               __nv_bfloat16* out, cudaStream_t stream) {
  BWN_CHECK(cols % 8 == 0, "embedding: hidden must be a multiple of 8");
  if (n == 0) return;
  launch_k(embedding_kernel, dim3(n), dim3(128), 0, stream, ids, table, rows, cols, offset, out);
  BWN_CUDA_CHECK(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// monotone map float -> uint32 (unsigned order = float order); -0.0 maps like
// +0.0 so equal logits of either zero sign tie and the lowest id wins
__device__ __forceinline__ uint32_t orderable(float f) {
  uint32_t u = __float_as_uint(f);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ unsigned long long pack_key(float v, long id) {
  return ((unsigned long long)orderable(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)id);
}

template <typename T>
__global__ void __launch_bounds__(1024) argmax_kernel(const T* __restrict__ logits, long ld, int cols, long id_offset,
                                                      int64_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const T* p = logits + (long)row * ld;
  unsigned long long best = 0;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const float v = to_f(p[c]);
    const unsigned long long k = pack_key(v, id_offset + c);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  __shared__ unsigned long long red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) best = red[i] > best ? red[i] : best;
    best = red[0] > best ? red[0] : best;
    // stored with the top bit flipped: a signed int64 max over shards (NCCL MAX
    // all-reduce, the fused greedy) then orders keys as the unsigned max does
    out[row] = (int64_t)(best ^ 0x8000000000000000ull);
  }
}

void argmax_packed(const float* logits, long ld, int rows, int cols, long id_offset, int64_t* out,
                   cudaStream_t stream) {
  if (rows == 0) return;
  launch_k(argmax_kernel<float>, dim3(rows), dim3(1024), 0, stream, logits, ld, cols, id_offset, out);
  BWN_CUDA_CHECK(cudaGetLastError());
}

void argmax_packed_bf16(const __nv_bfloat16* logits, long ld, int rows, int cols, long id_offset, int64_t* out,
                        cudaStream_t stream) {
  if (rows == 0) return;
  launch_k(argmax_kernel<__nv_bfloat16>, dim3(rows), dim3(1024), 0, stream, logits, ld, cols, id_offset, out);
  BWN_CUDA_CHECK(cudaGetLastError());
}

__global__ void unpack_argmax_kernel(const int64_t* packed, int rows, int* ids) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < rows) ids[i] = (int)(0xFFFFFFFFu - (uint32_t)((unsigned long long)packed[i] & 0xFFFFFFFFull));
}

void unpack_argmax(const int64_t* packed, int rows, int* ids_out, cudaStream_t stream) {
  if (rows == 0) return;
  launch_k(unpack_argmax_kernel, dim3((rows + 127) / 128), dim3(128), 0, stream, packed, rows, ids_out);
  BWN_CUDA_CHECK(cudaGetLastError());
}

}  // namespace bwn
