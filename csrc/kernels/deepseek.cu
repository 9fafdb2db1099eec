// DeepSeek V4 Flash device kernels.
//
//  * hc_pre      Hyper-Connection pre-mix, one CTA per token
//                (contrib/deepseek-v4-flash/run_deepseek_v4_tp.py:179-256);
//                for many tokens (prefill) the mix GEMV of every token is one
//                tensor-core GEMM run before it (mix_in) and the kernel does
//                the rest:
//                rms over the hc*dim flattened streams, the (2+hc)*hc mix GEMV,
//                sigmoid pre/post gates (+eps), the hc x hc Sinkhorn
//                normalisation of exp(comb) (20 alternating row/column passes),
//                and the pre-weighted stream sum -- all in one launch.  With
//                mix_out == hc it is the head variant (hc_head, :230-243).
//  * hc_post     out[j] = post[j] * x + sum_i comb[i][j] * residual[i]   (:221-227)
//  * mqa_attn    attention with ONE shared K/V head per token (the reference
//                uses kv as both key and value, :315-336), causal over a
//                per-query visible length.  Split over keys with an online
//                softmax and a last-CTA merge; q is expected already
//                normalised, roped and scaled.
#include "common/host.h"
#include "common/sm100.cuh"
#include "kernels/deepseek.h"

namespace bwn {

// ----------------------------------------------------------------------------
// hyper-connections
// ----------------------------------------------------------------------------
template <int HC>
__global__ void __launch_bounds__(256) hc_pre_kernel(HcPreArgs a) {
  constexpr int MIXMAX = (2 + HC) * HC;
  const int t = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long n = (long)HC * a.dim;
  const __nv_bfloat16* x = a.x + (long)t * n;
  __shared__ float s_red[8][MIXMAX + 1];
  __shared__ float s_mix[MIXMAX];
  float acc[MIXMAX];
#pragma unroll
  for (int j = 0; j < MIXMAX; ++j) acc[j] = 0.f;
  float ss = 0.f;
  if (a.mix_in) {  // mixes precomputed: only the sum of squares (16-byte loads)
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    for (long c = tid; c < n / 8; c += blockDim.x) {
      const uint4 u = xv[c];
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h2[e]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
  } else {
    for (long c = tid; c < n; c += blockDim.x) {
      const float v = __bfloat162float(x[c]);
      ss += v * v;
#pragma unroll
      for (int j = 0; j < MIXMAX; ++j)
        if (j < a.mix_out) acc[j] += v * a.fn[(long)j * n + c];
    }
  }
  ss = warp_sum(ss);
#pragma unroll
  for (int j = 0; j < MIXMAX; ++j) acc[j] = warp_sum(acc[j]);
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < MIXMAX; ++j) s_red[warp][j] = acc[j];
    s_red[warp][MIXMAX] = ss;
  }
  __syncthreads();
  if (tid == 0) {
    float tot = 0.f;
    for (int w = 0; w < 8; ++w) tot += s_red[w][MIXMAX];
    const float rs = rsqrtf(tot / (float)n + a.norm_eps);
    for (int j = 0; j < a.mix_out; ++j) {
      float m = 0.f;
      if (a.mix_in) {
        m = a.mix_in[(long)t * a.ld_mix + j];
      } else {
        for (int w = 0; w < 8; ++w) m += s_red[w][j];
      }
      s_mix[j] = m * rs;
    }
    if (a.mix_out == HC) {  // head: pre only, one scale
      for (int i = 0; i < HC; ++i) s_mix[i] = sigmoid_f(s_mix[i] * a.scale[0] + a.base[i]) + a.eps;
    } else {
      for (int i = 0; i < HC; ++i) {
        s_mix[i] = sigmoid_f(s_mix[i] * a.scale[0] + a.base[i]) + a.eps;
        s_mix[HC + i] = sigmoid_f(s_mix[HC + i] * a.scale[1] + a.base[HC + i]) + a.eps;
      }
      float m[HC][HC];
      for (int i = 0; i < HC; ++i)
        for (int j = 0; j < HC; ++j) m[i][j] = __expf(s_mix[2 * HC + i * HC + j] * a.scale[2] + a.base[2 * HC + i * HC + j]);
      for (int it = 0; it < a.sinkhorn_iters; ++it) {
        for (int i = 0; i < HC; ++i) {
          float r = 0.f;
          for (int j = 0; j < HC; ++j) r += m[i][j];
          for (int j = 0; j < HC; ++j) m[i][j] /= (r + a.eps);
        }
        for (int j = 0; j < HC; ++j) {
          float c = 0.f;
          for (int i = 0; i < HC; ++i) c += m[i][j];
          for (int i = 0; i < HC; ++i) m[i][j] /= (c + a.eps);
        }
      }
      for (int i = 0; i < HC; ++i) {
        a.post[(long)t * HC + i] = s_mix[HC + i];
        for (int j = 0; j < HC; ++j) a.comb[((long)t * HC + i) * HC + j] = m[i][j];
      }
    }
  }
  __syncthreads();
  // y = sum_i pre_i * x_i
  for (int c = tid; c < a.dim; c += blockDim.x) {
    float y = 0.f;
#pragma unroll
    for (int i = 0; i < HC; ++i) y += s_mix[i] * __bfloat162float(x[(long)i * a.dim + c]);
    a.y[(long)t * a.dim + c] = __float2bfloat16(y);
  }
}

template <int HC>
__global__ void __launch_bounds__(256) hc_post_kernel(const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* __restrict__ resid,
                                                      const float* __restrict__ post, const float* __restrict__ comb,
                                                      int dim, __nv_bfloat16* __restrict__ out) {
  const int t = blockIdx.x;
  __shared__ float s_post[HC], s_comb[HC * HC];
  if (threadIdx.x < HC) s_post[threadIdx.x] = post[(long)t * HC + threadIdx.x];
  if (threadIdx.x < HC * HC) s_comb[threadIdx.x] = comb[(long)t * HC * HC + threadIdx.x];
  __syncthreads();
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    const float xv = __bfloat162float(x[(long)t * dim + c]);
    float r[HC];
#pragma unroll
    for (int i = 0; i < HC; ++i) r[i] = __bfloat162float(resid[((long)t * HC + i) * dim + c]);
#pragma unroll
    for (int j = 0; j < HC; ++j) {
      float o = s_post[j] * xv;
#pragma unroll
      for (int i = 0; i < HC; ++i) o += s_comb[i * HC + j] * r[i];
      out[((long)t * HC + j) * dim + c] = __float2bfloat16(o);
    }
  }
}

void hc_pre(const HcPreArgs& a, cudaStream_t st) {
  BWN_CHECK(a.hc == 4, "hc_pre: hc_mult 4 supported");
  BWN_CHECK(a.mix_out == a.hc || a.mix_out == (2 + a.hc) * a.hc, "hc_pre: mix_out");
  if (a.tokens == 0) return;
  hc_pre_kernel<4><<<a.tokens, 256, 0, st>>>(a);
  BWN_CUDA_CHECK(cudaGetLastError());
}

void hc_post(const __nv_bfloat16* x, const __nv_bfloat16* resid, const float* post, const float* comb, int tokens,
             int hc, int dim, __nv_bfloat16* out, cudaStream_t st) {
  BWN_CHECK(hc == 4, "hc_post: hc_mult 4 supported");
  if (tokens == 0) return;
  hc_post_kernel<4><<<tokens, 256, 0, st>>>(x, resid, post, comb, dim, out);
  BWN_CUDA_CHECK(cudaGetLastError());
}

// ----------------------------------------------------------------------------
// single-KV-head attention (CUDA cores).  grid (splits, rows); a "row" is one
// query token with all its local heads.  kv [B, T, D] with D = 32 * DPL.
// ----------------------------------------------------------------------------
template <int DPL, int HMAX>
__global__ void __launch_bounds__(256) mqa_attn_kernel(MqaArgs a) {
  constexpr int D = 32 * DPL;
  const int sp = blockIdx.x, row = blockIdx.y;
  const int b = row / a.q_per_seq;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = a.visible[row];  // keys [0, L)
  int chunk = (L + a.splits - 1) / a.splits;
  const int k0 = sp * chunk, k1 = min(L, k0 + chunk);
  const __nv_bfloat16* kv = a.kv + (long)b * a.kv_seq_stride;
  const __nv_bfloat16* q = a.q + (long)row * a.H * D;
  // each warp owns heads warp, warp+8, ...; lane holds DPL dims of q and acc
  float qr[HMAX / 8][DPL], acc[HMAX / 8][DPL], m[HMAX / 8], l[HMAX / 8];
#pragma unroll
  for (int hh = 0; hh < HMAX / 8; ++hh) {
    const int h = warp + hh * 8;
    m[hh] = -INFINITY;
    l[hh] = 0.f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
      qr[hh][e] = h < a.H ? __bfloat162float(q[(long)h * D + lane * DPL + e]) : 0.f;
      acc[hh][e] = 0.f;
    }
  }
  // KU key rows are loaded together (their loads share one round trip), then
  // folded in one at a time; KU = 1 where the per-head registers leave no room
  constexpr int KU = HMAX <= 16 ? 4 : 1;
  for (int kb = k0; kb < k1; kb += KU) {
    float kvv[KU][DPL];
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int k = min(kb + u, k1 - 1);
      const __nv_bfloat16* src = kv + (long)k * D + lane * DPL;
      if constexpr (DPL % 8 == 0) {
#pragma unroll
        for (int e = 0; e < DPL; e += 8) {
          const uint4 w = *reinterpret_cast<const uint4*>(src + e);
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = __bfloat1622float2(h2[q]);
            kvv[u][e + 2 * q] = f.x;
            kvv[u][e + 2 * q + 1] = f.y;
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < DPL; ++e) kvv[u][e] = __bfloat162float(src[e]);
      }
    }
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      if (kb + u >= k1) break;
#pragma unroll
      for (int hh = 0; hh < HMAX / 8; ++hh) {
        if (warp + hh * 8 >= a.H) continue;
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) s += qr[hh][e] * kvv[u][e];
        s = warp_sum(s) * a.scale;
        const float mn = fmaxf(m[hh], s);
        const float al = __expf(m[hh] - mn), p = __expf(s - mn);
        l[hh] = l[hh] * al + p;
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[hh][e] = acc[hh][e] * al + p * kvv[u][e];
        m[hh] = mn;
      }
    }
  }
  // partials: [rows, splits, H, 2 + D]
  const int W = 2 + D;
#pragma unroll
  for (int hh = 0; hh < HMAX / 8; ++hh) {
    const int h = warp + hh * 8;
    if (h >= a.H) continue;
    float* ws = a.workspace + (((long)row * a.splits + sp) * a.H + h) * W;
    if (lane == 0) {
      ws[0] = m[hh];
      ws[1] = l[hh];
    }
#pragma unroll
    for (int e = 0; e < DPL; ++e) ws[2 + lane * DPL + e] = acc[hh][e];
  }
  __threadfence();
  __syncthreads();
  __shared__ int s_t;
  if (threadIdx.x == 0) s_t = atomicAdd(&a.tickets[row], 1);
  __syncthreads();
  if (s_t != a.splits - 1) return;
  __threadfence();
  for (int h = warp; h < a.H; h += 8) {
    float M = -INFINITY;
    for (int s = 0; s < a.splits; ++s) M = fmaxf(M, __ldcg(a.workspace + (((long)row * a.splits + s) * a.H + h) * W));
    float Ls = 0.f;
    float o[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) o[e] = 0.f;
    for (int s = 0; s < a.splits; ++s) {
      const float* e0 = a.workspace + (((long)row * a.splits + s) * a.H + h) * W;
      const float mm = __ldcg(e0);
      if (mm == -INFINITY) continue;
      const float w = __expf(mm - M);
      Ls += __ldcg(e0 + 1) * w;
#pragma unroll
      for (int e = 0; e < DPL; ++e) o[e] += __ldcg(e0 + 2 + lane * DPL + e) * w;
    }
    const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) a.out[((long)row * a.H + h) * D + lane * DPL + e] = __float2bfloat16(o[e] * inv);
  }
  if (threadIdx.x == 0) a.tickets[row] = 0;
}

void mqa_attn(const MqaArgs& a, cudaStream_t st) {
  BWN_CHECK(a.H <= 64, "mqa_attn: at most 64 local heads");
  if (a.rows == 0) return;
  dim3 grid(a.splits, a.rows);
#define BWN_MQA(DPL_, HM)                                         \
  mqa_attn_kernel<DPL_, HM><<<grid, 256, 0, st>>>(a);             \
  BWN_CUDA_CHECK(cudaGetLastError());                             \
  return;
  if (a.D == 512) {
    if (a.H <= 8) { BWN_MQA(16, 8) }
    if (a.H <= 16) { BWN_MQA(16, 16) }
    BWN_MQA(16, 64)
  } else if (a.D == 256) {
    if (a.H <= 8) { BWN_MQA(8, 8) }
    if (a.H <= 16) { BWN_MQA(8, 16) }
    BWN_MQA(8, 64)
  } else if (a.D == 128) {
    if (a.H <= 8) { BWN_MQA(4, 8) }
    BWN_MQA(4, 64)
  } else if (a.D == 64) {
    if (a.H <= 8) { BWN_MQA(2, 8) }
    BWN_MQA(2, 64)
  }
#undef BWN_MQA
  BWN_FAIL("mqa_attn: head_dim %d not supported", a.D);
}

}  // namespace bwn

namespace bwn {
// In-place RoPE on the trailing 2*half dims of x [rows, H, D] with interleaved
// (even, odd) pairs at each row's position (run_deepseek_v4_tp.py:147-160).
__global__ void rope_interleaved_kernel(__nv_bfloat16* x, int rows, int H, int D, int half, const float* cos,
                                        const float* sin, const int* pos) {
  const int r = blockIdx.x;
  const int p = pos[r];
  for (int i = threadIdx.x; i < H * half; i += blockDim.x) {
    const int h = i / half, j = i % half;
    __nv_bfloat16* e = x + ((long)r * H + h) * D + (D - 2 * half) + 2 * j;
    const float a = __bfloat162float(e[0]), b = __bfloat162float(e[1]);
    const float c = cos[(long)p * half + j], s = sin[(long)p * half + j];
    e[0] = __float2bfloat16(a * c - b * s);
    e[1] = __float2bfloat16(b * c + a * s);
  }
}

void rope_interleaved(__nv_bfloat16* x, int rows, int H, int D, int half, const float* cos, const float* sin,
                      const int* pos, cudaStream_t st) {
  if (rows == 0) return;
  rope_interleaved_kernel<<<rows, 128, 0, st>>>(x, rows, H, D, half, cos, sin, pos);
  BWN_CUDA_CHECK(cudaGetLastError());
}
}  // namespace bwn
