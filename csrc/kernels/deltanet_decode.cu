// Gated-DeltaNet recurrent decode step (one token per sequence), fully fused:
// causal conv4 (+SiLU) over the qkv row with the 4-slot conv ring, L2 norm of
// q and k, q scale 1/sqrt(Dk), gates g = -exp(A_log)*softplus(a+dt_bias) and
// beta = sigmoid(b), the delta-rule state update and read-out, and the per-head
// RMSNormGated output.  Reference: nki_deltanet_full / _batched
// (contrib/qwen3.6-27b/kernels/deltanet_full.py:54-427,
//  contrib/qwen3.6-35b-a3b/kernels/deltanet_full_batched_v2_35b.py:66).
//
// B200 mapping.  The update is column-separable in the value dimension, so
// each (sequence, V-head) is split over a cluster of NJ=4 CTAs, each owning 32
// of the 128 state columns (16 KB of fp32 state held in registers: 128 threads,
// one column per lane, 32 rows per warp; every row access is a coalesced
// 128-byte segment).  One pass over the state yields both S^T k and S^T q:
//   kv = e^g S^T k,  d = beta (v - kv),  o = e^g S^T q + d (k.q),
//   S' = e^g S + k d^T
// The RMSNormGated sum of squares spans all 128 columns: the four CTAs
// exchange partial sums through distributed shared memory.
#include <cooperative_groups.h>

#include "common/host.h"
#include "common/sm100.cuh"
#include "common/launch.cuh"
#include "kernels/launch.h"

namespace cg = cooperative_groups;

namespace bwn {

constexpr int kDnDk = 128;
constexpr int kDnDv = 128;
constexpr int kDnNJ = 4;
constexpr int kDnCols = kDnDv / kDnNJ;  // 32

template <typename StateT>
__global__ void __cluster_dims__(kDnNJ, 1, 1) __launch_bounds__(128)
    deltanet_decode_kernel(DeltaNetDecodeArgs p) {
  pdl_trigger();
  pdl_wait();
  cg::cluster_group cluster = cg::this_cluster();
  const int jb = blockIdx.x;  // column block == rank in cluster
  const int h = blockIdx.y;   // local V head
  const int b = blockIdx.z;   // sequence
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5;
  const int rep = p.v_heads / p.k_heads;
  const int kh = h / rep;
  const int KD = p.k_heads * kDnDk;
  const int C = 2 * KD + p.v_heads * kDnDv;

  __shared__ float s_q[kDnDk], s_k[kDnDk];
  __shared__ float s_red[4][kDnCols * 2];
  __shared__ float s_scal[8];
  __shared__ float s_sumsq;

  const int pos = p.positions[b];
  const bool active = pos >= 0;
  const __nv_bfloat16* qkv = p.qkv + (long)b * p.qkv_stride;
  // the state columns go into registers first: their HBM latency overlaps the
  // conv / norm / gate prologue below
  StateT* S = reinterpret_cast<StateT*>(p.state) + (((long)b * p.v_heads + h) * kDnDk) * kDnDv + jb * kDnCols + lane;
  float st[32];
  if (active) {
#pragma unroll
    for (int i = 0; i < 32; ++i) st[i] = to_f(S[(long)(warp * 32 + i) * kDnDv]);
  }
  const int rm = p.ring_slots - 1;
  __nv_bfloat16* ring = p.conv_ring + (long)b * p.ring_slots * C;
  const int ks0 = (pos - 3) & rm, ks1 = (pos - 2) & rm, ks2 = (pos - 1) & rm, kcur = pos & rm;

  // ---- conv + SiLU for q, k (128 ch each) and this block's 32 v channels ----
  auto conv = [&](int ch) -> float {
    const float x3 = __bfloat162float(qkv[ch]);
    const float4 w = *reinterpret_cast<const float4*>(p.conv_w + (long)ch * 4);
    const float x0 = __bfloat162float(ring[ks0 * C + ch]);  // pos-3
    const float x1 = __bfloat162float(ring[ks1 * C + ch]);  // pos-2
    const float x2 = __bfloat162float(ring[ks2 * C + ch]);  // pos-1
    return silu_f(w.x * x0 + w.y * x1 + w.z * x2 + w.w * x3);
  };
  float qv = 0.f, kv = 0.f, vv = 0.f;
  if (active) {
    qv = conv(kh * kDnDk + t);
    kv = conv(KD + kh * kDnDk + t);
    if (t < kDnCols) vv = conv(2 * KD + h * kDnDv + jb * kDnCols + t);
  }
  // L2 norms (x / max(||x||, eps)) over 128 channels
  float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv), skq = warp_sum(qv * kv);
  if (lane == 0) {
    s_red[warp][0] = sq;
    s_red[warp][1] = sk;
    s_red[warp][2] = skq;
  }
  __syncthreads();
  if (t == 0) {
    float a0 = 0, a1 = 0, a2 = 0;
    for (int w = 0; w < 4; ++w) {
      a0 += s_red[w][0];
      a1 += s_red[w][1];
      a2 += s_red[w][2];
    }
    const float nq = fmaxf(sqrtf(a0), p.l2_eps), nk = fmaxf(sqrtf(a1), p.l2_eps);
    const float qs = rsqrtf((float)kDnDk);
    s_scal[0] = qs / nq;        // q multiplier
    s_scal[1] = 1.f / nk;       // k multiplier
    s_scal[2] = a2 / (nq * nk) * qs;  // k.q after normalisation and scaling
    // gates
    const float a = __bfloat162float(p.a[(long)b * p.ab_stride + h]);
    const float bb = __bfloat162float(p.b[(long)b * p.ab_stride + h]);
    const float g = -__expf(p.A_log[h]) * softplus_f(a + p.dt_bias[h]);
    s_scal[3] = __expf(g);
    s_scal[4] = sigmoid_f(bb);
  }
  __syncthreads();
  // the ring slot of this position: q/k channels written by one CTA per K head,
  // v channels by their column block (nobody reads slot pos&(R-1) in this step)
  if (active) {
    if (jb == 0 && (h % rep) == 0) {
      ring[kcur * C + kh * kDnDk + t] = qkv[kh * kDnDk + t];
      ring[kcur * C + KD + kh * kDnDk + t] = qkv[KD + kh * kDnDk + t];
    }
    if (t < kDnCols) {
      const int ch = 2 * KD + h * kDnDv + jb * kDnCols + t;
      ring[kcur * C + ch] = qkv[ch];
    }
  }
  s_q[t] = qv * s_scal[0];
  s_k[t] = kv * s_scal[1];
  __shared__ float s_v[kDnCols];
  if (t < kDnCols) s_v[t] = vv;
  __syncthreads();

  // ---- state pass: rows [32*warp, 32*warp+32), column = lane ----
  float pk = 0.f, pq = 0.f;
  if (active) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int r = warp * 32 + i;
      pk += st[i] * s_k[r];
      pq += st[i] * s_q[r];
    }
  }
  s_red[warp][lane] = pk;
  s_red[warp][kDnCols + lane] = pq;
  __syncthreads();
  const float eg = s_scal[3], beta = s_scal[4], kq = s_scal[2];
  float delta = 0.f, o = 0.f;
  if (warp == 0) {
    float tk = 0.f, tq = 0.f;
    for (int w = 0; w < 4; ++w) {
      tk += s_red[w][lane];
      tq += s_red[w][kDnCols + lane];
    }
    delta = beta * (s_v[lane] - eg * tk);
    o = eg * tq + delta * kq;
    s_red[0][lane] = delta;  // broadcast (row 0 of s_red reused after the read above)
    const float ss = warp_sum(o * o);
    if (lane == 0) s_sumsq = ss;
  }
  __syncthreads();
  delta = s_red[0][lane];
  if (active) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int r = warp * 32 + i;
      S[(long)r * kDnDv] = from_f<StateT>(eg * st[i] + s_k[r] * delta);
    }
  }
  // ---- RMSNormGated across the cluster's 4 column blocks ----
  cluster.sync();
  if (warp == 0) {
    float tot = 0.f;
    for (int r = 0; r < kDnNJ; ++r) tot += *cluster.map_shared_rank(&s_sumsq, r);
    const float inv = rsqrtf(tot / (float)kDnDv + p.norm_eps);
    const int col = h * kDnDv + jb * kDnCols + lane;
    const float z = __bfloat162float(p.z[(long)b * p.z_stride + col]);
    const float y = active ? o * inv * p.norm_w[jb * kDnCols + lane] * silu_f(z) : 0.f;
    p.out[(long)b * p.out_stride + col] = __float2bfloat16(y);
  }
  cluster.sync();  // keep shared memory alive until every peer has read it
}

void deltanet_decode(const DeltaNetDecodeArgs& p, cudaStream_t stream) {
  dim3 grid(kDnNJ, p.v_heads, p.batch);
  if (p.state_bf16) {
    launch_k(deltanet_decode_kernel<__nv_bfloat16>, grid, dim3(128), 0, stream, p);
  } else {
    launch_k(deltanet_decode_kernel<float>, grid, dim3(128), 0, stream, p);
  }
}

}  // namespace bwn
