// Warp-level softmax + top-k of one token's router logits, shared by the
// standalone router (moe.cu) and the fused decode routing (moe_decode.cu).
#pragma once
#include "common/sm100.cuh"

namespace bwn {

// Softmax over a token's E logits, then its top-k (largest probability first,
// the lower expert id on ties, as torch.topk on the fp32 softmax in
// static_decode_35b.py:723-728).  Lane j holds experts j, 32 + j, ...; each
// lane sorts its EPL values once (bitonic network in registers), then every
// round is a warp max of the lanes' heads (redux.sync on the probability bits,
// which order like the values since they are >= 0), a min over the tied lanes'
// expert ids, and a pop of the winner's head.  NT tokens (rows l[j], null =
// none) go through together: their loads share one round trip and their
// reductions interleave.  Lane s gets slot s's (p, id) of each token; picked[j]
// is the sum of token j's k probabilities.
template <int EPL, int NT>
__device__ __forceinline__ void route_topk_n(const float* const (&l)[NT], int E, int k, int lane,
                                             float (&my_w)[NT], int (&my_id)[NT], float (&picked)[NT]) {
  float v[NT][EPL];
  int id[NT][EPL];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = i * 32 + lane;
      v[j][i] = (l[j] != nullptr && e < E) ? __ldcg(l[j] + e) : -INFINITY;
      id[j][i] = e;
    }
  float inv[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i) mx = fmaxf(mx, v[j][i]);
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const bool real = i * 32 + lane < E;
      v[j][i] = real ? __expf(v[j][i] - mx) : -1.f;  // absent experts sort last and never win
      sum += real ? v[j][i] : 0.f;
    }
    inv[j] = 1.f / warp_sum(sum);
  }
  // bitonic sort: position i before i+1 in (value desc, id asc) order
#pragma unroll
  for (int size = 2; size <= EPL; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const int q = i ^ stride;
        if (q > i) {
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const bool q_first = v[j][q] > v[j][i] || (v[j][q] == v[j][i] && id[j][q] < id[j][i]);
            const bool up = (i & size) == 0;
            if (q_first == up) {
              const float tv = v[j][i];
              v[j][i] = v[j][q];
              v[j][q] = tv;
              const int ti = id[j][i];
              id[j][i] = id[j][q];
              id[j][q] = ti;
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    picked[j] = 0.f;
    my_w[j] = 0.f;
    my_id[j] = -1;
  }
  for (int sl = 0; sl < k; ++sl) {
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      // key 0 = nothing left in this lane; a real probability p >= 0 has key bits(p) + 1
      const unsigned key = v[j][0] >= 0.f ? __float_as_uint(v[j][0]) + 1u : 0u;
      const unsigned m = __reduce_max_sync(0xffffffffu, key);
      const unsigned win = __reduce_min_sync(0xffffffffu, key == m ? (unsigned)id[j][0] : 0xffffffffu);
      const float p = __uint_as_float(m - 1u) * inv[j];
      picked[j] += p;
      if (lane == sl) {
        my_w[j] = p;
        my_id[j] = (int)win;
      }
      if (lane == (int)(win & 31u)) {  // pop the winner's head
#pragma unroll
        for (int i = 0; i + 1 < EPL; ++i) {
          v[j][i] = v[j][i + 1];
          id[j][i] = id[j][i + 1];
        }
        v[j][EPL - 1] = -1.f;
        id[j][EPL - 1] = 0x7fffffff;
      }
    }
  }
}

// One token (the standalone router).
template <int EPL>
__device__ __forceinline__ float route_topk(const float* l, int E, int k, int lane, float& my_w, int& my_id) {
  const float* ls[1] = {l};
  float w[1], p[1];
  int id[1];
  route_topk_n<EPL, 1>(ls, E, k, lane, w, id, p);
  my_w = w[0];
  my_id = id[0];
  return p[0];
}

}  // namespace bwn
