// Warp-level softmax + top-k of one token's router logits, shared by the
// standalone router (moe.cu) and the fused decode routing (moe_decode.cu).
#pragma once
#include "common/sm100.cuh"

namespace bwn {

// Softmax over one token's E logits, then its top-k (largest probability first,
// the lower expert id on ties, as torch.topk on the fp32 softmax in
// static_decode_35b.py:723-728).  Lane j holds experts j, 32 + j, ...; each
// lane sorts its EPL values once (bitonic network in registers), then every
// round is a warp max of the lanes' heads (redux.sync on the probability bits,
// which order like the values since they are >= 0), a min over the tied lanes'
// expert ids, and a pop of the winner's head.  Lane s gets slot s's (p, id);
// returns the sum of the k probabilities.
template <int EPL>
__device__ __forceinline__ float route_topk(const float* l, int E, int k, int lane, float& my_w, int& my_id) {
  float v[EPL];
  int id[EPL];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < E ? __ldcg(l + e) : -INFINITY;
    id[i] = e;
    mx = fmaxf(mx, v[i]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const bool real = i * 32 + lane < E;
    v[i] = real ? __expf(v[i] - mx) : -1.f;  // absent experts sort last and never win
    sum += real ? v[i] : 0.f;
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
  // bitonic sort: position i before i+1 in (value desc, id asc) order
#pragma unroll
  for (int size = 2; size <= EPL; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          const bool j_first = v[j] > v[i] || (v[j] == v[i] && id[j] < id[i]);
          const bool up = (i & size) == 0;
          if (j_first == up) {
            const float tv = v[i];
            v[i] = v[j];
            v[j] = tv;
            const int ti = id[i];
            id[i] = id[j];
            id[j] = ti;
          }
        }
      }
    }
  }
  float picked = 0.f;
  my_w = 0.f;
  my_id = -1;
  for (int sl = 0; sl < k; ++sl) {
    // key 0 = nothing left in this lane; a real probability p >= 0 has key bits(p) + 1
    const unsigned key = v[0] >= 0.f ? __float_as_uint(v[0]) + 1u : 0u;
    const unsigned m = __reduce_max_sync(0xffffffffu, key);
    const unsigned win = __reduce_min_sync(0xffffffffu, key == m ? (unsigned)id[0] : 0xffffffffu);
    const float p = __uint_as_float(m - 1u) * inv;
    picked += p;
    if (lane == sl) {
      my_w = p;
      my_id = (int)win;
    }
    if (lane == (int)(win & 31u)) {  // pop the winner's head
#pragma unroll
      for (int i = 0; i + 1 < EPL; ++i) {
        v[i] = v[i + 1];
        id[i] = id[i + 1];
      }
      v[EPL - 1] = -1.f;
      id[EPL - 1] = 0x7fffffff;
    }
  }
  return picked;
}

}  // namespace bwn
