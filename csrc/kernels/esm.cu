// ESM-2 attention glue on the GPU: rotary embedding (rotate-half form, HF
// esm.modeling_esm.RotaryEmbedding / apply_rotary_pos_emb; the reference fine-
// tunes that module, contrib/esm2/train_esm.py:250-370) fused with the q
// scaling and the [B, S, H, D] <-> [B, H, S, D] transpose around attention.
//
// Forward:  out[b, h, s, :] = scale * rot(x[b, s, h, :], s)
// Backward: out[b, s, h, :] = scale * rot^T(g[b, h, s, :], s)   (rot^T = rotation by -angle)
// with rot(x)[d] = x[d] cos - x[d + D/2] sin, rot(x)[d + D/2] = x[d + D/2] cos + x[d] sin
// for d < D/2 and angle(s, d) = s * inv_freq[d] (tables cos/sin [S, D/2], fp32).
// One thread per pair (d, d + D/2), two pairs per thread as bf16x2.
#include <cuda_bf16.h>

#include "common/host.h"
#include "common/launch.cuh"
#include "common/sm100.cuh"
#include "kernels/launch.h"

namespace bwn {

__global__ void __launch_bounds__(256) rope_half_kernel(RopeHalfArgs a) {
  pdl_trigger();
  pdl_wait();
  const int half = a.D >> 1, hp = half >> 1;  // bf16x2 pairs per half
  const long total = (long)a.B * a.S * a.H * hp;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int dp = (int)(i % hp);
    long r = i / hp;
    const int h = (int)(r % a.H);
    r /= a.H;
    const int s = (int)(r % a.S);
    const int b = (int)(r / a.S);
    const int d = dp * 2;
    const __nv_bfloat16* src = a.in + (long)b * a.in_b + (long)s * a.in_s + (long)h * a.in_h;
    __nv_bfloat16* dst = a.out + (long)b * a.out_b + (long)s * a.out_s + (long)h * a.out_h;
    const float2 x1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + d));
    const float2 x2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + half + d));
    const float2 c = *reinterpret_cast<const float2*>(a.cos + (long)s * half + d);
    const float2 sn = *reinterpret_cast<const float2*>(a.sin + (long)s * half + d);
    const float sx = a.sign * sn.x, sy = a.sign * sn.y;
    const float2 o1 = make_float2((x1.x * c.x - x2.x * sx) * a.scale, (x1.y * c.y - x2.y * sy) * a.scale);
    const float2 o2 = make_float2((x2.x * c.x + x1.x * sx) * a.scale, (x2.y * c.y + x1.y * sy) * a.scale);
    *reinterpret_cast<__nv_bfloat162*>(dst + d) = __float22bfloat162_rn(o1);
    *reinterpret_cast<__nv_bfloat162*>(dst + half + d) = __float22bfloat162_rn(o2);
  }
}

void rope_half(const RopeHalfArgs& a, cudaStream_t st) {
  BWN_CHECK(a.D % 4 == 0, "rope_half: head dim multiple of 4");
  const long total = (long)a.B * a.S * a.H * (a.D / 4);
  if (total == 0) return;
  const int grid = (int)std::min<long>((total + 255) / 256, (long)num_sms() * 16);
  launch_k(rope_half_kernel, dim3(grid), dim3(256), 0, st, a);
}

}  // namespace bwn
