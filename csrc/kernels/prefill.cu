// Prompt (prefill) kernels for the Qwen3.6 hybrid:
//
//  * gqa_prefill_prep   q/k RMSNorm(1+w) + partial RoPE at the runtime offset,
//                       q written head-major for TMA, K/V rows written into the
//                       cache (the reference's rope_kv_dynamic,
//                       contrib/qwen3.6-35b-a3b/kernels/gqa_rope_kv_35b.py:90-110).
//  * flash_prefill      prefix-aware causal attention on tcgen05 (reference:
//                       gqa_flash_prefill_35b.py:53-210 and the nkilib
//                       attention_cte call, static_decode_35b.py:2412-2419):
//                       S = Q K^T into TMEM (double-buffered), softmax with one
//                       thread per query row, P to shared memory (SW128),
//                       O += P V with V as an MN-major operand, O rescaled in
//                       TMEM only when a row max grows, sigmoid gate fused.
//  * dn_prefill_prep    causal depthwise conv (history from the conv ring) +
//                       SiLU, L2 norm of q/k (+1/sqrt(Dk) on q), gates; pad rows
//                       get g = beta = 0 (static_decode_35b.py:2172-2192).
//  * dn_ring_update     last 3 valid rows of the chunk into the conv ring.
//  * dn_chunk           chunked gated delta rule (reference
//                       nki_deltanet_chunked_prefill_v2, kernels/deltanet_chunked_v2.py),
//                       one CTA per (sequence, V head), chunks of 64 sequential,
//                       state carried in shared memory, (I - A)^-1 by forward
//                       substitution (stable, unlike full-width doubling at C >= 32),
//                       RMSNormGated output fused.
#include <cstdlib>

#include "common/host.h"
#include "common/sm100.cuh"
#include "kernels/prefill.h"

namespace bwn {

// =============================================================================
// GQA prep
// =============================================================================
__global__ void __launch_bounds__(256) gqa_prefill_prep_kernel(GqaPrefillArgs p) {
  const int t = blockIdx.x;  // row within the (padded) chunk
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = 256;
  const int pos = prefill_start(p) + t;
  if (t < p.S && pos >= p.s_max) {  // the chunk runs past the cache: nothing of this row is written
    if (threadIdx.x == 0) set_status(p.status, kStatusBounds);
    return;
  }
  const bool real = t < p.S;
  const int R = p.rope_dim, hr = R / 2;
  float c[8], s[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int d = lane * 8 + e;
    c[e] = (real && d < R) ? p.cos[(long)pos * R + d] : 1.f;
    s[e] = (real && d < R) ? p.sin[(long)pos * R + d] : 0.f;
  }
  auto norm_rope = [&](const __nv_bfloat16* src, const float* w, float (&y)[8]) {
    uint4 raw = *reinterpret_cast<const uint4*>(src + lane * 8);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float x[8];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h2[e]);
      x[2 * e] = f.x;
      x[2 * e + 1] = f.y;
      ss += f.x * f.x + f.y * f.y;
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / D + p.eps);
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = x[e] * inv * (1.f + w[lane * 8 + e]);
    // rotate-half partner of dim d (< R) is d +- R/2: lane +- R/16 for 8 dims per lane
    const int dl = hr / 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float up = __shfl_down_sync(0xffffffffu, x[e], dl);
      const float dn = __shfl_up_sync(0xffffffffu, x[e], dl);
      const int d = lane * 8 + e;
      float rot = 0.f;
      if (d < hr) rot = -up;
      else if (d < R) rot = dn;
      y[e] = d < R ? x[e] * c[e] + rot * s[e] : x[e];
    }
  };
  auto store8 = [&](__nv_bfloat16* dst, const float (&y)[8]) {
    alignas(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __float2bfloat16(y[e]);
    *reinterpret_cast<uint4*>(dst + lane * 8) = *reinterpret_cast<uint4*>(o);
  };
  for (int h = warp; h < p.q_heads; h += 8) {
    __nv_bfloat16* dst = p.q_rot + (((long)b * p.q_heads + h) * p.S_pad + t) * D;
    if (!real) {
      *reinterpret_cast<uint4*>(dst + lane * 8) = make_uint4(0, 0, 0, 0);
      continue;
    }
    float y[8];
    norm_rope(p.qg + ((long)b * p.S + t) * p.qg_row + (long)h * 2 * D, p.q_norm_w, y);
    store8(dst, y);
  }
  if (!real) return;
  for (int h = warp; h < p.kv_heads; h += 8) {
    float y[8];
    norm_rope(p.k + ((long)b * p.S + t) * p.kv_row + (long)h * D, p.k_norm_w, y);
    const long crow = ((long)b * p.kv_heads + h) * p.s_max + pos;
    store8(p.k_cache + crow * D, y);
    *reinterpret_cast<uint4*>(p.v_cache + crow * D + lane * 8) =
        *reinterpret_cast<const uint4*>(p.v + ((long)b * p.S + t) * p.kv_row + (long)h * D + lane * 8);
  }
}

// =============================================================================
// flash attention prefill (tcgen05)
// =============================================================================
constexpr int kFaM = 128;          // query rows per CTA
constexpr int kFaN = 128;          // keys per tile
constexpr int kFaBox = 128 * 128;  // one [128 rows x 64 dims] SW128 box (16 KB)
constexpr int kFaThreads = 192;
constexpr int kFaSmem = 1024 + 4 * kFaBox /*Q*/ + 4 * kFaBox /*K*/ + 4 * kFaBox /*V*/ + 2 * kFaBox /*P*/ + 256;

__global__ void __launch_bounds__(kFaThreads, 1)
    flash_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, GqaPrefillArgs p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = sm;
  uint8_t* sK = sQ + 4 * kFaBox;
  uint8_t* sV = sK + 4 * kFaBox;
  uint8_t* sP = sV + 4 * kFaBox;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kFaBox);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 2;
  uint64_t* v_full = bars + 3;
  uint64_t* v_empty = bars + 4;
  uint64_t* s_full = bars + 5;   // [2]
  uint64_t* s_empty = bars + 7;  // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* o_ready = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = warp_id(), lane = lane_id();
  const int G = p.q_heads / p.kv_heads;
  const int kvh = h / G;
  const int q0 = qt * kFaM;
  const int kv_end = min(prefill_start(p) + min(q0 + kFaM, p.S), p.s_max);
  const int ntiles = (kv_end + kFaN - 1) / kFaN;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 12; ++i) mbar_init(&bars[i], (i == 7 || i == 8 || i == 9) ? 128 : 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S0 @0, S1 @128, O @256

  if (warp == 0) {
    if (elect_one()) {
      const int qrow = (int)(((long)b * p.q_heads + h) * p.S_pad + q0);
      mbar_arrive_expect_tx(q_full, 4 * kFaBox);
      for (int bx = 0; bx < 4; ++bx) tma_load_2d(&tmQ, q_full, sQ + bx * kFaBox, bx * 64, qrow);
      const int krow0 = (int)(((long)b * p.kv_heads + kvh) * p.s_max);
      for (int j = 0; j < ntiles && !*abort_flag; ++j) {
        if (!mbar_wait(k_empty, (j & 1) ^ 1)) {
          set_status(p.status, kStatusMbarTimeout);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(k_full, 4 * kFaBox);
        for (int bx = 0; bx < 4; ++bx) tma_load_2d(&tmK, k_full, sK + bx * kFaBox, bx * 64, krow0 + j * kFaN);
        if (!mbar_wait(v_empty, (j & 1) ^ 1)) {
          set_status(p.status, kStatusMbarTimeout);
          *abort_flag = 1;
          mbar_wait(k_full, j & 1, 100000000ull);
          break;
        }
        mbar_arrive_expect_tx(v_full, 4 * kFaBox);
        for (int bx = 0; bx < 4; ++bx) tma_load_2d(&tmV, v_full, sV + bx * kFaBox, bx * 64, krow0 + j * kFaN);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t id_qk = idesc_bf16_f32_major(kFaM, kFaN, false, false);
      const uint32_t id_pv = idesc_bf16_f32_major(kFaM, 256, false, true);
      bool ok = mbar_wait(q_full, 0);
      auto issue_qk = [&](int j) -> bool {
        if (!mbar_wait(k_full, j & 1)) return false;
        if (!mbar_wait(&s_empty[j & 1], ((j >> 1) & 1) ^ 1)) return false;
        tc_fence_after();
        const uint32_t d = tmem + (j & 1) * kFaN;
        for (int bx = 0; bx < 4; ++bx) {
          const uint64_t da = smem_desc_sw128(smem_u32(sQ + bx * kFaBox));
          const uint64_t db = smem_desc_sw128(smem_u32(sK + bx * kFaBox));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_f16(d, da + 2 * kk, db + 2 * kk, id_qk, (bx | kk) ? 1u : 0u);
        }
        umma_commit(&s_full[j & 1]);
        umma_commit(k_empty);
        return true;
      };
      if (ok && ntiles > 0) ok = issue_qk(0);
      for (int j = 0; ok && j < ntiles; ++j) {
        if (j + 1 < ntiles && !issue_qk(j + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(v_full, j & 1) || !mbar_wait(p_full, j & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < 2; ++kb) {
          const uint64_t da = smem_desc_sw128(smem_u32(sP + kb * kFaBox));
          const uint64_t db = smem_desc_sw128_mn(smem_u32(sV + kb * 8192), kFaBox);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem + 256, da + 2 * kk, db + 128 * kk, id_pv, (j | kb | kk) ? 1u : 0u);
        }
        umma_commit(o_ready);
        umma_commit(v_empty);
      }
      if (!ok) {
        set_status(p.status, kStatusMbarTimeout);
        *abort_flag = 1;
      }
    }
  } else {
    // ------------------------------ softmax warps ----------------------------
    const int q = warp & 3;
    const int r = q * 32 + lane;  // query row in tile == TMEM lane
    const int qpos = prefill_start(p) + q0 + r;
    const bool row_real = (q0 + r) < p.S;
    const float sl2 = p.scale * 1.4426950408889634f;  // scale * log2(e)
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kFaN];
#pragma unroll
      for (int c = 0; c < kFaN; c += 32) {
        float v[32];
        tmem_ld32(tmem + lane_base + (j & 1) * kFaN + c, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) s[c + e] = v[e];
      }
      tc_fence_before();
      mbar_arrive(&s_empty[j & 1]);
      const int kbase = j * kFaN;
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < kFaN; ++c) {
        const bool vis = row_real && (kbase + c) <= qpos;
        s[c] = vis ? s[c] * sl2 : -INFINITY;
        mt = fmaxf(mt, s[c]);
      }
      const float mn = fmaxf(m, mt);
      const float alpha = (m == -INFINITY) ? 0.f : exp2f(m - mn);
      if (j > 0) {
        // O and the P buffer are free once PV(j-1) has retired
        if (!mbar_wait(o_ready, (j - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, mn > m)) {
#pragma unroll 1
          for (int c = 0; c < 256; c += 32) {
            float v[32];
            tmem_ld32(tmem + lane_base + 256 + c, v);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] *= alpha;
            tmem_st32(tmem + lane_base + 256 + c, v);
          }
        }
      }
      float ls = 0.f;
      const float msafe = mn == -INFINITY ? 0.f : mn;
#pragma unroll
      for (int c = 0; c < kFaN; c += 8) {
        alignas(16) __nv_bfloat16 pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float pe = exp2f(s[c + e] - msafe);
          ls += pe;
          pv[e] = __float2bfloat16(pe);
        }
        const int box = c >> 6;
        const int chunk = ((c & 63) >> 3) ^ (r & 7);
        *reinterpret_cast<uint4*>(sP + box * kFaBox + r * 128 + chunk * 16) = *reinterpret_cast<uint4*>(pv);
      }
      l = l * alpha + ls;
      m = mn;
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && ntiles > 0 && mbar_wait(o_ready, (ntiles - 1) & 1)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const long orow = (long)b * p.S + q0 + r;
      const __nv_bfloat16* gate = p.qg + orow * p.qg_row + (long)h * 512 + 256;
      __nv_bfloat16* out = p.out + orow * p.out_row + (long)h * 256;
#pragma unroll 1
      for (int c = 0; c < 256; c += 32) {
        float v[32];
        tmem_ld32(tmem + lane_base + 256 + c, v);
        if (row_real) {
          alignas(16) __nv_bfloat16 o[32];
          alignas(16) __nv_bfloat16 gv[32];
#pragma unroll
          for (int k = 0; k < 4; ++k) reinterpret_cast<uint4*>(gv)[k] = reinterpret_cast<const uint4*>(gate + c)[k];
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float2bfloat16(v[e] * inv * sigmoid_f(__bfloat162float(gv[e])));
#pragma unroll
          for (int k = 0; k < 4; ++k) reinterpret_cast<uint4*>(out + c)[k] = reinterpret_cast<uint4*>(o)[k];
        }
      }
    } else if (!ok) {
      set_status(p.status, kStatusMbarTimeout);
      *abort_flag = 1;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

void gqa_prefill(const GqaPrefillArgs& p, cudaStream_t stream) {
  BWN_CHECK(p.rope_dim % 16 == 0 && p.rope_dim <= 256, "gqa_prefill: rope_dim must be a multiple of 16");
  BWN_CHECK(p.q_heads % p.kv_heads == 0, "gqa_prefill: q_heads %% kv_heads");
  BWN_CHECK(p.S_pad % kFaM == 0 && p.S_pad >= p.S, "gqa_prefill: S_pad");
  gqa_prefill_prep_kernel<<<dim3(p.S_pad, p.batch), 256, 0, stream>>>(p);
  BWN_CUDA_CHECK(cudaGetLastError());
  CUtensorMap tq, tk, tv;
  make_tmap_2d_bf16(&tq, p.q_rot, (long)p.batch * p.q_heads * p.S_pad, 256, 256, kFaM, 64);
  const long kv_rows = (long)p.batch * p.kv_heads * p.s_max;
  make_tmap_2d_bf16(&tk, p.k_cache, kv_rows, 256, 256, kFaN, 64);
  make_tmap_2d_bf16(&tv, p.v_cache, kv_rows, 256, 256, kFaN, 64);
  static bool set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    BWN_CUDA_CHECK(cudaFuncSetAttribute(flash_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFaSmem));
    set[dev & 63] = true;
  }
  flash_prefill_kernel<<<dim3(p.S_pad / kFaM, p.q_heads, p.batch), kFaThreads, kFaSmem, stream>>>(tq, tk, tv, p);
  BWN_CUDA_CHECK(cudaGetLastError());
}

// =============================================================================
// DeltaNet prep: conv + SiLU, q/k L2 norm, gates
// =============================================================================
__global__ void __launch_bounds__(256) dn_prefill_prep_kernel(DnPrefillArgs p) {
  const int t = blockIdx.x, b = blockIdx.y;
  const int KD = p.k_heads * 128, C = 2 * KD + p.v_heads * 128;
  if (t >= p.S) {  // pad rows of the last chunk: zero, so whole-chunk tiles need no masking
    for (int i = threadIdx.x; i < p.k_heads * 128; i += blockDim.x) {
      const long o = (((long)b * p.k_heads + (i >> 7)) * p.S_pad + t) * 128 + (i & 127);
      p.q_out[o] = __float2bfloat16(0.f);
      p.k_out[o] = __float2bfloat16(0.f);
    }
    for (int i = threadIdx.x; i < p.v_heads * 128; i += blockDim.x)
      p.v_out[(((long)b * p.v_heads + (i >> 7)) * p.S_pad + t) * 128 + (i & 127)] = __float2bfloat16(0.f);
    for (int h = threadIdx.x; h < p.v_heads; h += blockDim.x) {
      p.g_out[((long)b * p.v_heads + h) * p.S_pad + t] = 0.f;
      p.beta_out[((long)b * p.v_heads + h) * p.S_pad + t] = 0.f;
    }
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __nv_bfloat16* row = p.qkv + ((long)b * p.S + t) * p.qkv_row;
  const __nv_bfloat16* ring = p.conv_ring + (long)b * p.ring_slots * C;
  const int start = prefill_start(p);
  auto hist = [&](int ch, int back) -> float {  // x at position start+t-back
    const int tt = t - back;
    if (tt >= 0) return __bfloat162float(row[(long)(-back) * p.qkv_row + ch]);
    const int pos = start + tt;
    if (pos < 0) return 0.f;
    return __bfloat162float(ring[(pos & (p.ring_slots - 1)) * C + ch]);
  };
  auto conv = [&](int ch) -> float {
    const float4 w = *reinterpret_cast<const float4*>(p.conv_w + (long)ch * 4);
    return silu_f(w.x * hist(ch, 3) + w.y * hist(ch, 2) + w.z * hist(ch, 1) + w.w * __bfloat162float(row[ch]));
  };
  // q and k heads: one warp per head, 4 channels per lane
  const float qs = rsqrtf(128.f);
  for (int hh = warp; hh < 2 * p.k_heads; hh += 8) {
    const bool isq = hh < p.k_heads;
    const int kh = isq ? hh : hh - p.k_heads;
    const int ch0 = (isq ? 0 : KD) + kh * 128;
    float x[4];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      x[e] = conv(ch0 + lane * 4 + e);
      ss += x[e] * x[e];
    }
    ss = warp_sum(ss);
    const float inv = 1.f / fmaxf(sqrtf(ss), p.l2_eps) * (isq ? qs : 1.f);
    __nv_bfloat16* dst = (isq ? p.q_out : p.k_out) + (((long)b * p.k_heads + kh) * p.S_pad + t) * 128 + lane * 4;
#pragma unroll
    for (int e = 0; e < 4; ++e) dst[e] = __float2bfloat16(x[e] * inv);
  }
  for (int ch = threadIdx.x; ch < p.v_heads * 128; ch += blockDim.x) {
    const int vh = ch >> 7, d = ch & 127;
    p.v_out[(((long)b * p.v_heads + vh) * p.S_pad + t) * 128 + d] = __float2bfloat16(conv(2 * KD + ch));
  }
  const bool live = t < p.valid_len[b];
  for (int h = threadIdx.x; h < p.v_heads; h += blockDim.x) {
    const long gi = ((long)b * p.v_heads + h) * p.S_pad + t;
    if (live) {
      const float a = __bfloat162float(p.a[((long)b * p.S + t) * p.ab_row + h]);
      const float bb = __bfloat162float(p.b[((long)b * p.S + t) * p.ab_row + h]);
      p.g_out[gi] = -__expf(p.A_log[h]) * softplus_f(a + p.dt_bias[h]);
      p.beta_out[gi] = sigmoid_f(bb);
    } else {
      p.g_out[gi] = 0.f;
      p.beta_out[gi] = 0.f;
    }
  }
}

__global__ void dn_ring_update_kernel(DnPrefillArgs p) {
  const int b = blockIdx.y;
  const int KD = p.k_heads * 128, C = 2 * KD + p.v_heads * 128;
  const int vl = p.valid_len[b];
  const int start = prefill_start(p);
  for (int back = 1; back <= 3; ++back) {
    const int t = vl - back;
    if (t < 0) continue;
    const __nv_bfloat16* row = p.qkv + ((long)b * p.S + t) * p.qkv_row;
    __nv_bfloat16* dst = p.conv_ring + ((long)b * p.ring_slots + ((start + t) & (p.ring_slots - 1))) * C;
    for (int ch = blockIdx.x * blockDim.x + threadIdx.x; ch < C; ch += gridDim.x * blockDim.x) dst[ch] = row[ch];
  }
}

// =============================================================================
// chunked gated delta rule (CUDA cores, fp32 in shared memory)
// =============================================================================
constexpr int kCk = 64;    // chunk length
constexpr int kLD = 129;   // padded row stride for [*, 128] fp32 tiles
constexpr int kLDc = 65;   // padded row stride for [64, 64] tiles
constexpr int kDnChunkSmem =
    (2 * kCk * kLD /*K,Q*/ + 2 * kCk * kLD /*V->U->Vn, W*/ + 128 * kLD /*S*/ + 2 * kCk * kLDc /*A/P, T*/ +
     4 * kCk /*G, beta, eG, misc*/) * 4;

// acc[i][j] += sum_k A(m_i, k) * B(k, n_j) with m_i = ty + i*(M/TM), n_j = tx + j*(N/TN)
template <int M, int N, int TM, int TN>
__device__ __forceinline__ void mm_acc(float (&acc)[TM][TN], const float* A, int ams, int aks, const float* B, int bks,
                                       int bns, int K) {
  const int tx = threadIdx.x % (N / TN), ty = threadIdx.x / (N / TN);
  for (int k = 0; k < K; ++k) {
    float a[TM], bv[TN];
#pragma unroll
    for (int i = 0; i < TM; ++i) a[i] = A[(ty + i * (M / TM)) * ams + k * aks];
#pragma unroll
    for (int j = 0; j < TN; ++j) bv[j] = B[k * bks + (tx + j * (N / TN)) * bns];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] += a[i] * bv[j];
  }
}

template <typename StateT>
__global__ void __launch_bounds__(256, 1) dn_chunk_kernel(DnPrefillArgs p) {
  extern __shared__ float fsm[];
  float* sK = fsm;                   // [64][129]
  float* sQ = sK + kCk * kLD;        // [64][129]
  float* sV = sQ + kCk * kLD;        // [64][129]  v -> U -> Vn
  float* sW = sV + kCk * kLD;        // [64][129]
  float* sS = sW + kCk * kLD;        // [128][129] state (k rows, v cols)
  float* sA = sS + 128 * kLD;        // [64][65]   A, later P
  float* sT = sA + kCk * kLDc;       // [64][65]   T = (I - A)^-1
  float* sG = sT + kCk * kLDc;       // [64] cumulative log-decay
  float* sB = sG + kCk;              // [64] beta
  float* sRow = sB + kCk;            // [64] row scratch (norm sums)
  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x;
  const int rep = p.v_heads / p.k_heads, kh = h / rep;
  StateT* gS = reinterpret_cast<StateT*>(p.state) + ((long)b * p.v_heads + h) * 128 * 128;
  for (int i = tid; i < 128 * 128; i += 256) sS[(i >> 7) * kLD + (i & 127)] = to_f(gS[i]);
  const __nv_bfloat16* gq = p.q_out + ((long)b * p.k_heads + kh) * p.S_pad * 128;
  const __nv_bfloat16* gk = p.k_out + ((long)b * p.k_heads + kh) * p.S_pad * 128;
  const __nv_bfloat16* gv = p.v_out + ((long)b * p.v_heads + h) * p.S_pad * 128;
  const float* gg = p.g_out + ((long)b * p.v_heads + h) * p.S_pad;
  const float* gb = p.beta_out + ((long)b * p.v_heads + h) * p.S_pad;
  const int nchunks = (p.S + kCk - 1) / kCk;
  for (int cidx = 0; cidx < nchunks; ++cidx) {
    const int t0 = cidx * kCk;
    __syncthreads();
    // ---- load chunk (rows beyond S are zero; their g = beta = 0) ----
    for (int i = tid; i < kCk * 128; i += 256) {
      const int r = i >> 7, d = i & 127;
      const bool in = t0 + r < p.S;
      sK[r * kLD + d] = in ? __bfloat162float(gk[(long)(t0 + r) * 128 + d]) : 0.f;
      sQ[r * kLD + d] = in ? __bfloat162float(gq[(long)(t0 + r) * 128 + d]) : 0.f;
      sV[r * kLD + d] = in ? __bfloat162float(gv[(long)(t0 + r) * 128 + d]) : 0.f;
    }
    if (tid < 32) {  // cumulative sum of g over the chunk (two values per lane)
      float g0 = (t0 + 2 * tid < p.S) ? gg[t0 + 2 * tid] : 0.f;
      float g1 = (t0 + 2 * tid + 1 < p.S) ? gg[t0 + 2 * tid + 1] : 0.f;
      float s2 = g0 + g1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n = __shfl_up_sync(0xffffffffu, s2, o);
        if (tid >= o) s2 += n;
      }
      sG[2 * tid] = s2 - g1;
      sG[2 * tid + 1] = s2;
      sB[2 * tid] = (t0 + 2 * tid < p.S) ? gb[t0 + 2 * tid] : 0.f;
      sB[2 * tid + 1] = (t0 + 2 * tid + 1 < p.S) ? gb[t0 + 2 * tid + 1] : 0.f;
    }
    __syncthreads();
    // ---- A = -beta_i exp(G_i - G_j) k_i.k_j  (j < i) ----
    {
      float acc[4][4] = {};
      mm_acc<64, 64, 4, 4>(acc, sK, kLD, 1, sK, 1, kLD, 128);
      const int tx = tid % 16, ty = tid / 16;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int m = ty + i * 16, n = tx + j * 16;
          sA[m * kLDc + n] = n < m ? -sB[m] * __expf(sG[m] - sG[n]) * acc[i][j] : 0.f;
        }
    }
    __syncthreads();
    // ---- T = (I - A)^-1 by forward substitution: 4 threads per column ----
    {
      const int c = tid >> 2, qq = tid & 3;
      for (int i = 0; i < kCk; ++i) {
        float part = 0.f;
        if (i > c)
          for (int j = c + 1 + qq; j < i; j += 4) part += sA[i * kLDc + j] * sT[j * kLDc + c];
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
        if (qq == 0) sT[i * kLDc + c] = i == c ? 1.f : (i > c ? sA[i * kLDc + c] + part : 0.f);
        __syncwarp();
      }
    }
    __syncthreads();
    // ---- U = T (beta V)  -> registers;  W = T (beta K e^G) -> sW ----
    {
      float u[4][8] = {};
      float w[4][8] = {};
      const int tx = tid % 16, ty = tid / 16;
      for (int k = 0; k < kCk; ++k) {
        const float bk = sB[k], bke = sB[k] * __expf(sG[k]);
        float a[4], bv[8], bw[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = sT[(ty + i * 16) * kLDc + k];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          bv[j] = sV[k * kLD + tx + j * 16] * bk;
          bw[j] = sK[k * kLD + tx + j * 16] * bke;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            u[i][j] += a[i] * bv[j];
            w[i][j] += a[i] * bw[j];
          }
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          sV[(ty + i * 16) * kLD + tx + j * 16] = u[i][j];
          sW[(ty + i * 16) * kLD + tx + j * 16] = w[i][j];
        }
    }
    __syncthreads();
    // ---- Vn = U - W S ----
    {
      float x[4][8] = {};
      mm_acc<64, 128, 4, 8>(x, sW, kLD, 1, sS, kLD, 1, 128);
      const int tx = tid % 16, ty = tid / 16;
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) sV[(ty + i * 16) * kLD + tx + j * 16] -= x[i][j];
    }
    // ---- P = (Q K^T) . exp(G_i - G_j), j <= i  -> sA ----
    {
      float acc[4][4] = {};
      mm_acc<64, 64, 4, 4>(acc, sQ, kLD, 1, sK, 1, kLD, 128);
      const int tx = tid % 16, ty = tid / 16;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int m = ty + i * 16, n = tx + j * 16;
          sA[m * kLDc + n] = n <= m ? __expf(sG[m] - sG[n]) * acc[i][j] : 0.f;
        }
    }
    __syncthreads();
    // ---- O = (Q S) e^G + P Vn ; gated RMSNorm ; store ----
    {
      float o[4][8] = {};
      mm_acc<64, 128, 4, 8>(o, sQ, kLD, 1, sS, kLD, 1, 128);
      const int tx = tid % 16, ty = tid / 16;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float e = __expf(sG[ty + i * 16]);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[i][j] *= e;
      }
      mm_acc<64, 128, 4, 8>(o, sA, kLDc, 1, sV, kLD, 1, kCk);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += o[i][j] * o[i][j];
        // the 16 threads sharing this row are 16 consecutive lanes
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        const int m = ty + i * 16;
        const int t = t0 + m;
        if (t < p.S) {
          const float inv = rsqrtf(ss / 128.f + p.norm_eps);
          const __nv_bfloat16* z = p.z + ((long)b * p.S + t) * p.z_row + h * 128;
          __nv_bfloat16* out = p.out + ((long)b * p.S + t) * p.out_row + h * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int n = tx + j * 16;
            out[n] = __float2bfloat16(o[i][j] * inv * p.norm_w[n] * silu_f(__bfloat162float(z[n])));
          }
        }
      }
    }
    __syncthreads();
    // ---- S' = e^{G_C} S + (K e^{G_C - G})^T Vn ----
    {
      const float gC = sG[kCk - 1];
      const float egC = __expf(gC);
      float s2[8][8];
      const int tx = tid % 16, ty = tid / 16;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) s2[i][j] = egC * sS[(ty + i * 16) * kLD + tx + j * 16];
      for (int k = 0; k < kCk; ++k) {
        const float dk = __expf(gC - sG[k]);
        float a[8], bv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) a[i] = sK[k * kLD + ty + i * 16] * dk;
#pragma unroll
        for (int j = 0; j < 8; ++j) bv[j] = sV[k * kLD + tx + j * 16];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) s2[i][j] += a[i] * bv[j];
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) sS[(ty + i * 16) * kLD + tx + j * 16] = s2[i][j];
    }
  }
  __syncthreads();
  for (int i = tid; i < 128 * 128; i += 256) gS[i] = from_f<StateT>(sS[(i >> 7) * kLD + (i & 127)]);
}

static bool dn_tc_enabled() {
  static const bool on = [] {
    const char* e = getenv("BWN_DN_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

void deltanet_prefill(const DnPrefillArgs& p, cudaStream_t stream) {
  BWN_CHECK(p.S_pad >= p.S, "deltanet_prefill: S_pad");
  dn_prefill_prep_kernel<<<dim3(p.S_pad, p.batch), 256, 0, stream>>>(p);
  BWN_CUDA_CHECK(cudaGetLastError());
  if (dn_tc_enabled() && p.status && deltanet_chunk_tc_supported(p)) {
    deltanet_chunk_tc(p, p.status, stream);
    dn_ring_update_kernel<<<dim3(8, p.batch), 256, 0, stream>>>(p);
    BWN_CUDA_CHECK(cudaGetLastError());
    return;
  }
  static bool set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    BWN_CUDA_CHECK(cudaFuncSetAttribute(dn_chunk_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kDnChunkSmem));
    BWN_CUDA_CHECK(cudaFuncSetAttribute(dn_chunk_kernel<__nv_bfloat16>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, kDnChunkSmem));
    set[dev & 63] = true;
  }
  if (p.state_bf16)
    dn_chunk_kernel<__nv_bfloat16><<<dim3(p.v_heads, p.batch), 256, kDnChunkSmem, stream>>>(p);
  else
    dn_chunk_kernel<float><<<dim3(p.v_heads, p.batch), 256, kDnChunkSmem, stream>>>(p);
  BWN_CUDA_CHECK(cudaGetLastError());
  dn_ring_update_kernel<<<dim3(8, p.batch), 256, 0, stream>>>(p);
  BWN_CUDA_CHECK(cudaGetLastError());
}

}  // namespace bwn
