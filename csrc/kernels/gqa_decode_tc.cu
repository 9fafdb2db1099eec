// Gated GQA decode attention on the tcgen05 tensor cores (one or a few query
// tokens per sequence).  Reference: the GQA tail kernels
// (contrib/qwen3.6-27b/kernels/gqa_tail.py:48-203,
//  contrib/qwen3.6-35b-a3b/kernels/gqa_tail_35b.py:52-394).
//
// The G query heads of a KV head (times the tokens of a multi-token verify)
// are the MMA rows of one CTA: Q [128 rows x 256] is normalised (RMSNorm(1+w)),
// rotated (partial RoPE) and scaled by the softmax warps straight into shared
// memory, then every 128-key tile of the CTA's split of the cache runs
//   S = Q K^T   (tcgen05, fp32 in TMEM, double-buffered)
//   P = exp2(S - m)  -> bf16 in shared memory (one thread per query row)
//   O += P V    (tcgen05, V MN-major, O rescaled lazily in TMEM)
// with 64-key K/V tiles streamed by TMA in the 128-byte swizzle through
// two-stage rings, so the next tile's K and V are in flight while this one
// is multiplied and soft-maxed.  The new K/V rows
// are appended by gqa_kv_append_kernel before this kernel runs, so every CTA
// only reads the cache.  Each split writes (max, sum, O) partials; the last
// CTA of a (sequence, KV head) merges them and applies the sigmoid gate.
#include "common/host.h"
#include "common/launch.cuh"
#include "common/sm100.cuh"
#include "kernels/launch.h"

namespace bwn {

namespace {
constexpr int kTM = 128;             // query rows per CTA (G * n_tok, padded)
constexpr int kTN = 64;              // keys per tile
constexpr int kTBox = 128 * 128;     // [128 rows x 64 dims] SW128 box, 16 KB (Q, P)
constexpr int kKBox = kTN * 128;     // [64 keys x 64 dims] SW128 box, 8 KB (K, V)
constexpr int kKTile = 4 * kKBox;    // one 64-key x 256-dim tile, 32 KB
constexpr int kTStages = 2;
constexpr int kTThreads = 192;
constexpr int kTSmem = 1024 + 4 * kTBox /*Q*/ + kTStages * kKTile /*K*/ + kTStages * kKTile /*V*/ + 2 * kTBox /*P*/ + 256;
constexpr float kTLazy = 8.f;        // O is rescaled only when a row's max grows by more than 2^8
constexpr int kTW = 4 + 256;         // partial record: max (log2 units), sum, 2 pad, O[256] (16-byte aligned)
}  // namespace

__global__ void __launch_bounds__(kTThreads, 1)
    gqa_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                         GqaDecodeArgs p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = sm;
  uint8_t* sK = sQ + 4 * kTBox;              // [kTStages] tiles
  uint8_t* sV = sK + kTStages * kKTile;      // [kTStages] tiles (contiguous with sK)
  uint8_t* sP = sV + kTStages * kKTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kTBox);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_empty = bars + 11; // [2]
  uint64_t* p_full = bars + 13;  // [2] P buffer written (128 arrivals)
  uint64_t* p_done = bars + 15;  // [2] PV that read the P buffer has completed (commit)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_ticket = const_cast<int*>(reinterpret_cast<volatile int*>(tmem_slot + 2));

  const int sp = blockIdx.x, kvh = blockIdx.y, cb = blockIdx.z;
  const int warp = warp_id(), lane = lane_id();
  const int ntok = p.n_tok > 1 ? p.n_tok : 1;
  const int G = p.q_heads / p.kv_heads;
  const int nrows = ntok * G;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 17; ++i) mbar_init(&bars[i], (i == 0 || i == 11 || i == 12 || i == 13 || i == 14) ? 128 : 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S0 @0, S1 @128, O @256
  pdl_wait();

  int Lmax = 0;
  for (int i = 0; i < ntok; ++i) {
    const int pi = p.positions[cb * ntok + i];
    if (pi < p.s_max) Lmax = max(Lmax, pi + 1);  // rows at or past s_max are inactive
  }
  int chunk = (Lmax + p.splits - 1) / p.splits;
  chunk = (chunk + kTN - 1) / kTN * kTN;
  const int k0 = sp * chunk;
  const int k1 = min(Lmax, k0 + chunk);
  const int ntiles = k1 > k0 ? (k1 - k0 + kTN - 1) / kTN : 0;
  const long krow0 = ((long)cb * p.kv_heads + kvh) * p.s_max + k0;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (elect_one()) {
      for (int j = 0; j < ntiles && !*abort_flag; ++j) {
        const int st = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(&k_empty[st], ph ^ 1u)) {
          set_status(p.status, kStatusMbarTimeout);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], kKTile);
        for (int bx = 0; bx < 4; ++bx)
          tma_load_2d(&tmK, &k_full[st], sK + st * kKTile + bx * kKBox, bx * 64, (int)(krow0 + j * kTN));
        if (!mbar_wait(&v_empty[st], ph ^ 1u)) {
          set_status(p.status, kStatusMbarTimeout);
          *abort_flag = 1;
          mbar_wait(&k_full[st], ph, 100000000ull);
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], kKTile);
        for (int bx = 0; bx < 4; ++bx)
          tma_load_2d(&tmV, &v_full[st], sV + st * kKTile + bx * kKBox, bx * 64, (int)(krow0 + j * kTN));
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (elect_one()) {
      const uint32_t id_qk = idesc_bf16_f32_major(kTM, kTN, false, false);
      const uint32_t id_pv = idesc_bf16_f32_major(kTM, 256, false, true);
      bool ok = ntiles == 0 || mbar_wait(q_full, 0);
      auto issue_qk = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(&k_full[st], ph)) return false;
        if (!mbar_wait(&s_empty[st], ph ^ 1u)) return false;
        tc_fence_after();
        const uint32_t d = tmem + st * kTN;
        for (int bx = 0; bx < 4; ++bx) {
          const uint64_t da = smem_desc_sw128(smem_u32(sQ + bx * kTBox));
          const uint64_t db = smem_desc_sw128(smem_u32(sK + st * kKTile + bx * kKBox));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_f16(d, da + 2 * kk, db + 2 * kk, id_qk, (bx | kk) ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        umma_commit(&k_empty[st]);
        return true;
      };
      if (ok && ntiles > 0) ok = issue_qk(0);
      for (int j = 0; ok && j < ntiles; ++j) {
        if (j + 1 < ntiles && !issue_qk(j + 1)) {
          ok = false;
          break;
        }
        const int st = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(&v_full[st], ph) || !mbar_wait(&p_full[st], ph)) {
          ok = false;
          break;
        }
        tc_fence_after();
        {
          const uint64_t da = smem_desc_sw128(smem_u32(sP + st * kTBox));
          const uint64_t db = smem_desc_sw128_mn(smem_u32(sV + st * kKTile), kKBox);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_f16(tmem + 256, da + 2 * kk, db + 128 * kk, id_pv, (j | kk) ? 1u : 0u);
        }
        umma_commit(&p_done[st]);
        umma_commit(&v_empty[st]);
      }
      if (!ok) {
        set_status(p.status, kStatusMbarTimeout);
        *abort_flag = 1;
      }
    }
  } else {
    // ------------------------- Q prologue + softmax warps ---------------------
    const int q = warp & 3;
    const int r = q * 32 + lane;  // query row == TMEM lane
    const bool real = r < nrows;
    const int pos_in = real ? p.positions[cb * ntok + r / G] : -1;
    const int pos = pos_in < p.s_max ? pos_in : -1;
    // Q rows, one warp per row (lane = 8 consecutive dims, one 16-byte load):
    // RMSNorm(1+w), partial RoPE (rotate-half within rope_dim, the partner
    // dims fetched from the lane rope_dim/16 away), 1/sqrt(256); an inactive
    // row's q is zero (no RoPE row to read).  Rows past nrows are zeroed.
    {
      const int R = p.rope_dim, hr = R >> 1;
      const int c = lane * 8;
      const float qscale = rsqrtf(256.f);
      float w8[8];
      {
        const float4 w0 = *reinterpret_cast<const float4*>(p.q_norm_w + c);
        const float4 w1 = *reinterpret_cast<const float4*>(p.q_norm_w + c + 4);
        w8[0] = w0.x; w8[1] = w0.y; w8[2] = w0.z; w8[3] = w0.w;
        w8[4] = w1.x; w8[5] = w1.y; w8[6] = w1.z; w8[7] = w1.w;
      }
      const int src_lane = c < R ? (c < hr ? lane + (hr >> 3) : lane - (hr >> 3)) : lane;
      for (int rr = q; rr < kTM; rr += 4) {
        alignas(16) __nv_bfloat16 o8[8];
        const int prr = rr < nrows ? __ldg(p.positions + cb * ntok + rr / G) : -1;
        const bool act = prr >= 0 && prr < p.s_max;  // warp-uniform
        if (act) {
          const int vr = cb * ntok + rr / G, qh = kvh * G + rr % G;
          const uint4 u = *reinterpret_cast<const uint4*>(p.qg + (long)vr * p.qg_stride + (long)qh * 512 + c);
          const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&u);
          float x[8];
          float ss = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            x[e] = __bfloat162float(hb[e]);
            ss += x[e] * x[e];
          }
          ss = warp_sum(ss);
          const float inv = rsqrtf(ss / 256.f + p.eps);
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] *= inv * (1.f + w8[e]);
          float y[8], cs[8], sn[8];
          if (c < R) {
            const float4* cp = reinterpret_cast<const float4*>(p.cos + (long)prr * R + c);
            const float4* sp4 = reinterpret_cast<const float4*>(p.sin + (long)prr * R + c);
            const float4 c0 = cp[0], c1 = cp[1], s0 = sp4[0], s1 = sp4[1];
            cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w; cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
            sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w; sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float xp = __shfl_sync(0xffffffffu, x[e], src_lane);
            y[e] = c < R ? x[e] * cs[e] + (c < hr ? -1.f : 1.f) * xp * sn[e] : x[e];
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) o8[e] = __float2bfloat16(y[e] * qscale);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) o8[e] = __float2bfloat16(0.f);
        }
        const int box = c >> 6, chk = ((c & 63) >> 3) ^ (rr & 7);
        *reinterpret_cast<uint4*>(sQ + box * kTBox + rr * 128 + chk * 16) = *reinterpret_cast<uint4*>(o8);
      }
    }
    fence_async_smem();
    mbar_arrive(q_full);

    const float sl2 = 1.4426950408889634f;  // log2(e); 1/sqrt(D) is folded into q
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    // m: the reference max the row's P and O are taken against (log2 units).
    // It is raised (and O rescaled) only when the row's running max exceeds it
    // by more than kTLazy, so P <= 2^kTLazy and, after the first tiles, the
    // softmax of tile j+1 overlaps the PV of tile j (P is double-buffered).
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // A warp whose 32 rows are all padding (G * n_tok <= 96) computes nothing:
    // it only keeps the barrier phases (same waits and arrivals, same order).
    const bool live = q * 32 < nrows;
    for (int j = 0; j < ntiles; ++j) {
      const int pb = j & 1;
      if (!mbar_wait(&s_full[pb], (uint32_t)(j >> 1) & 1u)) {
        ok = false;
        break;
      }
      // P buffer pb was last read by the PV of tile j - 2
      auto wait_p_free = [&]() -> bool {
        return j < 2 || mbar_wait(&p_done[pb], (uint32_t)((j >> 1) & 1) ^ 1u);
      };
      if (!live) {
        mbar_arrive(&s_empty[pb]);
        if (!wait_p_free()) {
          ok = false;
          break;
        }
        mbar_arrive(&p_full[pb]);
        continue;
      }
      tc_fence_after();
      float s[kTN];
#pragma unroll
      for (int c = 0; c < kTN; c += 32) {
        float v[32];
        tmem_ld32(tmem + lane_base + pb * kTN + c, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) s[c + e] = v[e];
      }
      tc_fence_before();
      mbar_arrive(&s_empty[pb]);
      const int kbase = k0 + j * kTN;
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < kTN; ++c) {
        const int key = kbase + c;
        const bool vis = key <= pos && key < k1;
        s[c] = vis ? s[c] * sl2 : -INFINITY;
        mt = fmaxf(mt, s[c]);
      }
      const bool raise = mt > m + kTLazy;  // (m = -inf: any visible key raises)
      const float mn = raise ? mt : m;
      const float alpha = (m == -INFINITY || !raise) ? 1.f : exp2f(m - mn);
      if (j > 0 && __any_sync(0xffffffffu, raise && m != -INFINITY)) {
        // rescale O: every PV so far (the last one is tile j - 1) must be done
        if (!mbar_wait(&p_done[(j - 1) & 1], (uint32_t)((j - 1) >> 1) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 256; c += 32) {
          float v[32];
          tmem_ld32(tmem + lane_base + 256 + c, v);
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] *= alpha;
          tmem_st32(tmem + lane_base + 256 + c, v);
        }
      }
      if (!wait_p_free()) {
        ok = false;
        break;
      }
      float ls = 0.f;
      const float msafe = mn == -INFINITY ? 0.f : mn;
      uint8_t* pbuf = sP + pb * kTBox;
#pragma unroll
      for (int c = 0; c < kTN; c += 8) {
        alignas(16) __nv_bfloat16 pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float pe = exp2f(s[c + e] - msafe);
          ls += pe;
          pv[e] = __float2bfloat16(pe);
        }
        const int chk = (c >> 3) ^ (r & 7);
        *reinterpret_cast<uint4*>(pbuf + r * 128 + chk * 16) = *reinterpret_cast<uint4*>(pv);
      }
      l = l * alpha + ls;
      m = mn;
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[pb]);
    }
    // ---- this split's partial (max, sum, O) ----
    float* ws = p.workspace + ((((long)cb * p.kv_heads + kvh) * p.splits + sp) * nrows) * kTW;
    if (!live) {
      if (!ok) {
        set_status(p.status, kStatusMbarTimeout);
        *abort_flag = 1;
      }
    } else if (ok && ntiles > 0 && mbar_wait(&p_done[(ntiles - 1) & 1], (uint32_t)((ntiles - 1) >> 1) & 1u)) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 256; c += 32) {
        float v[32];
        tmem_ld32(tmem + lane_base + 256 + c, v);
        if (real) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(ws + (long)r * kTW + 4 + c + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
        }
      }
      if (real) {
        ws[(long)r * kTW + 0] = m;
        ws[(long)r * kTW + 1] = l;
      }
    } else {
      if (!ok) {
        set_status(p.status, kStatusMbarTimeout);
        *abort_flag = 1;
      }
      if (real) {
        ws[(long)r * kTW + 0] = -INFINITY;
        ws[(long)r * kTW + 1] = 0.f;
      }
    }
  }
  // ---- last CTA of (sequence, KV head) merges the splits, applies the gate ----
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) *s_ticket = atomicAdd(&p.tickets[cb * p.kv_heads + kvh], 1);
  __syncthreads();
  if (*s_ticket == p.splits - 1) {
    __threadfence();
    const float* wsb = p.workspace + (((long)cb * p.kv_heads + kvh) * p.splits) * nrows * kTW;
    // Stage every split's partial records in the (now idle) K/V buffers with
    // one coalesced pass, then merge all (row, dim) outputs in parallel.  If a
    // wait gave up, TMA copies may still target those buffers: merge from
    // global memory instead.
    const int nfl = p.splits * nrows * kTW;
    const bool staged = !*abort_flag && nfl * 4 <= 8 * kTBox;
    const float* src = wsb;
    auto ld = [&](const float* q) { return staged ? *q : __ldcg(q); };
    if (staged) {
      float* sw = reinterpret_cast<float*>(sK);  // sK and sV are contiguous: 8 boxes
      for (int i = threadIdx.x * 4; i < nfl; i += blockDim.x * 4)
        *reinterpret_cast<float4*>(sw + i) = __ldcg(reinterpret_cast<const float4*>(wsb + i));
      __syncthreads();
      src = sw;
    }
    for (int idx = threadIdx.x; idx < nrows * 256; idx += blockDim.x) {
      const int rr = idx >> 8, d = idx & 255;
      const int vr = cb * ntok + rr / G, qh2 = kvh * G + rr % G;
      const float gate = __bfloat162float(p.qg[(long)vr * p.qg_stride + (long)qh2 * 512 + 256 + d]);
      float M = -INFINITY;
      for (int s2 = 0; s2 < p.splits; ++s2) M = fmaxf(M, ld(src + ((long)s2 * nrows + rr) * kTW));
      float Ls = 0.f, o = 0.f;
      for (int s2 = 0; s2 < p.splits; ++s2) {
        const float* e = src + ((long)s2 * nrows + rr) * kTW;
        const float mm = ld(e);
        if (mm == -INFINITY) continue;
        const float w = exp2f(mm - M);
        Ls += ld(e + 1) * w;
        o += ld(e + 4 + d) * w;
      }
      p.out[(long)vr * p.out_stride + (long)qh2 * 256 + d] = __float2bfloat16((Ls > 0.f ? o / Ls : 0.f) * sigmoid_f(gate));
    }
    if (threadIdx.x == 0) p.tickets[cb * p.kv_heads + kvh] = 0;
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool gqa_decode_tc_supported(const GqaDecodeArgs& p) {
  const int ntok = p.n_tok > 1 ? p.n_tok : 1;
  const int G = p.q_heads / p.kv_heads;
  return G * ntok <= kTM && p.rope_dim % 16 == 0;  // rope halves on 16-byte chunks
}

void gqa_decode_tc(const CUtensorMap& tk, const CUtensorMap& tv, const GqaDecodeArgs& p, cudaStream_t st) {
  static bool set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    BWN_CUDA_CHECK(cudaFuncSetAttribute(gqa_decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmem));
    set[dev & 63] = true;
  }
  const int ntok = p.n_tok > 1 ? p.n_tok : 1;
  launch_k(gqa_decode_tc_kernel, dim3(p.splits, p.kv_heads, p.batch / ntok), dim3(kTThreads), kTSmem, st, tk, tv,
           p);
}

}  // namespace bwn
