// Gated GQA decode step (one query token per sequence), fused end to end:
// per-head q RMSNorm(1+w) and partial RoPE, the new K row's RMSNorm + RoPE,
// append of the new K/V rows to the cache, softmax(q k^T / sqrt(D)) V over the
// used prefix [0, pos] (the current row included), and the sigmoid output gate.
// Reference: the GQA tail / stateful tail kernels
// (contrib/qwen3.6-27b/kernels/gqa_tail.py:48-203,
//  contrib/qwen3.6-35b-a3b/kernels/gqa_tail_35b.py:52-394); unlike the
// reference, only the used prefix is read (not the whole max_seq_len).
//
// B200 mapping: flash-decoding.  Grid (splits, KV heads, batch); each CTA takes
// a contiguous key range of its sequence, sized on the device from the
// sequence's own position (so a CUDA graph stays valid as positions advance),
// and streams it in 64-key tiles that TMA loads with the 128-byte swizzle into
// a double-buffered shared-memory ring.  The G query heads of a KV head share
// every K/V byte read.  Scores: 4 threads per key (one 64-dim swizzled box
// each, q quarters padded 4 banks apart so the four boxes' q reads do not
// conflict); P.V: each thread owns 2 head dims over half of the tile's keys and
// reads the probabilities 4 keys at a time.  Per-split (max, sum, acc)
// partials go to a workspace; the last CTA of a (sequence, KV head) to finish
// (atomic ticket, re-armed afterwards) merges them and applies the gate.  Only
// the CTA whose range holds `pos` touches cache row `pos`: it writes the new
// row and substitutes it into its smem tile, so no CTA reads a row being written.
#include <cstdlib>
#include <exception>

#include "common/host.h"
#include "common/sm100.cuh"
#include "common/launch.cuh"
#include "kernels/gqa_decode_noalloc.h"
#include "kernels/launch.h"

namespace bwn {

constexpr int kGD = 256;        // head dim
constexpr int kGTile = 64;      // keys per tile
constexpr int kGThreads = 256;
constexpr int kGBoxBytes = kGTile * 128;           // one [64 keys x 64 dims] swizzled box
constexpr int kGTileBytes = 4 * kGBoxBytes;        // 256 dims = 4 boxes (32 KB)

constexpr int kQStride = 4 * (64 + 4);  // padded q row: each 64-dim quarter starts 4 banks later

__device__ __forceinline__ int qidx(int g, int d) { return g * kQStride + (d >> 6) * 68 + (d & 63); }

// byte offset of element (row r, dim d) inside a tile of 4 swizzled boxes
__device__ __forceinline__ int swz_off(int r, int d) {
  return (d >> 6) * kGBoxBytes + r * 128 + ((((d & 63) >> 3) ^ (r & 7)) << 4) + ((d & 7) << 1);
}

template <int G>
__global__ void __launch_bounds__(kGThreads, 1)
    gqa_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      GqaDecodeArgs p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sK = sm;                         // [2][kGTileBytes]
  uint8_t* sV = sm + 2 * kGTileBytes;       // [2][kGTileBytes]
  float* sQ = reinterpret_cast<float*>(sm + 4 * kGTileBytes);  // [G][kQStride] (padded)
  float* sP = sQ + G * kQStride;            // [G][64]
  float* sNew = sP + G * kGTile;            // [2][256] new k (normed+roped), new v
  float* sRed = sNew + 2 * kGD;             // [8][G+1]
  float* sM = sRed + 8 * (G + 1);           // running max [G]
  float* sL = sM + G;                       // running sum [G]
  float* sAlpha = sL + G;                   // [G]
  // 8-byte align the barriers (float offset of sAlpha+G from the 1024-aligned base)
  const int used = G * kQStride + G * kGTile + 2 * kGD + 8 * (G + 1) + 3 * G;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sAlpha + G + ((used & 1) ? 1 : 2));  // [2]
  int* sTicket = reinterpret_cast<int*>(bar + 2);

  pdl_trigger();
  pdl_wait();
  const int sp = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;  // b: query row
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int ntok = p.n_tok > 1 ? p.n_tok : 1;
  // a position outside [0, s_max) marks an inactive row: nothing is appended
  // and no key is read (the cache row it names does not exist)
  const int pos_in = p.positions[b];
  const int pos = pos_in < p.s_max ? pos_in : -1;
  const int L = pos + 1;  // keys 0..pos
  int chunk = (L + p.splits - 1) / p.splits;
  chunk = (chunk + kGTile - 1) / kGTile * kGTile;
  const int k0 = sp * chunk;
  const int k1 = min(L, k0 + chunk);
  const bool has_pos = ntok == 1 && (pos >= k0 && pos < k1);
  const long row_base = ((long)(b / ntok) * p.kv_heads + kvh) * p.s_max;

  if (t == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  // ---- prologue: q heads (RMSNorm(1+w) -> RoPE -> * 1/sqrt(D)) ----
  const float qscale = rsqrtf((float)kGD);
  {
    float x[G];
    float ss[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int qh = kvh * G + g;
      x[g] = pos >= 0 ? __bfloat162float(p.qg[(long)b * p.qg_stride + (long)qh * 2 * kGD + t]) : 0.f;
      ss[g] = warp_sum(x[g] * x[g]);
    }
    float kx = 0.f, kss = 0.f;
    if (has_pos) {
      kx = __bfloat162float(p.k_new[(long)b * p.kv_new_stride + (long)kvh * kGD + t]);
      kss = warp_sum(kx * kx);
    }
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) sRed[warp * (G + 1) + g] = ss[g];
      sRed[warp * (G + 1) + G] = kss;
    }
    __syncthreads();
    const float qw = 1.f + p.q_norm_w[t];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float tot = 0.f;
      for (int w = 0; w < 8; ++w) tot += sRed[w * (G + 1) + g];
      sQ[qidx(g, t)] = x[g] * rsqrtf(tot / kGD + p.eps) * qw;
    }
    if (has_pos) {
      float tot = 0.f;
      for (int w = 0; w < 8; ++w) tot += sRed[w * (G + 1) + G];
      sNew[t] = kx * rsqrtf(tot / kGD + p.eps) * (1.f + p.k_norm_w[t]);
      sNew[kGD + t] = __bfloat162float(p.v_new[(long)b * p.kv_new_stride + (long)kvh * kGD + t]);
    }
    __syncthreads();
    // partial RoPE on dims [0, R): rotate-half pairing within R
    const int R = p.rope_dim, hr = R >> 1;
    float qr[G];
    float kr = 0.f;
    if (t < R && pos >= 0) {
      const float c = p.cos[(long)pos * R + t], s = p.sin[(long)pos * R + t];
      const int pt = t < hr ? t + hr : t - hr;
      const float sg = t < hr ? -1.f : 1.f;
#pragma unroll
      for (int g = 0; g < G; ++g) qr[g] = sQ[qidx(g, t)] * c + sg * sQ[qidx(g, pt)] * s;
      if (has_pos) kr = sNew[t] * c + sg * sNew[pt] * s;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (t < R) sQ[qidx(g, t)] = qr[g];
      sQ[qidx(g, t)] *= qscale;
    }
    if (has_pos && t < R) sNew[t] = kr;
    if (t < G) {
      sM[t] = -INFINITY;
      sL[t] = 0.f;
    }
    __syncthreads();
    if (has_pos) {  // append the new row to the cache (only this CTA touches row pos)
      p.k_cache[(row_base + pos) * kGD + t] = __float2bfloat16(sNew[t]);
      p.v_cache[(row_base + pos) * kGD + t] = __float2bfloat16(sNew[kGD + t]);
    }
  }

  // ---- main loop over 64-key tiles ----
  float acc[G], acc2[G];  // dims 2*dp and 2*dp+1 over this thread's key half
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g] = acc2[g] = 0.f;
  const int ntiles = k1 > k0 ? (k1 - k0 + kGTile - 1) / kGTile : 0;
  auto issue = [&](int i) {
    const int buf = i & 1;
    const int r0 = (int)(row_base + k0 + i * kGTile);
    mbar_arrive_expect_tx(&bar[buf], 2 * kGTileBytes);
#pragma unroll
    for (int bx = 0; bx < 4; ++bx) {
      tma_load_2d(&tmK, &bar[buf], sK + buf * kGTileBytes + bx * kGBoxBytes, bx * 64, r0);
      tma_load_2d(&tmV, &bar[buf], sV + buf * kGTileBytes + bx * kGBoxBytes, bx * 64, r0);
    }
  };
  if (t == 0 && ntiles > 0) issue(0);
  bool ok = true;
  for (int i = 0; i < ntiles; ++i) {
    const int buf = i & 1;
    if (t == 0 && i + 1 < ntiles) issue(i + 1);
    if (!mbar_wait(&bar[buf], (i >> 1) & 1)) {
      set_status(p.status, kStatusMbarTimeout);
      ok = false;
    }
    if (!__syncthreads_and(ok)) {
      // drain whatever may still be in flight, then leave
      if (t == 0)
        for (int j = 0; j < 2; ++j) mbar_wait(&bar[j], ((i + j) >> 1) & 1, 100000000ull);
      __syncthreads();
      return;
    }
    uint8_t* tk = sK + buf * kGTileBytes;
    uint8_t* tv = sV + buf * kGTileBytes;
    const int kbase = k0 + i * kGTile;
    if (has_pos && pos >= kbase && pos < kbase + kGTile) {
      const int r = pos - kbase;
      *reinterpret_cast<__nv_bfloat16*>(tk + swz_off(r, t)) = __float2bfloat16(sNew[t]);
      *reinterpret_cast<__nv_bfloat16*>(tv + swz_off(r, t)) = __float2bfloat16(sNew[kGD + t]);
      __syncthreads();
    }
    // scores: thread -> (key r, box qt)
    {
      const int r = t >> 2, qt = t & 3;
      float sc[G];
#pragma unroll
      for (int g = 0; g < G; ++g) sc[g] = 0.f;
      const uint8_t* rowp = tk + qt * kGBoxBytes + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 raw4 = *reinterpret_cast<const uint4*>(rowp + ((c ^ (r & 7)) << 4));
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw4);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h2[e]);
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
        const int d0 = qt * 64 + c * 8;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float4 qa = *reinterpret_cast<const float4*>(sQ + qidx(g, d0));
          const float4 qb = *reinterpret_cast<const float4*>(sQ + qidx(g, d0) + 4);
          sc[g] += kf[0] * qa.x + kf[1] * qa.y + kf[2] * qa.z + kf[3] * qa.w + kf[4] * qb.x + kf[5] * qb.y +
                   kf[6] * qb.z + kf[7] * qb.w;
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], 1);
        sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], 2);
      }
      if (qt == 0) {
        const bool valid = (kbase + r) < k1;
#pragma unroll
        for (int g = 0; g < G; ++g) sP[g * kGTile + r] = valid ? sc[g] : -INFINITY;
      }
    }
    __syncthreads();
    // online softmax: warp g handles head g
    if (warp < G) {
      const int g = warp;
      const float s0 = sP[g * kGTile + lane], s1 = sP[g * kGTile + 32 + lane];
      const float mt = warp_max(fmaxf(s0, s1));
      const float mold = sM[g];
      const float mnew = fmaxf(mold, mt);
      const float p0 = s0 == -INFINITY ? 0.f : __expf(s0 - mnew);
      const float p1 = s1 == -INFINITY ? 0.f : __expf(s1 - mnew);
      const float ls = warp_sum(p0 + p1);
      sP[g * kGTile + lane] = p0;
      sP[g * kGTile + 32 + lane] = p1;
      if (lane == 0) {
        const float al = mold == -INFINITY ? 0.f : __expf(mold - mnew);
        sAlpha[g] = al;
        sL[g] = sL[g] * al + ls;
        sM[g] = mnew;
      }
    }
    __syncthreads();
    // P.V: thread -> (key half hf, dim pair dp); probabilities read 4 keys at a time
    {
      const int hf = t >> 7, dp = t & 127;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        acc[g] *= sAlpha[g];
        acc2[g] *= sAlpha[g];
      }
      const int nk = min(kGTile, k1 - kbase);
      const int r0 = hf * 32;
      const int r1 = min(r0 + 32, nk);
      for (int r = r0; r < r1; r += 4) {
        float4 pp[G];
#pragma unroll
        for (int g = 0; g < G; ++g) pp[g] = *reinterpret_cast<const float4*>(sP + g * kGTile + r);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const __nv_bfloat162 v2 = *reinterpret_cast<const __nv_bfloat162*>(tv + swz_off(r + j, 2 * dp));
          const float2 v = __bfloat1622float2(v2);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float pj = j == 0 ? pp[g].x : j == 1 ? pp[g].y : j == 2 ? pp[g].z : pp[g].w;
            acc[g] += pj * v.x;
            acc2[g] += pj * v.y;
          }
        }
      }
    }
    __syncthreads();  // tile buffer free for the TMA issued next iteration
  }

  // ---- fold the two key halves, write partials, last CTA merges ----
  float* sAcc = reinterpret_cast<float*>(sK);  // tile buffers are idle now: [G][256]
  if (t >= 128) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      sAcc[g * kGD + 2 * (t - 128)] = acc[g];
      sAcc[g * kGD + 2 * (t - 128) + 1] = acc2[g];
    }
  }
  __syncthreads();
  const int G2 = 2 + kGD;
  float* ws = p.workspace + ((((long)b * p.kv_heads + kvh) * p.splits + sp) * G) * G2;
  if (t < 128) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      ws[g * G2 + 2 + 2 * t] = acc[g] + sAcc[g * kGD + 2 * t];
      ws[g * G2 + 3 + 2 * t] = acc2[g] + sAcc[g * kGD + 2 * t + 1];
    }
  }
  if (t < G) {
    ws[t * G2 + 0] = sM[t];
    ws[t * G2 + 1] = sL[t];
  }
  __threadfence();
  __syncthreads();
  if (t == 0) *sTicket = atomicAdd(&p.tickets[b * p.kv_heads + kvh], 1);
  __syncthreads();
  if (*sTicket != p.splits - 1) return;
  __threadfence();
  const float* wsb = p.workspace + (((long)b * p.kv_heads + kvh) * p.splits) * G * G2;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float M = -INFINITY;
    for (int s = 0; s < p.splits; ++s) M = fmaxf(M, __ldcg(wsb + ((long)s * G + g) * G2));
    float Lsum = 0.f, o = 0.f;
    for (int s = 0; s < p.splits; ++s) {
      const float* e = wsb + ((long)s * G + g) * G2;
      const float m = __ldcg(e);
      if (m == -INFINITY) continue;
      const float w = __expf(m - M);
      Lsum += __ldcg(e + 1) * w;
      o += __ldcg(e + 2 + t) * w;
    }
    const int qh = kvh * G + g;
    const float gate = __bfloat162float(p.qg[(long)b * p.qg_stride + (long)qh * 2 * kGD + kGD + t]);
    const float y = (Lsum > 0.f ? o / Lsum : 0.f) * sigmoid_f(gate);
    p.out[(long)b * p.out_stride + (long)qh * kGD + t] = __float2bfloat16(y);
  }
  if (t == 0) p.tickets[b * p.kv_heads + kvh] = 0;
}

int gqa_decode_workspace_floats(int batch, int q_heads, int kv_heads, int splits) {
  // per (row, head, split): the larger of the two kernels' partial records
  // (CUDA-core: max, sum, O[256]; tensor-core: 16-byte aligned, 4 + 256)
  return batch * q_heads * splits * (4 + kGD);
}

static int gqa_smem_bytes(int G) {
  return 1024 + 4 * kGTileBytes + (G * kQStride + G * kGTile + 2 * kGD + 8 * (G + 1) + 3 * G + 2) * 4 + 64;
}

template <int G>
static void launch_gqa(const CUtensorMap& tk, const CUtensorMap& tv, const GqaDecodeArgs& p, cudaStream_t st) {
  const int smem = gqa_smem_bytes(G);
  static bool set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    BWN_CUDA_CHECK(cudaFuncSetAttribute(gqa_decode_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    set[dev & 63] = true;
  }
  dim3 grid(p.splits, p.kv_heads, p.batch);
  launch_k(gqa_decode_kernel<G>, grid, dim3(kGThreads), smem, st, tk, tv, p);
}

// Multi-token verify: RMSNorm(1+w) + partial RoPE of every new K row, and the
// K/V rows written at their positions, before any row's attention reads them.
__global__ void __launch_bounds__(kGD) gqa_kv_append_kernel(GqaDecodeArgs p) {
  pdl_trigger();
  pdl_wait();
  const int kvh = blockIdx.x, r = blockIdx.y, t = threadIdx.x;
  const int pos = p.positions[r];
  if (pos < 0 || pos >= p.s_max) return;
  __shared__ float sk[kGD];
  __shared__ float red[kGD / 32];
  const float kx = __bfloat162float(p.k_new[(long)r * p.kv_new_stride + (long)kvh * kGD + t]);
  const float ss = warp_sum(kx * kx);
  if ((t & 31) == 0) red[t >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < kGD / 32; ++w) tot += red[w];
  sk[t] = kx * rsqrtf(tot / kGD + p.eps) * (1.f + p.k_norm_w[t]);
  __syncthreads();
  const int R = p.rope_dim, hr = R >> 1;
  float kv = sk[t];
  if (t < R) {
    const float c = p.cos[(long)pos * R + t], s = p.sin[(long)pos * R + t];
    kv = sk[t] * c + (t < hr ? -1.f : 1.f) * sk[t < hr ? t + hr : t - hr] * s;
  }
  const long row = ((long)(r / p.n_tok) * p.kv_heads + kvh) * p.s_max + pos;
  p.k_cache[row * kGD + t] = __float2bfloat16(kv);
  p.v_cache[row * kGD + t] = p.v_new[(long)r * p.kv_new_stride + (long)kvh * kGD + t];
}

bool gqa_decode_tc_supported(const GqaDecodeArgs& p);
void gqa_decode_tc(const CUtensorMap& tk, const CUtensorMap& tv, const GqaDecodeArgs& p, cudaStream_t st);

static bool tc_enabled() {
  static const bool on = [] {
    const char* e = getenv("BWN_GQA_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

void gqa_decode(const GqaDecodeArgs& p, cudaStream_t stream) {
  BWN_CHECK(p.q_heads % p.kv_heads == 0, "gqa_decode: q_heads %% kv_heads");
  BWN_CHECK(p.rope_dim <= kGD && p.rope_dim % 2 == 0, "gqa_decode: bad rope_dim");
  const int ntok = p.n_tok > 1 ? p.n_tok : 1;
  BWN_CHECK(p.batch % ntok == 0, "gqa_decode: rows %% n_tok");
  if (tc_enabled() && gqa_decode_tc_supported(p)) {
    // tensor-core path: append the new K/V rows, then attention over the cache
    GqaDecodeArgs q = p;
    q.n_tok = ntok;
    launch_k(gqa_kv_append_kernel, dim3(q.kv_heads, q.batch), dim3(kGD), 0, stream, q);
    const int pairs = (q.batch / ntok) * q.kv_heads;
    int splits = std::max(1, std::min(p.splits, num_sms() / std::max(1, pairs)));
    splits = std::min(splits, (q.s_max + 63) / 64);
    q.splits = splits;
    CUtensorMap tk, tv;  // 64-key x 64-dim boxes (the kernel's K/V tile is four of them)
    const long rows = (long)(q.batch / ntok) * q.kv_heads * q.s_max;
    make_tmap_2d_bf16(&tk, q.k_cache, rows, kGD, kGD, 64, 64);
    make_tmap_2d_bf16(&tv, q.v_cache, rows, kGD, kGD, 64, 64);
    gqa_decode_tc(tk, tv, q, stream);
    return;
  }
  if (ntok > 1) launch_k(gqa_kv_append_kernel, dim3(p.kv_heads, p.batch), dim3(kGD), 0, stream, p);
  const int G = p.q_heads / p.kv_heads;
  CUtensorMap tk, tv;
  const long rows = (long)(p.batch / ntok) * p.kv_heads * p.s_max;
  make_tmap_2d_bf16(&tk, p.k_cache, rows, kGD, kGD, kGTile, 64);
  make_tmap_2d_bf16(&tv, p.v_cache, rows, kGD, kGD, kGTile, 64);
  switch (G) {
    case 1: launch_gqa<1>(tk, tv, p, stream); break;
    case 2: launch_gqa<2>(tk, tv, p, stream); break;
    case 3: launch_gqa<3>(tk, tv, p, stream); break;
    case 4: launch_gqa<4>(tk, tv, p, stream); break;
    case 6: launch_gqa<6>(tk, tv, p, stream); break;
    case 8: launch_gqa<8>(tk, tv, p, stream); break;
    default: BWN_FAIL("gqa_decode: unsupported group size %d", G);
  }
}


// ===========================================================================
// Allocation-free entry point (C ABI, declared in kernels/gqa_decode_noalloc.h).
// It has no counterpart in the reference: it serves callers that cannot
// allocate device memory (runtimes that own every byte of GPU memory, plugin
// hosts that forbid allocation after start-up, paths that must not risk the
// implicit synchronisation of cudaMalloc).  Its split-KV partials, merge
// tickets and status word are the file-scope device arrays below: one copy
// per GPU that loads the library, kept until exit, shared by every call (calls
// that overlap on the GPU race).  kNoAllocScratchFloats (1 Mi floats = 4 MiB)
// holds batch * q_heads * splits * (4 + 256) floats; the split count is
// lowered to fit, and a problem that does not fit with one split is rejected.
// ===========================================================================
namespace {
constexpr long kNoAllocScratchFloats = 1L << 20;
constexpr int kNoAllocTickets = 4096;
constexpr int kNoAllocMaxDevices = 64;
}  // namespace

static __device__ __align__(256) float g_noalloc_partials[kNoAllocScratchFloats];
static __device__ __align__(256) int g_noalloc_tickets[kNoAllocTickets];
static __device__ __align__(256) int g_noalloc_status[64];

static float* g_noalloc_partials_ptr[kNoAllocMaxDevices] = {nullptr};
static int* g_noalloc_tickets_ptr[kNoAllocMaxDevices] = {nullptr};
static int* g_noalloc_status_ptr[kNoAllocMaxDevices] = {nullptr};

// Resolves the arrays' device addresses once per device, with that device
// current (host code cannot pass the symbols themselves to a kernel).
static bool noalloc_setup(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return false;
  *dev_out = dev;
  if (g_noalloc_partials_ptr[dev]) return true;
  void* p0 = nullptr;
  void* p1 = nullptr;
  void* p2 = nullptr;
  if (cudaGetSymbolAddress(&p0, g_noalloc_partials) != cudaSuccess) return false;
  if (cudaGetSymbolAddress(&p1, g_noalloc_tickets) != cudaSuccess) return false;
  if (cudaGetSymbolAddress(&p2, g_noalloc_status) != cudaSuccess) return false;
  g_noalloc_tickets_ptr[dev] = static_cast<int*>(p1);
  g_noalloc_status_ptr[dev] = static_cast<int*>(p2);
  g_noalloc_partials_ptr[dev] = static_cast<float*>(p0);
  return true;
}

}  // namespace bwn

extern "C" int bwn_gqa_decode_noalloc_status(int* status_out, cudaStream_t stream) {
  using namespace bwn;
  if (!status_out) return BWN_NOALLOC_BAD_ARGUMENT;
  int dev = 0;
  if (!noalloc_setup(&dev)) return BWN_NOALLOC_CUDA_ERROR;
  if (cudaMemcpyAsync(status_out, g_noalloc_status_ptr[dev], sizeof(int), cudaMemcpyDeviceToHost, stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return BWN_NOALLOC_CUDA_ERROR;
  return BWN_NOALLOC_OK;
}

extern "C" int bwn_gqa_decode_noalloc(const void* qg, long qg_stride, const void* k_new, const void* v_new,
                                      long kv_new_stride, const float* q_norm_w, const float* k_norm_w,
                                      const float* cos, const float* sin, void* k_cache, void* v_cache,
                                      const int* positions, void* out, long out_stride, int batch, int q_heads,
                                      int kv_heads, int s_max, int rope_dim, float eps, int splits,
                                      cudaStream_t stream) {
  using namespace bwn;
  if (!qg || !k_new || !v_new || !q_norm_w || !k_norm_w || !cos || !sin || !k_cache || !v_cache || !positions ||
      !out || batch <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads != 0 || s_max <= 0 ||
      rope_dim <= 0 || rope_dim > 256 || (rope_dim & 1))
    return BWN_NOALLOC_BAD_ARGUMENT;
  const int G = q_heads / kv_heads;
  if (!(G == 1 || G == 2 || G == 3 || G == 4 || G == 6 || G == 8)) return BWN_NOALLOC_BAD_ARGUMENT;
  if ((long)batch * kv_heads > kNoAllocTickets) return BWN_NOALLOC_SCRATCH_TOO_SMALL;
  const long per_split = (long)batch * q_heads * (4 + 256);
  if (per_split > kNoAllocScratchFloats) return BWN_NOALLOC_SCRATCH_TOO_SMALL;
  int dev = 0;
  if (!noalloc_setup(&dev)) return BWN_NOALLOC_CUDA_ERROR;
  if (splits <= 0) splits = 8;
  const long max_splits = kNoAllocScratchFloats / per_split;
  if (splits > max_splits) splits = (int)max_splits;
  if (splits > (s_max + 63) / 64) splits = (s_max + 63) / 64;
  if (splits < 1) splits = 1;
  // tickets must start at zero (a call that gave up a bounded wait may leave
  // them set); the status word reports this call only
  if (cudaMemsetAsync(g_noalloc_tickets_ptr[dev], 0, sizeof(int) * (size_t)batch * kv_heads, stream) != cudaSuccess)
    return BWN_NOALLOC_CUDA_ERROR;
  if (cudaMemsetAsync(g_noalloc_status_ptr[dev], 0, sizeof(int), stream) != cudaSuccess) return BWN_NOALLOC_CUDA_ERROR;
  GqaDecodeArgs p{};
  p.qg = static_cast<const __nv_bfloat16*>(qg);
  p.qg_stride = qg_stride;
  p.k_new = static_cast<const __nv_bfloat16*>(k_new);
  p.v_new = static_cast<const __nv_bfloat16*>(v_new);
  p.kv_new_stride = kv_new_stride;
  p.q_norm_w = q_norm_w;
  p.k_norm_w = k_norm_w;
  p.cos = cos;
  p.sin = sin;
  p.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  p.positions = positions;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.workspace = g_noalloc_partials_ptr[dev];
  p.tickets = g_noalloc_tickets_ptr[dev];
  p.status = g_noalloc_status_ptr[dev];
  p.batch = batch;
  p.q_heads = q_heads;
  p.kv_heads = kv_heads;
  p.s_max = s_max;
  p.rope_dim = rope_dim;
  p.splits = splits;
  p.eps = eps;
  try {
    gqa_decode(p, stream);
  } catch (const std::exception&) {
    return cudaPeekAtLastError() != cudaSuccess ? BWN_NOALLOC_CUDA_ERROR : BWN_NOALLOC_INTERNAL_ERROR;
  }
  return BWN_NOALLOC_OK;
}
