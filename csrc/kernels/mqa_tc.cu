// Single-KV-head ("MQA") attention of DeepSeek V4's latent attention at
// prefill, on the tcgen05 tensor cores.  Reference: the attention of
// contrib/deepseek-v4-flash/run_deepseek_v4_tp.py:315-336 (kv is both the key
// and the value; causal over each token's visible prefix).
//
// MMA rows are (token, head) pairs: a 128-row tile holds 128 / H consecutive
// tokens of one sequence with all H local heads, so the one K/V tile of the
// sequence feeds every row.  Head dim D = 512: S = Q K^T contracts all 512
// dims, while the 128 x 512 fp32 output would fill TMEM alone, so each tile is
// run by two CTAs that own 256 output dims each (both compute S).  Per CTA:
//   Q tile [128 x 512] resident in shared memory (TMA, 8 SW128 boxes);
//   K tiles of 32 keys x 512 dims stream through a two-stage ring; the same
//   tile is the MN-major V operand of PV (this CTA's 256 dims), so K and V
//   cross HBM once;
//   S (double-buffered, 32 TMEM columns each) -> softmax warps -> P (bf16,
//   double-buffered) -> O += P V (256 TMEM columns), with the lazy rescale of
//   O (only when a row's max grows by more than 2^8).
// Key tiles past a tile's last visible key are skipped; tiles are issued
// longest first.  No split over keys, so no partials and no merge.
#include "common/host.h"
#include "common/launch.cuh"
#include "common/sm100.cuh"
#include "kernels/deepseek.h"

namespace bwn {

namespace {
constexpr int kMM = 128;               // MMA rows per tile
constexpr int kMN = 32;                // keys per tile
constexpr int kMD = 512;               // head dim
constexpr int kMQBox = 128 * 128;      // Q box [128 rows x 64 dims], 16 KB
constexpr int kMKBox = kMN * 128;      // K box [32 keys x 64 dims], 4 KB
constexpr int kMKTile = 8 * kMKBox;    // 32 keys x 512 dims, 32 KB
constexpr int kMPBuf = 128 * 128;      // P [128 rows x 128 B] (32 keys used), 16 KB
constexpr int kMThreads = 192;
constexpr int kMSmem = 1024 + 8 * kMQBox + 2 * kMKTile + 2 * kMPBuf + 256;
constexpr float kMLazy = 8.f;
}  // namespace

__global__ void __launch_bounds__(kMThreads, 1)
    mqa_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          MqaArgs a, int kv_rows_per_seq, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = sm;
  uint8_t* sK = sQ + 8 * kMQBox;     // [2] tiles
  uint8_t* sP = sK + 2 * kMKTile;    // [2] buffers
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kMPBuf);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2] (committed after the PV that last read the tile)
  uint64_t* s_full = bars + 5;   // [2]
  uint64_t* s_empty = bars + 7;  // [2] 128 arrivals
  uint64_t* p_full = bars + 9;   // [2] 128 arrivals
  uint64_t* p_done = bars + 11;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_nt = const_cast<int*>(reinterpret_cast<volatile int*>(tmem_slot + 2));

  const int ntiles_m = gridDim.x;
  const int tile = ntiles_m - 1 - (int)blockIdx.x;  // longest (latest tokens) first
  const int half = blockIdx.y;                       // output dims [256 * half, 256 * half + 256)
  const int warp = warp_id(), lane = lane_id();
  const int H = a.H;
  const int tok0 = tile * (kMM / H);
  const int seq = tok0 / a.q_per_seq;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 13; ++i) mbar_init(&bars[i], (i == 7 || i == 8 || i == 9 || i == 10) ? 128 : 1);
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
  const uint32_t tmem = *tmem_slot;  // S0 @0, S1 @32, O @256
  pdl_wait();
  if (threadIdx.x == 0) {
    int mv = 0;
    for (int t = tok0; t < tok0 + kMM / H; ++t) mv = max(mv, a.visible[t]);
    mv = min(mv, kv_rows_per_seq);
    *s_nt = (mv + kMN - 1) / kMN;
  }
  __syncthreads();
  const int ntiles = *s_nt;
  const int krow0 = seq * kv_rows_per_seq;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      if (ntiles > 0) {  // (with no visible key nothing is loaded: no copy may outlive the CTA)
        mbar_arrive_expect_tx(q_full, 8 * kMQBox);
        for (int bx = 0; bx < 8; ++bx) tma_load_2d(&tmQ, q_full, sQ + bx * kMQBox, bx * 64, tile * kMM);
      }
      for (int j = 0; j < ntiles && !*abort_flag; ++j) {
        const int st = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(&k_empty[st], ph ^ 1u)) {
          set_status(status, kStatusMbarTimeout);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], kMKTile);
        for (int bx = 0; bx < 8; ++bx)
          tma_load_2d(&tmK, &k_full[st], sK + st * kMKTile + bx * kMKBox, bx * 64, krow0 + j * kMN);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (elect_one()) {
      const uint32_t id_qk = idesc_bf16_f32_major(kMM, kMN, false, false);
      const uint32_t id_pv = idesc_bf16_f32_major(kMM, 256, false, true);
      bool ok = ntiles == 0 || mbar_wait(q_full, 0);
      auto issue_qk = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(&k_full[st], ph)) return false;
        if (!mbar_wait(&s_empty[st], ph ^ 1u)) return false;
        tc_fence_after();
        const uint32_t d = tmem + st * kMN;
        for (int bx = 0; bx < 8; ++bx) {
          const uint64_t da = smem_desc_sw128(smem_u32(sQ + bx * kMQBox));
          const uint64_t db = smem_desc_sw128(smem_u32(sK + st * kMKTile + bx * kMKBox));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_f16(d, da + 2 * kk, db + 2 * kk, id_qk, (bx | kk) ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
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
        if (!mbar_wait(&p_full[st], ph)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t da = smem_desc_sw128(smem_u32(sP + st * kMPBuf));
        const uint64_t db = smem_desc_sw128_mn(smem_u32(sK + st * kMKTile + 4 * half * kMKBox), kMKBox);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) umma_f16(tmem + 256, da + 2 * kk, db + 128 * kk, id_pv, (j | kk) ? 1u : 0u);
        umma_commit(&p_done[st]);
        umma_commit(&k_empty[st]);
      }
      if (!ok) {
        set_status(status, kStatusMbarTimeout);
        *abort_flag = 1;
      }
    }
  } else {
    // ------------------------------ softmax warps -----------------------------
    const int q = warp & 3;
    const int r = q * 32 + lane;  // tile row == TMEM lane
    const int row = tile * kMM + r;
    const int vis = a.visible[row / H];
    const float sl2 = a.scale * 1.4426950408889634f;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int pb = j & 1;
      if (!mbar_wait(&s_full[pb], (uint32_t)(j >> 1) & 1u)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kMN];
      tmem_ld32(tmem + lane_base + pb * kMN, s);
      tc_fence_before();
      mbar_arrive(&s_empty[pb]);
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < kMN; ++c) {
        const bool v = j * kMN + c < vis;
        s[c] = v ? s[c] * sl2 : -INFINITY;
        mt = fmaxf(mt, s[c]);
      }
      const bool raise = mt > m + kMLazy;
      const float mn = raise ? mt : m;
      const float alpha = (m == -INFINITY || !raise) ? 1.f : exp2f(m - mn);
      if (j > 0 && __any_sync(0xffffffffu, raise && m != -INFINITY)) {
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
      if (j >= 2 && !mbar_wait(&p_done[pb], (uint32_t)((j >> 1) & 1) ^ 1u)) {
        ok = false;
        break;
      }
      float ls = 0.f;
      const float msafe = mn == -INFINITY ? 0.f : mn;
      uint8_t* pbuf = sP + pb * kMPBuf;
#pragma unroll
      for (int c = 0; c < kMN; c += 8) {
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
    // ---- normalised output of this CTA's 256 dims ----
    __nv_bfloat16* orow = a.out + (long)row * kMD + half * 256;
    const bool have = ok && ntiles > 0 && mbar_wait(&p_done[(ntiles - 1) & 1], (uint32_t)((ntiles - 1) >> 1) & 1u);
    if (!ok) {
      set_status(status, kStatusMbarTimeout);
      *abort_flag = 1;
    }
    if (have) tc_fence_after();
    const float inv = (have && l > 0.f) ? 1.f / l : 0.f;
#pragma unroll 1
    for (int c = 0; c < 256; c += 32) {
      float v[32];
      if (have) {
        tmem_ld32(tmem + lane_base + 256 + c, v);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 32; e += 8) {
        alignas(16) __nv_bfloat16 o8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) o8[u] = __float2bfloat16(v[e + u] * inv);
        *reinterpret_cast<uint4*>(orow + c + e) = *reinterpret_cast<uint4*>(o8);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool mqa_prefill_tc_supported(const MqaArgs& a, int kv_rows_per_seq) {
  const int tpt = a.H > 0 ? kMM / a.H : 0;
  return a.D == kMD && a.H > 0 && a.H <= kMM && kMM % a.H == 0 && ((long)a.rows * a.H) % kMM == 0 &&
         a.q_per_seq % tpt == 0 && kv_rows_per_seq % kMN == 0 && a.kv_seq_stride == (long)kv_rows_per_seq * kMD;
}

void mqa_prefill_tc(const MqaArgs& a, int kv_rows_per_seq, long kv_total_rows, int* status, cudaStream_t st) {
  static bool set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    BWN_CUDA_CHECK(cudaFuncSetAttribute(mqa_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMSmem));
    set[dev & 63] = true;
  }
  CUtensorMap tq, tk;
  make_tmap_2d_bf16(&tq, a.q, (long)a.rows * a.H, kMD, kMD, 128, 64);
  make_tmap_2d_bf16(&tk, a.kv, kv_total_rows, kMD, kMD, kMN, 64);
  const int tiles = (int)(((long)a.rows * a.H) / kMM);
  launch_k(mqa_prefill_tc_kernel, dim3(tiles, 2), dim3(kMThreads), kMSmem, st, tq, tk, a, kv_rows_per_seq, status);
}

}  // namespace bwn
