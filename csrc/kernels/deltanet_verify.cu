// Gated-DeltaNet multi-token verify for speculative decoding, with deferred
// commit.  A verify step feeds N tokens per sequence (the last accepted token
// plus N-1 drafts); only the accepted prefix of them may reach the recurrent
// state.  The reference keeps the state after every verify token and restores
// the accepted one (contrib/qwen3.6-27b/kernels/tests/
// test_deltanet_spec_verify_rollback.py:1-30), which writes N states per step.
//
// Here the state in memory is always the COMMITTED state: this kernel
//   1. commits the tokens the previous step accepted (`pending`, their raw
//      qkv/a/b rows kept in a parity-indexed stash) -- conv + delta rule
//      applied to the state held in registers, then written back once;
//   2. runs the N new tokens on a register copy of that state, producing their
//      outputs (RMSNormGated) without writing any state;
//   3. stashes the N new raw rows for the next step's commit.
// State traffic is one read and one write per step, as for a single-token
// decode, whatever N and the acceptance.  The conv history is read through a
// window gathered at the start: ring rows of positions p-a-3..p-a-1, the a
// pending rows, the N new rows.  Ring slots are position-addressed with
// R >= N+3, so the rows this launch writes (positions max(p-3, p-a)..p-1)
// never alias a row another CTA of the launch still reads (positions
// p-a-3..p-a-1).
//
// Thread mapping as in deltanet_decode.cu: a cluster of 4 CTAs per
// (sequence, V-head), each owning 32 state columns in registers.
#include <cooperative_groups.h>

#include "common/host.h"
#include "common/launch.cuh"
#include "common/sm100.cuh"
#include "kernels/launch.h"

namespace cg = cooperative_groups;

namespace bwn {

namespace {
constexpr int kVDk = 128, kVDv = 128, kVNJ = 4, kVCols = 32;
constexpr int kVW = 3 + 2 * kDnVerifyMaxTok;  // window rows

struct VShared {
  float wq[kVW][kVDk], wk[kVW][kVDk], wv[kVW][kVCols];
  float s_q[kVDk], s_k[kVDk], s_v[kVCols], s_delta[kVCols];
  float s_red[4][2 * kVCols];
  float s_red3[4][3];
  float s_scal[8];
  float o_buf[kDnVerifyMaxTok][kVCols];
  float ss_buf[kDnVerifyMaxTok];
  float ga[2 * kDnVerifyMaxTok], gb[2 * kDnVerifyMaxTok];
};

// One token through conv + norms + gates + delta rule on the state `st`
// (rows warp*32.., column = lane).  Window row r holds this token's input.
template <bool kOut>
__device__ __forceinline__ void dn_token(VShared& s, float (&st)[32], int r, float ga, float gb, const float4& cq,
                                         const float4& ck, const float4& cv, float Alog, float dtb, float l2_eps,
                                         int oi) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float kx = silu_f(ck.x * s.wk[r - 3][t] + ck.y * s.wk[r - 2][t] + ck.z * s.wk[r - 1][t] + ck.w * s.wk[r][t]);
  const float qx =
      kOut ? silu_f(cq.x * s.wq[r - 3][t] + cq.y * s.wq[r - 2][t] + cq.z * s.wq[r - 1][t] + cq.w * s.wq[r][t]) : 0.f;
  const float vx = t < kVCols ? silu_f(cv.x * s.wv[r - 3][t] + cv.y * s.wv[r - 2][t] + cv.z * s.wv[r - 1][t] +
                                       cv.w * s.wv[r][t])
                              : 0.f;
  const float sq = warp_sum(qx * qx), sk = warp_sum(kx * kx), skq = warp_sum(qx * kx);
  if (lane == 0) {
    s.s_red3[warp][0] = sq;
    s.s_red3[warp][1] = sk;
    s.s_red3[warp][2] = skq;
  }
  __syncthreads();
  if (t == 0) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f;
    for (int w = 0; w < 4; ++w) {
      a0 += s.s_red3[w][0];
      a1 += s.s_red3[w][1];
      a2 += s.s_red3[w][2];
    }
    const float nq = fmaxf(sqrtf(a0), l2_eps), nk = fmaxf(sqrtf(a1), l2_eps);
    const float qs = rsqrtf((float)kVDk);
    s.s_scal[0] = qs / nq;
    s.s_scal[1] = 1.f / nk;
    s.s_scal[2] = a2 / (nq * nk) * qs;
    const float g = -__expf(Alog) * softplus_f(ga + dtb);
    s.s_scal[3] = __expf(g);
    s.s_scal[4] = sigmoid_f(gb);
  }
  __syncthreads();
  s.s_q[t] = qx * s.s_scal[0];
  s.s_k[t] = kx * s.s_scal[1];
  if (t < kVCols) s.s_v[t] = vx;
  __syncthreads();
  float pk = 0.f, pq = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    pk += st[i] * s.s_k[warp * 32 + i];
    if (kOut) pq += st[i] * s.s_q[warp * 32 + i];
  }
  s.s_red[warp][lane] = pk;
  s.s_red[warp][kVCols + lane] = pq;
  __syncthreads();
  const float eg = s.s_scal[3], beta = s.s_scal[4], kq = s.s_scal[2];
  if (warp == 0) {
    float tk = 0.f, tq = 0.f;
    for (int w = 0; w < 4; ++w) {
      tk += s.s_red[w][lane];
      tq += s.s_red[w][kVCols + lane];
    }
    const float delta = beta * (s.s_v[lane] - eg * tk);
    s.s_delta[lane] = delta;
    if (kOut) {
      const float o = eg * tq + delta * kq;
      s.o_buf[oi][lane] = o;
      const float ss = warp_sum(o * o);
      if (lane == 0) s.ss_buf[oi] = ss;
    }
  }
  __syncthreads();
  const float delta = s.s_delta[lane];
#pragma unroll
  for (int i = 0; i < 32; ++i) st[i] = eg * st[i] + s.s_k[warp * 32 + i] * delta;
}
}  // namespace

template <typename StateT>
__global__ void __cluster_dims__(kVNJ, 1, 1) __launch_bounds__(128) deltanet_verify_kernel(DnVerifyArgs p) {
  pdl_trigger();
  pdl_wait();
  __shared__ VShared s;
  cg::cluster_group cluster = cg::this_cluster();
  const int jb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int rep = p.v_heads / p.k_heads, kh = h / rep;
  const int KD = p.k_heads * kVDk, C = 2 * KD + p.v_heads * kVDv, VH = p.v_heads;
  const int N = p.n_tok;
  const int pos = p.positions[b];
  const bool active = pos >= 0;
  int a = active ? p.pending[b] : 0;
  if (a < 0 || a > p.stash_n) {
    if (t == 0) set_status(p.status, kStatusBadArg);
    a = 0;
  }
  const int par = (*p.vstep) & 1;
  const int rm = p.ring_slots - 1;
  __nv_bfloat16* ring = p.conv_ring + (long)b * p.ring_slots * C;
  const int qc = kh * kVDk + t, kc = KD + kh * kVDk + t, vc = 2 * KD + h * kVDv + jb * kVCols + t;
  const int SN = p.stash_n;
  auto stash_row = [&](int parity, int i) { return p.stash_qkv + (((long)parity * p.batch + b) * SN + i) * C; };

  // ---- gather the conv window and the gates ----
  const int W = 3 + a + N;
  for (int r = 0; r < W; ++r) {
    const int P = pos - a - 3 + r;
    const __nv_bfloat16* src = nullptr;
    if (r < 3) {
      if (P >= 0) src = ring + (long)(P & rm) * C;
    } else if (r < 3 + a) {
      src = stash_row(par, r - 3);
    } else {
      src = p.qkv + ((long)b * N + (r - 3 - a)) * p.qkv_row;
    }
    s.wq[r][t] = (active && src) ? __bfloat162float(src[qc]) : 0.f;
    s.wk[r][t] = (active && src) ? __bfloat162float(src[kc]) : 0.f;
    if (t < kVCols) s.wv[r][t] = (active && src) ? __bfloat162float(src[vc]) : 0.f;
  }
  if (t < a) {
    const __nv_bfloat16* g = p.stash_ab + (((long)par * p.batch + b) * SN + t) * 2 * VH;
    s.ga[t] = __bfloat162float(g[h]);
    s.gb[t] = __bfloat162float(g[VH + h]);
  } else if (t < a + N) {
    const long row = (long)b * N + (t - a);
    s.ga[t] = __bfloat162float(p.a[row * p.ab_row + h]);
    s.gb[t] = __bfloat162float(p.b[row * p.ab_row + h]);
  }
  __syncthreads();
  const float4 cq = *reinterpret_cast<const float4*>(p.conv_w + (long)qc * 4);
  const float4 ck = *reinterpret_cast<const float4*>(p.conv_w + (long)kc * 4);
  const float4 cv = t < kVCols ? *reinterpret_cast<const float4*>(p.conv_w + (long)vc * 4) : make_float4(0, 0, 0, 0);
  const float Alog = p.A_log[h], dtb = p.dt_bias[h];

  StateT* S = reinterpret_cast<StateT*>(p.state) + (((long)b * VH + h) * kVDk) * kVDv + jb * kVCols + lane;
  float st[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) st[i] = active ? to_f(S[(long)(warp * 32 + i) * kVDv]) : 0.f;

  // ---- 1. commit the previous step's accepted tokens ----
  for (int j = 0; j < a; ++j) dn_token<false>(s, st, 3 + j, s.ga[j], s.gb[j], cq, ck, cv, Alog, dtb, p.l2_eps, 0);
  if (active && a > 0) {
#pragma unroll
    for (int i = 0; i < 32; ++i) S[(long)(warp * 32 + i) * kVDv] = from_f<StateT>(st[i]);
    // ring rows of the newly committed positions still needed as history
    const bool qk_writer = jb == 0 && (h % rep) == 0;
    for (int j = max(0, a - 3); j < a; ++j) {
      __nv_bfloat16* dst = ring + (long)((pos - a + j) & rm) * C;
      if (qk_writer) {
        dst[qc] = __float2bfloat16(s.wq[3 + j][t]);
        dst[kc] = __float2bfloat16(s.wk[3 + j][t]);
      }
      if (t < kVCols) dst[vc] = __float2bfloat16(s.wv[3 + j][t]);
    }
  }

  // ---- 2. the new tokens on a copy of the committed state ----
  for (int i = 0; i < N; ++i)
    dn_token<true>(s, st, 3 + a + i, s.ga[a + i], s.gb[a + i], cq, ck, cv, Alog, dtb, p.l2_eps, i);

  // ---- 3. stash the new raw rows for the next step's commit ----
  if (active) {
    const bool qk_writer = jb == 0 && (h % rep) == 0;
    for (int i = 0; i < N; ++i) {
      __nv_bfloat16* dst = stash_row(par ^ 1, i);
      if (qk_writer) {
        dst[qc] = __float2bfloat16(s.wq[3 + a + i][t]);
        dst[kc] = __float2bfloat16(s.wk[3 + a + i][t]);
      }
      if (t < kVCols) dst[vc] = __float2bfloat16(s.wv[3 + a + i][t]);
    }
    if (jb == 0 && t < N) {
      __nv_bfloat16* g = p.stash_ab + (((long)(par ^ 1) * p.batch + b) * SN + t) * 2 * VH;
      g[h] = __float2bfloat16(s.ga[a + t]);
      g[VH + h] = __float2bfloat16(s.gb[a + t]);
    }
  }

  // ---- RMSNormGated of the N outputs across the cluster's column blocks ----
  cluster.sync();
  if (warp == 0) {
    const int col = h * kVDv + jb * kVCols + lane;
    for (int i = 0; i < N; ++i) {
      float tot = 0.f;
      for (int r = 0; r < kVNJ; ++r) tot += cluster.map_shared_rank(s.ss_buf, r)[i];
      const float inv = rsqrtf(tot / (float)kVDv + p.norm_eps);
      const long row = (long)b * N + i;
      const float z = __bfloat162float(p.z[row * p.z_row + col]);
      const float y = active ? s.o_buf[i][lane] * inv * p.norm_w[jb * kVCols + lane] * silu_f(z) : 0.f;
      p.out[row * p.out_row + col] = __float2bfloat16(y);
    }
  }
  cluster.sync();
}

void deltanet_verify(const DnVerifyArgs& p, cudaStream_t stream) {
  BWN_CHECK(p.n_tok >= 0 && p.n_tok <= kDnVerifyMaxTok, "deltanet_verify: n_tok must be in [0, %d]", kDnVerifyMaxTok);
  BWN_CHECK(p.stash_n >= p.n_tok && p.stash_n <= kDnVerifyMaxTok, "deltanet_verify: stash holds %d tokens", p.stash_n);
  BWN_CHECK(p.ring_slots >= p.stash_n + 3 && (p.ring_slots & (p.ring_slots - 1)) == 0,
            "deltanet_verify: the conv ring needs a power-of-two slot count >= n_tok + 3");
  dim3 grid(kVNJ, p.v_heads, p.batch);
  if (p.state_bf16) {
    launch_k(deltanet_verify_kernel<__nv_bfloat16>, grid, dim3(128), 0, stream, p);
  } else {
    launch_k(deltanet_verify_kernel<float>, grid, dim3(128), 0, stream, p);
  }
}

}  // namespace bwn
