// Decode-sized MoE block (Qwen3.6-35B-A3B: softmax router, top-k, routed SwiGLU
// experts, sigmoid-gated shared expert; the reference's moe_forward / _moe,
// contrib/qwen3.6-35b-a3b/static_decode_35b.py:701-833, 1110-1185) in four
// launches instead of twelve:
//
//  1. moe_route_fused  the router GEMV (and the shared-expert gate row), a
//                      grid barrier, softmax / top-k / renormalisation, the
//                      stable expert-major packing of this rank's (token, slot)
//                      pairs, and the gather of the packed token rows -- one
//                      launch.  The shared expert is packed as one more group
//                      (its rows: the tokens this rank owns), so the grouped
//                      GEMMs run it with the routed experts.
//  2, 3. grouped tcgen05 GEMMs (gate/up with the SwiGLU epilogue, then down;
//                      csrc/kernels/moe.cu) over the packed rows.
//  4. moe_combine_ex   per token: sum of w * expert rows + sigmoid(gate) *
//                      shared row in fp32, rounded to bf16 once, then either
//                      stored (the partial), added to the residual and
//                      RMSNorm(1+w)'d (one GPU), or stored into this rank's
//                      symmetric slot with the completion flag published to
//                      every rank (the fused NVLink reduction follows).
//
// Every CTA of moe_route_fused computes the (tiny) routing itself from the
// logits all CTAs produced, so the packing is identical everywhere and no
// second barrier is needed: each CTA then gathers its share of the rows.  The
// grid is at most one CTA per SM and each CTA starts its dependents only once
// all of them run, so the barrier's CTAs are co-resident; its wait is bounded
// and reports a timeout through the status word.
#include "comm/signal.cuh"
#include "common/host.h"
#include "common/launch.cuh"
#include "common/sm100.cuh"
#include "kernels/moe.h"
#include "kernels/moe_topk.cuh"

// Phase hook of moe_route_fused (empty in the product build; a timing harness
// may define it to record a timestamp per CTA and phase).
#ifndef BWN_ROUTE_PHASE
#define BWN_ROUTE_PHASE(n)
#endif

namespace bwn {

namespace {
constexpr int kRtThreads = 256;
constexpr int kRtWarps = kRtThreads / 32;
constexpr int kRtMaxT = 64;
constexpr int kRtMaxK = 16;
constexpr int kRtMaxPairs = kRtMaxT * kRtMaxK;
constexpr int kRtMaxVec = 16;  // hidden <= 16 * 256

struct RouteSmem {
  float w[kRtMaxPairs];
  int ids[kRtMaxPairs];
  int pos[kRtMaxPairs];
  int src[kRtMaxPairs + kRtMaxT];  // token of each packed row
  unsigned long long msk[kMoeDecodeMaxGroups];  // tokens routed to each local expert (bit t)
  int cnt[kMoeDecodeMaxGroups];
  int off[kMoeDecodeMaxGroups + 1];
  float sg[kRtMaxT];
  int abort;
};

__device__ __forceinline__ float dot8_bf16(const uint4& a, const uint4& b) {
  const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b);
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 x = __bfloat1622float2(a2[e]);
    const float2 y = __bfloat1622float2(b2[e]);
    s = fmaf(x.x, y.x, s);
    s = fmaf(x.y, y.y, s);
  }
  return s;
}

__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
}  // namespace

template <int NV, int EPL>  // NV: 16-byte vectors per lane per hidden row (H = 256 * NV); EPL: experts per lane
__global__ void __launch_bounds__(kRtThreads) moe_route_fused_kernel(MoeRouteFusedArgs a) {
  __shared__ RouteSmem s;
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = a.E + (a.has_sg ? 1 : 0);  // router rows (+ shared gate row)
  const int ntg = (a.T + 7) / 8;
  BWN_ROUTE_PHASE(0);
  // ---- 1. router logits: one warp per (router row, group of 8 tokens) ----
  for (int item = blockIdx.x * kRtWarps + warp; item < rows * ntg; item += gridDim.x * kRtWarps) {
    const int e = item / ntg, tg = item % ntg;
    const uint4* wr = reinterpret_cast<const uint4*>(a.router + (long)e * a.H);
    uint4 wv[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) wv[j] = wr[lane + 32 * j];
    const int t1 = min(a.T, tg * 8 + 8);
    constexpr int TPF = NV <= 8 ? 4 : 2;  // token rows in flight at once (register budget)
    for (int t = tg * 8; t < t1; t += TPF) {
      uint4 xv[TPF][NV];
#pragma unroll
      for (int u = 0; u < TPF; ++u) {
        const uint4* xr = reinterpret_cast<const uint4*>(a.x + (long)min(t + u, t1 - 1) * a.ldx);
#pragma unroll
        for (int j = 0; j < NV; ++j) xv[u][j] = __ldg(xr + lane + 32 * j);
      }
      float acc[TPF];
#pragma unroll
      for (int u = 0; u < TPF; ++u) {
        acc[u] = 0.f;
#pragma unroll
        for (int j = 0; j < NV; ++j) acc[u] += dot8_bf16(wv[j], xv[u][j]);
        acc[u] = warp_sum(acc[u]);
      }
      if (lane == 0) {
#pragma unroll
        for (int u = 0; u < TPF; ++u)
          if (t + u < t1) a.logits[(long)(t + u) * rows + e] = acc[u];
      }
    }
  }
  // ---- 2. grid barrier (count, generation); bounded wait ----
  if (threadIdx.x == 0) s.abort = 0;
  __syncthreads();
  BWN_ROUTE_PHASE(1);
  // arrival count and generation live on separate 128-byte lines, and the
  // waiters back off between polls, so polling never starves the arrivals
  unsigned* const bar_count = a.bar;
  unsigned* const bar_gen = a.bar + 32;
  if (threadIdx.x == 0) {
    const unsigned gen = ld_acquire_gpu_u32(bar_gen);
    __threadfence();
    const unsigned arrived = atomicAdd(bar_count, 1u);
    if (arrived == gridDim.x - 1) {
      atomicExch(bar_count, 0u);
      __threadfence();
      atomicAdd(bar_gen, 1u);
    } else {
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_gpu_u32(bar_gen) == gen) {
        __nanosleep(64);
        if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > a.limit_ns) {
          set_status(a.status, kStatusFlagTimeout);
          s.abort = 1;
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
  BWN_ROUTE_PHASE(2);
  if (s.abort) return;
  // ---- 3. routing (every CTA, identically): softmax -> top-k -> renormalise ----
  const int E = a.E, k = a.k, T = a.T;
  constexpr int NT = EPL <= 8 ? 4 : 2;  // tokens per warp routed together
  for (int t0 = warp; t0 < T; t0 += kRtWarps * NT) {
    const float* l[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int t = t0 + j * kRtWarps;
      l[j] = t < T ? a.logits + (long)t * rows : nullptr;
    }
    float my_w[NT], picked[NT];
    int my_id[NT];
    route_topk_n<EPL, NT>(l, E, k, lane, my_w, my_id, picked);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int t = t0 + j * kRtWarps;
      if (t >= T) continue;
      if (lane < k) {
        s.w[t * k + lane] = a.renorm ? my_w[j] / picked[j] : my_w[j];
        s.ids[t * k + lane] = my_id[j];
      }
      if (lane == 0) s.sg[t] = a.has_sg ? __ldcg(l[j] + E) : 0.f;
    }
  }
  // ---- stable expert-major packing of this rank's pairs (+ the shared group) ----
  // Each token routes to an expert at most once, so a pair's rank inside its
  // expert's group is the number of earlier tokens routed there: one bit per
  // token in the expert's mask, set in parallel, counted with popc.
  const int G = a.E_local + (a.shared_group ? 1 : 0);
  for (int g = threadIdx.x; g < G; g += blockDim.x) s.msk[g] = 0ull;
  __syncthreads();
  const int n = T * k;
  BWN_ROUTE_PHASE(3);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int el = s.ids[i] - a.e0;
    if (el >= 0 && el < a.E_local) atomicOr(&s.msk[el], 1ull << (i / k));
  }
  __syncthreads();
  for (int g = threadIdx.x; g < G; g += blockDim.x)
    s.cnt[g] = g < a.E_local ? __popcll(s.msk[g]) : a.t_hi - a.t_lo;
  __syncthreads();
  // exclusive prefix sum of the group counts: each thread scans a run of
  // consecutive groups, the run totals are scanned by one warp
  {
    constexpr int kRun = (kMoeDecodeMaxGroups + kRtThreads - 1) / kRtThreads;
    const int g0 = threadIdx.x * kRun;
    int run = 0;
#pragma unroll
    for (int u = 0; u < kRun; ++u)
      if (g0 + u < G) run += s.cnt[g0 + u];
    // inclusive scan of the 256 run totals: warp scans, then the 8 warp totals
    int incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int nb = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += nb;
    }
    __shared__ int s_wtot[kRtWarps];
    if (lane == 31) s_wtot[warp] = incl;
    __syncthreads();
    int before = 0;
    for (int w = 0; w < warp; ++w) before += s_wtot[w];
    int o = before + incl - run;  // exclusive start of this thread's run
#pragma unroll
    for (int u = 0; u < kRun; ++u)
      if (g0 + u < G) {
        s.off[g0 + u] = o;
        o += s.cnt[g0 + u];
      }
    if (threadIdx.x == kRtThreads - 1) {
      int tot = 0;
      for (int w = 0; w < kRtWarps; ++w) tot += s_wtot[w];
      s.off[G] = tot;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int el = s.ids[i] - a.e0;
    const int t = i / k;
    int p = -1;
    if (el >= 0 && el < a.E_local) {
      p = s.off[el] + __popcll(s.msk[el] & ((1ull << t) - 1ull));
      s.src[p] = t;
    }
    s.pos[i] = p;
  }
  if (a.shared_group)
    for (int t = a.t_lo + threadIdx.x; t < a.t_hi; t += blockDim.x) s.src[s.off[a.E_local] + t - a.t_lo] = t;
  __syncthreads();
  BWN_ROUTE_PHASE(4);
  // ---- 4. gather this CTA's share of the packed rows; CTA 0 writes the routing ----
  const int total = s.off[G];
  const int hv = a.H / 8;
  for (int r = blockIdx.x; r < total; r += gridDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(a.x + (long)s.src[r] * a.ldx);
    uint4* dst = reinterpret_cast<uint4*>(a.x_perm + (long)r * a.H);
    for (int v = threadIdx.x; v < hv; v += blockDim.x) dst[v] = src[v];
  }
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      a.w[i] = s.w[i];
      a.ids[i] = s.ids[i];
      a.pos_of[i] = s.pos[i];
    }
    for (int g = threadIdx.x; g < G; g += blockDim.x) a.counts[g] = s.off[g + 1] - s.off[g];
    for (int g = threadIdx.x; g <= G; g += blockDim.x) a.offsets[g] = s.off[g];
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
      a.pos_sh[t] = (a.shared_group && t >= a.t_lo && t < a.t_hi) ? s.off[a.E_local] + t - a.t_lo : -1;
      a.sg[t] = s.sg[t];
    }
  }
  __syncthreads();
  BWN_ROUTE_PHASE(5);
}

// One CTA per token.  VPT: 8-column vectors per thread (H <= 256 * 8 * VPT).
template <int VPT>
__global__ void __launch_bounds__(256) moe_combine_ex_kernel(MoeCombineExArgs a) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  __shared__ int s_pos[kRtMaxK + 1];
  __shared__ float s_w[kRtMaxK + 1];
  __shared__ float red[8];
  if (threadIdx.x < a.k) {
    s_pos[threadIdx.x] = a.pos_of[(long)t * a.k + threadIdx.x];
    s_w[threadIdx.x] = a.w[(long)t * a.k + threadIdx.x];
  }
  if (threadIdx.x == 0) {
    const int ps = a.pos_sh ? a.pos_sh[t] : -1;
    s_pos[kRtMaxK] = ps;
    s_w[kRtMaxK] = ps >= 0 ? sigmoid_f(a.sg[t]) : 0.f;
  }
  __syncthreads();
  const float gsep = a.shared_y ? sigmoid_f(a.shared_gate[t]) : 0.f;
  const int nvec = a.H >> 3;
  const bool to_slot = a.mode == kCombineSymm || a.mode == kCombineSymmNorm;
  const int sel = to_slot ? ((*a.sig.sel) & 1) : 0;
  __nv_bfloat16* slot = to_slot ? a.symm_base + (long)sel * a.sig.buf_stride : nullptr;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi >= nvec) continue;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    auto add_row = [&](const __nv_bfloat16* rowp, float wt) {
      const uint4 u = reinterpret_cast<const uint4*>(rowp)[vi];
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h2[e]);
        acc[2 * e] += wt * f.x;
        acc[2 * e + 1] += wt * f.y;
      }
    };
    for (int sl = 0; sl < a.k; ++sl) {
      const int r = s_pos[sl];
      if (r >= 0) add_row(a.y + (long)r * a.H, s_w[sl]);
    }
    if (s_pos[kRtMaxK] >= 0) add_row(a.y + (long)s_pos[kRtMaxK] * a.H, s_w[kRtMaxK]);
    if (a.shared_y) add_row(a.shared_y + (long)t * a.ld_shared, gsep);
    alignas(16) __nv_bfloat16 pb[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) pb[e] = __float2bfloat16(acc[e]);
    if (a.mode == kCombinePartial) {
      reinterpret_cast<uint4*>(a.out + (long)t * a.ldo)[vi] = *reinterpret_cast<uint4*>(pb);
    } else if (to_slot) {
      reinterpret_cast<uint4*>(slot + (long)t * a.H)[vi] = *reinterpret_cast<uint4*>(pb);
    } else {  // residual add (bf16, as the unfused add_rms_norm) then RMSNorm(1+w)
      const uint4 rr = reinterpret_cast<const uint4*>(a.resid + (long)t * a.ldr)[vi];
      const __nv_bfloat16* rh = reinterpret_cast<const __nv_bfloat16*>(&rr);
      alignas(16) __nv_bfloat16 nr[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        nr[e] = __float2bfloat16(__bfloat162float(pb[e]) + __bfloat162float(rh[e]));
        v[i][e] = __bfloat162float(nr[e]);
        ss += v[i][e] * v[i][e];
      }
      reinterpret_cast<uint4*>(a.resid + (long)t * a.ldr)[vi] = *reinterpret_cast<uint4*>(nr);
    }
  }
  if (to_slot) {
    __shared__ unsigned s_epoch;
    __syncthreads();  // the CTA's slot stores precede thread 0's system-scope fence
    if (threadIdx.x == 0) {
      s_epoch = (unsigned)(*a.sig.epoch) + 1u;  // the epoch this launch publishes (read before the ticket)
      signal_done(a.sig);
    }
    if (a.mode == kCombineSymm) return;
    // ---- symm-norm: wait for every rank, then this token's row of the sum ----
    __shared__ int s_ok;
    if (threadIdx.x == 0) s_ok = 1;
    __syncthreads();
    if ((int)threadIdx.x < a.sig.world) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      while ((int)(ld_acquire_sys(a.flags + threadIdx.x) - s_epoch) < 0) {
        if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > a.limit_ns) {
          set_status(a.status, kStatusPeerTimeout);
          s_ok = 0;
          break;
        }
      }
    }
    __syncthreads();
    if (s_ok) {  // a peer that never signalled: nothing is read or written
      const __nv_bfloat16* buf = a.mc_base + (long)sel * a.sig.buf_stride + (long)t * a.H;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = threadIdx.x + i * blockDim.x;
        if (vi < nvec) mc_ld_reduce_bf16x8(buf + vi * 8, v[i]);
      }
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = threadIdx.x + i * blockDim.x;
        if (vi >= nvec) continue;
        const uint4 rr = reinterpret_cast<const uint4*>(a.resid + (long)t * a.ldr)[vi];
        const __nv_bfloat16* rh = reinterpret_cast<const __nv_bfloat16*>(&rr);
        alignas(16) __nv_bfloat16 nr[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {  // the reduced partial rounded to bf16, as the unfused all-reduce output
          const float pr = __bfloat162float(__float2bfloat16(v[i][e]));
          nr[e] = __float2bfloat16(pr + __bfloat162float(rh[e]));
          v[i][e] = __bfloat162float(nr[e]);
          ss += v[i][e] * v[i][e];
        }
        reinterpret_cast<uint4*>(a.resid + (long)t * a.ldr)[vi] = *reinterpret_cast<uint4*>(nr);
      }
    }
  } else if (a.mode != kCombineAddNorm) {
    return;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = rsqrtf(tot / a.H + a.eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi >= nvec) continue;
    alignas(16) __nv_bfloat16 o[8];
    const float4 w0 = reinterpret_cast<const float4*>(a.norm_w)[2 * vi];
    const float4 w1 = reinterpret_cast<const float4*>(a.norm_w)[2 * vi + 1];
    const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __float2bfloat16(v[i][e] * inv * (1.f + ww[e]));
    reinterpret_cast<uint4*>(a.out + (long)t * a.ldo)[vi] = *reinterpret_cast<uint4*>(o);
  }
  if (a.mode == kCombineSymmNorm) {  // flip the slot selector once every CTA has read it
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const int tk = atomicAdd(a.sel_rw + 1, 1);
      if (tk == (int)gridDim.x - 1) {
        a.sel_rw[1] = 0;
        a.sel_rw[0] = a.sel_rw[0] + 1;
      }
    }
  }
}

int moe_route_fused_grid(int T, int E, bool has_sg) {
  const int items = (E + (has_sg ? 1 : 0)) * ((T + 7) / 8);
  int grid = (items + kRtWarps - 1) / kRtWarps;
  return std::max(1, std::min(grid, num_sms()));
}

template <int EPL>
static void route_launch(const MoeRouteFusedArgs& a, dim3 grid, cudaStream_t st) {
  switch (a.H / 256) {
    case 1: launch_k(moe_route_fused_kernel<1, EPL>, grid, dim3(kRtThreads), 0, st, a); break;
    case 2: launch_k(moe_route_fused_kernel<2, EPL>, grid, dim3(kRtThreads), 0, st, a); break;
    case 4: launch_k(moe_route_fused_kernel<4, EPL>, grid, dim3(kRtThreads), 0, st, a); break;
    case 8: launch_k(moe_route_fused_kernel<8, EPL>, grid, dim3(kRtThreads), 0, st, a); break;
    case 16: launch_k(moe_route_fused_kernel<16, EPL>, grid, dim3(kRtThreads), 0, st, a); break;
    default: BWN_FAIL("moe_route_fused: hidden %d (256, 512, 1024, 2048 or 4096)", a.H);
  }
}

void moe_route_fused(const MoeRouteFusedArgs& a, cudaStream_t st) {
  BWN_CHECK(a.T >= 1 && a.T <= kRtMaxT, "moe_route_fused: 1..%d tokens", kRtMaxT);
  BWN_CHECK(a.k >= 1 && a.k <= kRtMaxK && a.k <= a.E && a.E <= 512, "moe_route_fused: k <= 16, E <= 512");
  BWN_CHECK(a.H % 256 == 0 && a.H / 256 <= kRtMaxVec && a.ldx % 8 == 0, "moe_route_fused: H multiple of 256, <= 4096");
  BWN_CHECK(a.E_local + (a.shared_group ? 1 : 0) <= kMoeDecodeMaxGroups, "moe_route_fused: too many groups");
  BWN_CHECK(!a.shared_group || (0 <= a.t_lo && a.t_lo <= a.t_hi && a.t_hi <= a.T), "moe_route_fused: token range");
  const dim3 grid(moe_route_fused_grid(a.T, a.E, a.has_sg));
  const int epl = (a.E + 31) / 32;
  switch (epl <= 1 ? 1 : epl <= 2 ? 2 : epl <= 4 ? 4 : epl <= 8 ? 8 : 16) {
    case 1: route_launch<1>(a, grid, st); break;
    case 2: route_launch<2>(a, grid, st); break;
    case 4: route_launch<4>(a, grid, st); break;
    case 8: route_launch<8>(a, grid, st); break;
    default: route_launch<16>(a, grid, st); break;
  }
}

void moe_combine_ex(const MoeCombineExArgs& a, cudaStream_t st) {
  if (a.T == 0) return;
  BWN_CHECK(a.H % 8 == 0 && a.k <= kRtMaxK, "moe_combine_ex: H multiple of 8, k <= 16");
  BWN_CHECK(a.mode != kCombinePartial || a.ldo % 8 == 0, "moe_combine_ex: 16-byte aligned output rows");
  BWN_CHECK((a.mode != kCombineAddNorm && a.mode != kCombineSymmNorm) || (a.ldr % 8 == 0 && a.ldo % 8 == 0),
            "moe_combine_ex: aligned rows");
  BWN_CHECK(a.mode != kCombineSymmNorm || (a.mc_base && a.flags && a.sel_rw && a.resid && a.norm_w && a.out),
            "moe_combine_ex: symm-norm needs the reduction tail");
  BWN_CHECK(!a.shared_y || a.ld_shared % 8 == 0, "moe_combine_ex: aligned shared rows");
  const int vpt = (a.H / 8 + 255) / 256;
  switch (vpt) {
    case 1: launch_k(moe_combine_ex_kernel<1>, dim3(a.T), dim3(256), 0, st, a); break;
    case 2: launch_k(moe_combine_ex_kernel<2>, dim3(a.T), dim3(256), 0, st, a); break;
    case 3: launch_k(moe_combine_ex_kernel<3>, dim3(a.T), dim3(256), 0, st, a); break;
    case 4: launch_k(moe_combine_ex_kernel<4>, dim3(a.T), dim3(256), 0, st, a); break;
    default: BWN_FAIL("moe_combine_ex: hidden %d too wide", a.H);
  }
}

}  // namespace bwn
