// Mixture-of-experts kernels (Qwen3.6-35B-A3B routed experts; DeepSeek V4 MoE):
//
//  * moe_topk_softmax  one warp per token: softmax over E logits, top-k,
//                      optional renormalisation (HF Qwen3_5MoeTopKRouter; the
//                      reference _moe_routing, static_decode_35b.py:1187-1194).
//  * moe_topk_deepseek sqrt(softplus) / sigmoid scores, bias for selection only,
//                      renormalise x route_scale (run_deepseek_v4_tp.py:397-428).
//  * moe_route_count / moe_route_place
//                      stable expert-major packing of the (token, slot) pairs
//                      routed to this rank's experts: one CTA per local expert,
//                      ballot compaction in token order, so the layout is
//                      deterministic (the reference's route packer,
//                      moe_cte_adapter.py:9-71, kernels/moe_cte_35b.py:111).
//  * moe_gather        x rows into expert-major order.
//  * grouped GEMM      tcgen05, swap-AB: each unit is (expert, 128 weight rows,
//                      BN token rows of that expert); units past an expert's row
//                      count are skipped by all warp roles, so one launch shape
//                      serves every routing (CUDA-graph safe).
//  * moe_combine       out[t] = sum_slot w * y[pos(t, slot)] (+ gated shared
//                      expert), fp32 accumulation, this rank's partial sum.
#include "common/host.h"
#include "common/launch.cuh"
#include "common/sm100.cuh"
#include "kernels/moe.h"
#include "kernels/grouped_units.cuh"
#include "kernels/moe_topk.cuh"

namespace bwn {

// =============================================================================
// routers
// =============================================================================
template <int EPL>  // experts per lane (E / 32)
__global__ void moe_topk_softmax_kernel(const float* __restrict__ logits, int T, int E, int k, bool renorm,
                                        float* __restrict__ w_out, int* __restrict__ id_out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* l = logits + (long)warp * E;
  float my_w;
  int my_id;
  const float picked = route_topk<EPL>(l, E, k, lane, my_w, my_id);
  if (lane < k) {
    w_out[(long)warp * k + lane] = renorm ? my_w / picked : my_w;
    id_out[(long)warp * k + lane] = my_id;
  }
}

template <int EPL>
__global__ void moe_topk_deepseek_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int T,
                                         int E, int k, int sqrt_softplus, float route_scale, float* __restrict__ w_out,
                                         int* __restrict__ id_out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* l = logits + (long)warp * E;
  float sc[EPL], sel[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    if (e < E) {
      const float x = l[e];
      sc[i] = sqrt_softplus ? sqrtf(softplus_f(x)) : sigmoid_f(x);
      sel[i] = sc[i] + (bias ? bias[e] : 0.f);
    } else {
      sc[i] = 0.f;
      sel[i] = -INFINITY;
    }
  }
  float tot = 0.f, my_w = 0.f;
  int my_id = -1;
  for (int s = 0; s < k; ++s) {
    float best = -INFINITY, bsc = 0.f;
    int bid = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = i * 32 + lane;
      if (e < E && (sel[i] > best || (sel[i] == best && e < bid))) {
        best = sel[i];
        bid = e;
        bsc = sc[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bid, o);
      const float os = __shfl_xor_sync(0xffffffffu, bsc, o);
      if (ob > best || (ob == best && oi < bid)) {
        best = ob;
        bid = oi;
        bsc = os;
      }
    }
    tot += bsc;
    if (lane == s) {
      my_w = bsc;
      my_id = bid;
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (i * 32 + lane == bid) sel[i] = -INFINITY;
  }
  if (lane < k) {
    w_out[(long)warp * k + lane] = my_w / tot * route_scale;
    id_out[(long)warp * k + lane] = my_id;
  }
}

void moe_topk(const MoeTopkArgs& a, cudaStream_t st) {
  if (a.T == 0) return;
  BWN_CHECK(a.E <= 512 && a.k <= 32 && a.k <= a.E, "moe_topk: E <= 512, k <= 32");
  const int threads = 256, blocks = (a.T * 32 + threads - 1) / threads;
  const int epl = (a.E + 31) / 32;
#define BWN_TOPK(EPLV)                                                                                       \
  if (epl <= EPLV) {                                                                                         \
    if (a.deepseek)                                                                                          \
      moe_topk_deepseek_kernel<EPLV><<<blocks, threads, 0, st>>>(a.logits, a.bias, a.T, a.E, a.k,            \
                                                                 a.sqrt_softplus, a.route_scale, a.w, a.ids); \
    else                                                                                                     \
      moe_topk_softmax_kernel<EPLV><<<blocks, threads, 0, st>>>(a.logits, a.T, a.E, a.k, a.renorm, a.w, a.ids); \
    BWN_CUDA_CHECK(cudaGetLastError());                                                                      \
    return;                                                                                                  \
  }
  BWN_TOPK(1)
  BWN_TOPK(2)
  BWN_TOPK(4)
  BWN_TOPK(8)
  BWN_TOPK(16)
#undef BWN_TOPK
}

// =============================================================================
// route packing (stable, expert-major)
// =============================================================================
__global__ void __launch_bounds__(256) moe_route_count_kernel(const int* __restrict__ ids, int n, int e0,
                                                              int* __restrict__ counts) {
  const int e = e0 + blockIdx.x;
  int c = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) c += ids[i] == e;
  c = __reduce_add_sync(0xffffffffu, c);
  __shared__ int red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < 8; ++w) t += red[w];
    counts[blockIdx.x] = t;
  }
}

// pos_of[i] = packed row of pair i (or -1 when its expert is not local);
// row_src[r] = pair index feeding packed row r; offsets[e] = first row of expert e.
__global__ void __launch_bounds__(256) moe_route_place_kernel(const int* __restrict__ ids, int n, int e0, int E_local,
                                                              const int* __restrict__ counts, int* __restrict__ offsets,
                                                              int* __restrict__ pos_of, int* __restrict__ row_src) {
  const int el = blockIdx.x, e = e0 + el;
  __shared__ int s_base;
  __shared__ int s_warp[8];
  if (threadIdx.x == 0) {
    int o = 0;
    for (int j = 0; j < el; ++j) o += counts[j];
    s_base = o;
    offsets[el] = o;
    if (el == E_local - 1) offsets[E_local] = o + counts[el];
  }
  __syncthreads();
  int base = s_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i0 = 0; i0 < n; i0 += blockDim.x) {
    const int i = i0 + threadIdx.x;
    const int id = i < n ? ids[i] : -1;
    const bool hit = id == e;
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) s_warp[warp] = __popc(m);
    __syncthreads();
    int before = 0, tot = 0;
    for (int w = 0; w < 8; ++w) {
      if (w < warp) before += s_warp[w];
      tot += s_warp[w];
    }
    if (hit) {
      const int r = base + before + __popc(m & ((1u << lane) - 1));
      pos_of[i] = r;
      row_src[r] = i;
    } else if (i < n && (id < e0 || id >= e0 + E_local) && el == 0) {
      pos_of[i] = -1;
    }
    base += tot;
    __syncthreads();
  }
}

__global__ void moe_gather_kernel(const __nv_bfloat16* __restrict__ x, long ldx, const int* __restrict__ row_src,
                                  const int* __restrict__ offsets, int E_local, int k, int H,
                                  __nv_bfloat16* __restrict__ out) {
  const int r = blockIdx.x;
  if (r >= offsets[E_local]) return;
  const int tok = row_src[r] / k;
  const uint4* src = reinterpret_cast<const uint4*>(x + (long)tok * ldx);
  uint4* dst = reinterpret_cast<uint4*>(out + (long)r * H);
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) dst[v] = src[v];
}

void moe_route(const MoeRouteArgs& a, cudaStream_t st) {
  const int n = a.T * a.k;
  if (n == 0) return;
  moe_route_count_kernel<<<a.E_local, 256, 0, st>>>(a.ids, n, a.e0, a.counts);
  BWN_CUDA_CHECK(cudaGetLastError());
  moe_route_place_kernel<<<a.E_local, 256, 0, st>>>(a.ids, n, a.e0, a.E_local, a.counts, a.offsets, a.pos_of,
                                                    a.row_src);
  BWN_CUDA_CHECK(cudaGetLastError());
  if (a.x) {
    BWN_CHECK(a.H % 8 == 0 && a.ldx % 8 == 0, "moe_gather: H multiple of 8");
    moe_gather_kernel<<<n, 128, 0, st>>>(a.x, a.ldx, a.row_src, a.offsets, a.E_local, a.k, a.H, a.x_perm);
    BWN_CUDA_CHECK(cudaGetLastError());
  }
}

// =============================================================================
// combine
// =============================================================================
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, const float* __restrict__ w,
                                   const int* __restrict__ pos_of, int k, int H,
                                   const __nv_bfloat16* __restrict__ shared_y, long ld_shared,
                                   const float* __restrict__ shared_gate, __nv_bfloat16* __restrict__ out, long ldo) {
  const int t = blockIdx.x;
  __shared__ int s_pos[32];
  __shared__ float s_w[32];
  if (threadIdx.x < k) {
    s_pos[threadIdx.x] = pos_of[(long)t * k + threadIdx.x];
    s_w[threadIdx.x] = w[(long)t * k + threadIdx.x];
  }
  __syncthreads();
  const float sg = shared_gate ? sigmoid_f(shared_gate[t]) : 0.f;
  for (int c = threadIdx.x * 2; c < H; c += blockDim.x * 2) {
    float a0 = 0.f, a1 = 0.f;
    for (int s = 0; s < k; ++s) {
      const int r = s_pos[s];
      if (r < 0) continue;
      const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(y + (long)r * H + c));
      a0 += s_w[s] * v.x;
      a1 += s_w[s] * v.y;
    }
    if (shared_y) {
      const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(shared_y + (long)t * ld_shared + c));
      a0 += sg * v.x;
      a1 += sg * v.y;
    }
    *reinterpret_cast<__nv_bfloat162*>(out + (long)t * ldo + c) = __floats2bfloat162_rn(a0, a1);
  }
}

void moe_combine(const MoeCombineArgs& a, cudaStream_t st) {
  if (a.T == 0) return;
  BWN_CHECK(a.H % 2 == 0 && a.k <= 32, "moe_combine: H even, k <= 32");
  moe_combine_kernel<<<a.T, 256, 0, st>>>(a.y, a.w, a.pos_of, a.k, a.H, a.shared_y, a.ld_shared, a.shared_gate,
                                          a.out, a.ldo);
  BWN_CUDA_CHECK(cudaGetLastError());
}

// =============================================================================
// grouped GEMM (swap-AB):  for expert e and its rows [off_e, off_e + n_e):
//   out[off_e + j, :] = epi( W_e[N_out, K] . X[off_e + j, :]^T )
// =============================================================================
constexpr int kGBM = 128, kGBK = 64, kGThreadsG = 192;

template <int BN>
struct GCfg {
  static constexpr int kA = kGBM * kGBK * 2, kB = BN * kGBK * 2, kStage = kA + kB;
  static constexpr int kStages = (200 * 1024 / kStage) > 10 ? 10 : (200 * 1024 / kStage);
  static constexpr int kTmem = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kSmem = kStages * kStage + 1024 + 256;
};

template <int BN, bool SWIGLU>
__global__ void __launch_bounds__(kGThreadsG, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                        GroupedArgs a) {
  using C = GCfg<BN>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * C::kA;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S * C::kStage);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* tfull = empty_bar + S;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmem);
    tmem_relinquish();
  }
  __shared__ GUnits gu;
  // the row counts and packed rows come from the previous kernel (PDL)
  pdl_trigger();
  pdl_wait();
  for (int e = threadIdx.x; e < a.groups; e += blockDim.x) {
    const int c = min(a.counts[e], a.max_tiles_n * BN);
    gu.cnt[e] = c;
    gu.off[e] = a.offsets[e];
    gu.pref[e + 1] = a.tiles_m * ((c + BN - 1) / BN);
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    gu.pref[0] = 0;
    for (int e = 0; e < a.groups; ++e) gu.pref[e + 1] += gu.pref[e];
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int units = gu.pref[a.groups];
  const int num_kb = (a.K + kGBK - 1) / kGBK;
  if (warp == 0) {
    if (elect_one()) {
      const uint64_t polA = l2_policy_evict_first();
      const uint64_t polB = l2_policy_evict_last();
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_mask = 0, issued_ph = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int e, tm, tn, n0, nr;
        if (!gunit(a, gu, u, e, tm, tn, n0, nr, BN)) continue;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1)) {
            set_status(a.status, kStatusMbarTimeout);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[s], C::kStage);
          tma_load_2d_hint(&tmW, &full_bar[s], sA + s * C::kA, kb * kGBK, e * a.N + tm * kGBM, polA);
          tma_load_2d_hint(&tmX, &full_bar[s], sB + s * C::kB, kb * kGBK, n0, polB);
          issued_mask |= 1u << s;
          issued_ph = (issued_ph & ~(1u << s)) | (ph << s);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (*abort_flag)
        for (int j = 0; j < S; ++j)
          if (issued_mask & (1u << j)) mbar_wait(&full_bar[j], (issued_ph >> j) & 1u, 100000000ull);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = idesc_bf16_f32(kGBM, BN);
      int s = 0, i = 0;
      uint32_t ph = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int e, tm, tn, n0, nr;
        if (!gunit(a, gu, u, e, tm, tn, n0, nr, BN)) continue;
        const int ab = i & 1;
        if (!mbar_wait(&tempty[ab], ((i >> 1) & 1) ^ 1)) {
          set_status(a.status, kStatusMbarTimeout);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[s], ph)) {
            set_status(a.status, kStatusMbarTimeout);
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_sw128(smem_u32(sA + s * C::kA));
          const uint64_t db = smem_desc_sw128(smem_u32(sB + s * C::kB));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_f16(tmem + ab * BN, da + 2 * kk, db + 2 * kk, idesc, (kb | kk) ? 1u : 0u);
          umma_commit(&empty_bar[s]);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
        umma_commit(&tfull[ab]);
        ++i;
      }
    }
  } else {
    const int q = warp & 3;
    const int row = q * 32 + lane;  // weight row within the 128-row tile
    int i = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      int e, tm, tn, n0, nr;
      if (!gunit(a, gu, u, e, tm, tn, n0, nr, BN)) continue;
      const int ab = i & 1;
      if (!mbar_wait(&tfull[ab], (i >> 1) & 1)) {
        set_status(a.status, kStatusMbarTimeout);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + ab * BN;
      const int f = tm * kGBM + row;  // output feature (or gate/up row)
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        tmem_ld16(tb + c, v);
        if (SWIGLU) {
          const int fo = (f >> 5) * 16 + (lane & 15);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float up = __shfl_down_sync(0xffffffffu, v[j], 16);
            float gt = v[j];
            if (a.swiglu_limit > 0.f) {
              gt = fminf(gt, a.swiglu_limit);
              up = fminf(fmaxf(up, -a.swiglu_limit), a.swiglu_limit);
            }
            if (lane < 16 && c + j < nr)
              a.out[(long)(n0 + c + j) * a.ldo + fo] = __float2bfloat16(silu_f(gt) * up);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c + j < nr) a.out[(long)(n0 + c + j) * a.ldo + f] = __float2bfloat16(v[j]);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[ab]);
      ++i;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmem);
  }
}

template <int BN, bool SW>
static void launch_grouped(const CUtensorMap& tw, const CUtensorMap& tx, const GroupedArgs& a, cudaStream_t st) {
  using C = GCfg<BN>;
  auto k = grouped_gemm_kernel<BN, SW>;
  static bool set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    BWN_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    set[dev & 63] = true;
  }
  const int units = a.groups * a.tiles_m * a.max_tiles_n;
  const int sms = num_sms();
  launch_k(k, dim3(units < sms ? units : sms), dim3(kGThreadsG), C::kSmem, st, tw, tx, a);
}

void grouped_gemm(const GroupedProblem& p, cudaStream_t st) {
  BWN_CHECK(p.N % kGBM == 0, "grouped_gemm: N_out must be a multiple of 128");
  BWN_CHECK(p.groups <= kGMaxGroups, "grouped_gemm: at most %d groups", kGMaxGroups);
  BWN_CHECK(p.K % 8 == 0, "grouped_gemm: K multiple of 8");
  if (p.swiglu) BWN_CHECK(p.N % 32 == 0, "grouped_gemm: swiglu rows multiple of 32");
  int bn = 16;
  while (bn < p.max_rows_per_group && bn < 128) bn *= 2;
  if (p.max_rows_per_group > 128) bn = 128;
  CUtensorMap tw, tx;
  make_tmap_2d_bf16(&tw, p.W, (long)p.groups * p.N, p.K, p.K, kGBM, kGBK);
  make_tmap_2d_bf16(&tx, p.X, p.rows_total > 0 ? p.rows_total : 1, p.K, p.K, bn, kGBK);
  GroupedArgs a{};
  a.counts = p.counts;
  a.offsets = p.offsets;
  a.groups = p.groups;
  a.N = p.N;
  a.K = p.K;
  a.tiles_m = p.N / kGBM;
  a.max_tiles_n = (p.max_rows_per_group + bn - 1) / bn;
  a.out = p.out;
  a.ldo = p.ldo;
  a.status = p.status;
  a.swiglu_limit = p.swiglu_limit;
  if (a.max_tiles_n == 0) return;
  switch (bn) {
    case 16: p.swiglu ? launch_grouped<16, true>(tw, tx, a, st) : launch_grouped<16, false>(tw, tx, a, st); break;
    case 32: p.swiglu ? launch_grouped<32, true>(tw, tx, a, st) : launch_grouped<32, false>(tw, tx, a, st); break;
    case 64: p.swiglu ? launch_grouped<64, true>(tw, tx, a, st) : launch_grouped<64, false>(tw, tx, a, st); break;
    default: p.swiglu ? launch_grouped<128, true>(tw, tx, a, st) : launch_grouped<128, false>(tw, tx, a, st); break;
  }
}

}  // namespace bwn
