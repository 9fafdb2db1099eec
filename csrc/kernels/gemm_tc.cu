// Persistent tcgen05 GEMM for sm_100a:  D[M, N] = A[M, K] * B[N, K]^T
//
// Both operands are K-major bf16 (row-major activations and nn.Linear weights),
// fed by TMA with the 128-byte swizzle into a multi-stage shared-memory ring.
// Warp roles (192 threads):
//   warp 0      TMA producer (one elected lane)
//   warp 1      MMA issuer (one elected lane), TMEM allocator
//   warps 2..5  epilogue: tcgen05.ld from TMEM lanes 32*(warp%4).., fused
//               post-processing, global stores
// Accumulators are double-buffered in TMEM so the epilogue of tile i overlaps
// the main loop of tile i+1.  Split-K (for decode shapes where M/128 tiles
// cannot fill 148 SMs) writes fp32 partials to a workspace; the last CTA to
// finish a tile (atomic ticket) sums them and runs the epilogue, then re-arms
// the ticket so the same launch can be replayed from a CUDA graph.
//
// For decode ("swap-AB") the host passes the weight matrix as A (so the 128-row
// MMA M dimension spans output features) and the few token rows as B, and asks
// for a transposed store.  Epilogues: bf16 store, bf16 store + residual,
// SwiGLU over gate/up rows interleaved in blocks of 16, fp32 store.
#include "common/host.h"
#include "common/sm100.cuh"
#include <cstdlib>

#include "common/launch.cuh"
#include "kernels/gemm_epilogue.cuh"

namespace bwn {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kGemmThreads = 192;

// SMALL: a 4-stage ring (decode GEMMs whose units hold at most 8 K blocks):
// ~80 KB of shared memory at BN <= 32, so two CTAs fit on an SM and a GEMM
// launched with PDL can stream its first weight tiles while the previous
// kernel's CTAs are still resident.
template <int BN, bool SMALL = false>
struct GemmCfg {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStagesRaw = (200 * 1024) / kStageBytes;
  static constexpr int kStages = SMALL ? 4 : (kStagesRaw > 12 ? 12 : kStagesRaw);
  static constexpr int kTmemCols = (2 * BN) < 32 ? 32 : (2 * BN);
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// The reduction tail of kEpiSymmNorm (all 192 threads, after the CTA's tiles
// and the completion signal): every CTA that owns token rows waits for every
// rank's flag to reach `epoch`, then for each of its rows reads the sum of the
// ranks' partials through the switch, adds the residual and normalises.  The
// grid is at most one CTA per SM and every CTA triggers its dependents only
// once all of them run, so CTAs waiting here never keep a peer CTA of their own
// grid from being scheduled; the wait is bounded.
constexpr int kTailVec = 4;  // 8-column vectors per thread: cols <= 192 * 8 * 4
__device__ __forceinline__ void gemm_ar_tail(const GemmArgs& args, unsigned epoch) {
  const ArTail& t = args.tail;
  __shared__ float red[kGemmThreads / 32];
  __shared__ int s_ok;
  const int world = args.sig.world;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if ((int)blockIdx.x < t.rows && (int)threadIdx.x < world) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while ((int)(ld_acquire_sys(t.flags + threadIdx.x) - epoch) < 0) {
      if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > t.limit_ns) {
        set_status(args.status, kStatusPeerTimeout);
        s_ok = 0;  // a peer that never signalled: nothing is read or written
        break;
      }
    }
  }
  __syncthreads();
  const int sel = (*t.sel) & 1;
  for (int row = blockIdx.x; s_ok && row < t.rows; row += gridDim.x) {
    const __nv_bfloat16* buf = t.mc_base + (long)sel * args.sig.buf_stride + (long)row * t.cols;
    float v[kTailVec][8];
#pragma unroll
    for (int n = 0; n < kTailVec; ++n) {  // every reduction load in flight before use
      const int c = (threadIdx.x + n * kGemmThreads) * 8;
      if (c < t.cols) mc_ld_reduce_bf16x8(buf + c, v[n]);
    }
    float ss = 0.f;
#pragma unroll
    for (int n = 0; n < kTailVec; ++n) {
      const int c = (threadIdx.x + n * kGemmThreads) * 8;
      if (c >= t.cols) continue;
      const uint4 rr = *reinterpret_cast<const uint4*>(t.resid + (long)row * t.ldr + c);
      const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rr);
      uint4 o;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {  // the reduced partial is rounded to bf16, as the unfused all-reduce output
        const float2 rf = __bfloat1622float2(r2[e]);
        const float p0 = __bfloat162float(__float2bfloat16(v[n][2 * e]));
        const float p1 = __bfloat162float(__float2bfloat16(v[n][2 * e + 1]));
        const __nv_bfloat162 nb = __floats2bfloat162_rn(rf.x + p0, rf.y + p1);
        o2[e] = nb;
        const float2 nf = __bfloat1622float2(nb);
        v[n][2 * e] = nf.x;
        v[n][2 * e + 1] = nf.y;
        ss += nf.x * nf.x + nf.y * nf.y;
      }
      *reinterpret_cast<uint4*>(t.resid + (long)row * t.ldr + c) = o;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kGemmThreads / 32; ++i) tot += red[i];
    const float inv = rsqrtf(tot / t.cols + t.eps);
#pragma unroll
    for (int n = 0; n < kTailVec; ++n) {
      const int c = (threadIdx.x + n * kGemmThreads) * 8;
      if (c >= t.cols) continue;
      uint4 o;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        o2[e] = __floats2bfloat162_rn(v[n][2 * e] * inv * (1.f + t.w[c + 2 * e]),
                                      v[n][2 * e + 1] * inv * (1.f + t.w[c + 2 * e + 1]));
      *reinterpret_cast<uint4*>(t.out + (long)row * t.ldo + c) = o;
    }
    __syncthreads();  // red[] is reused by the next row
  }
  // flip the slot selector once every CTA has read it: last CTA (ticket)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int tk = atomicAdd(t.sel + 1, 1);
    if (tk == (int)gridDim.x - 1) {
      t.sel[1] = 0;
      t.sel[0] = t.sel[0] + 1;
    }
  }
}

// MAJ bit 0: A is MN-major (stored [K, M]); bit 1: B is MN-major (stored [K, N]);
// bit 2: the small (4-stage) ring.
template <int BN, int EPI, bool TRANS, int MAJ>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        GemmArgs args) {
  using C = GemmCfg<BN, (MAJ & 4) != 0>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * C::kABytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S * C::kStageBytes);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* tfull_bar = empty_bar + S;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* ticket_bcast = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles = args.tiles_m * args.tiles_n;
  const int units = tiles * args.splits;
  constexpr bool A_MN = (MAJ & 1) != 0, B_MN = (MAJ & 2) != 0;
  const uint32_t idesc = idesc_bf16_f32_major(kBM, BN, A_MN, B_MN);
  if (warp != 0) pdl_wait();  // the producer waits after prefetching static weight tiles

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (elect_one()) {
      const uint64_t polA = l2_policy_evict_first();
      const uint64_t polB = l2_policy_evict_last();
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_mask = 0, issued_ph = 0;  // per stage: issued at least once / parity of last issue
      // Weight prefetch: when B is the activation (swap-AB decode), the first
      // stages' A tiles (static weights) are issued before waiting for the
      // previous kernel, so the weight stream overlaps its tail.
      int pre = 0, pre_n = 0, kb00 = 0, tn0 = 0;
      if (TRANS && !A_MN && !B_MN && (int)blockIdx.x < units) {
        const int sp0 = blockIdx.x % args.splits, tile0 = blockIdx.x / args.splits;
        const int tm0 = tile0 % args.tiles_m;
        tn0 = tile0 / args.tiles_m;
        kb00 = sp0 * args.kb_per_split;
        const int kb01 = min(args.num_kb, kb00 + args.kb_per_split);
        pre = pre_n = min(S, kb01 - kb00);
        for (int j = 0; j < pre; ++j) {
          mbar_arrive_expect_tx(&full_bar[j], C::kStageBytes);
          tma_load_2d_hint(&tmA, &full_bar[j], sA + j * C::kABytes, (kb00 + j) * kBK, tm0 * kBM, polA);
          issued_mask |= 1u << j;
        }
      }
      pdl_wait();
      // all-gathered A: owners whose rows have arrived (this rank's are local)
      uint32_t ag_ready = args.ag.flags ? (1u << args.ag.rank) : 0xFFFFFFFFu;
      const unsigned ag_epoch = args.ag.flags ? (unsigned)(*args.ag.epoch) : 0u;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        const int tile = u / args.splits, sp = u % args.splits;
        const int tm = gemm_tile_m(args, tile, kBM), tn = tile / args.tiles_m;
        const int kb0 = sp * args.kb_per_split;
        const int kb1 = min(args.num_kb, kb0 + args.kb_per_split);
        if (!TRANS && !A_MN && args.ag.flags) {
          const int owner = (tm * kBM) / args.ag.rows;
          if (owner < args.ag.world && !((ag_ready >> owner) & 1u)) {
            const uint64_t t0 = globaltimer_ns();
            uint32_t spins = 0;
            while ((int)(ld_acquire_sys(args.ag.flags + owner) - ag_epoch) < 0) {
              if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > args.ag.limit_ns) {
                set_status(args.status, kStatusPeerTimeout);
                *abort_flag = 1;
                break;
              }
            }
            if (*abort_flag) break;
            ag_ready |= 1u << owner;
          }
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (pre > 0) {  // A already in flight for this stage: only B remains
            tma_load_2d_hint(&tmB, &full_bar[s], sB + s * C::kBBytes, kb * kBK, tn * BN, polB);
            issued_mask |= 1u << s;
            issued_ph = (issued_ph & ~(1u << s)) | (ph << s);
            --pre;
            if (++s == S) {
              s = 0;
              ph ^= 1;
            }
            continue;
          }
          if (!mbar_wait(&empty_bar[s], ph ^ 1)) {
            set_status(args.status, kStatusMbarTimeout);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[s], C::kStageBytes);
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < kBM / 64; ++j)
              tma_load_2d_hint(&tmA, &full_bar[s], sA + s * C::kABytes + j * 8192, tm * kBM + j * 64, kb * kBK, polA);
          } else {
            tma_load_2d_hint(&tmA, &full_bar[s], sA + s * C::kABytes, kb * kBK, tm * kBM, polA);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d_hint(&tmB, &full_bar[s], sB + s * C::kBBytes + j * 8192, tn * BN + j * 64, kb * kBK, polB);
          } else {
            tma_load_2d_hint(&tmB, &full_bar[s], sB + s * C::kBBytes, kb * kBK, tn * BN, polB);
          }
          issued_mask |= 1u << s;
          issued_ph = (issued_ph & ~(1u << s)) | (ph << s);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (*abort_flag) {
        // complete the transaction count of prefetched stages that never got
        // their B tile, then a bounded wait for this CTA's own copies in flight
        for (int j = pre_n - pre; j < pre_n; ++j)
          tma_load_2d_hint(&tmB, &full_bar[j], sB + j * C::kBBytes, (kb00 + j) * kBK, tn0 * BN, polB);
        for (int j = 0; j < S; ++j)
          if (issued_mask & (1u << j)) mbar_wait(&full_bar[j], (issued_ph >> j) & 1u, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (elect_one()) {
      int s = 0;
      uint32_t ph = 0;
      int i = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x, ++i) {
        const int sp = u % args.splits;
        const int kb0 = sp * args.kb_per_split;
        const int kb1 = min(args.num_kb, kb0 + args.kb_per_split);
        const int ab = i & 1;
        const uint32_t use = (uint32_t)(i >> 1);
        if (!mbar_wait(&tempty_bar[ab], (use & 1) ^ 1)) {
          set_status(args.status, kStatusMbarTimeout);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + ab * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[s], ph)) {
            set_status(args.status, kStatusMbarTimeout);
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint64_t da = A_MN ? smem_desc_sw128_mn(smem_u32(sA + s * C::kABytes), 8192)
                                   : smem_desc_sw128(smem_u32(sA + s * C::kABytes));
          const uint64_t db = B_MN ? smem_desc_sw128_mn(smem_u32(sB + s * C::kBBytes), 8192)
                                   : smem_desc_sw128(smem_u32(sB + s * C::kBBytes));
          // K step of 16: K-major +32 bytes (encoded +2); MN-major +16 rows x 128 B (encoded +128)
          constexpr uint64_t kStepA = A_MN ? 128 : 2, kStepB = B_MN ? 128 : 2;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            umma_f16(d, da + kStepA * kk, db + kStepB * kk, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[s]);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
        umma_commit(&tfull_bar[ab]);
      }
    }
  } else {
    // ------------------------------ epilogue ------------------------------
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = q * 32 + lane;
    int i = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++i) {
      const int tile = u / args.splits, sp = u % args.splits;
      const int tm = gemm_tile_m(args, tile, kBM), tn = tile / args.tiles_m;
      const int ab = i & 1;
      const uint32_t use = (uint32_t)(i >> 1);
      if (!mbar_wait(&tfull_bar[ab], use & 1)) {
        set_status(args.status, kStatusMbarTimeout);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + ab * BN;
      const int m = tm * kBM + row;
      if (args.splits == 1) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          if (BN >= 32) {
            tmem_ld32(tbase + c, v);
          } else {
            float h[16];
            tmem_ld16(tbase + c, h);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = h[j];
#pragma unroll
            for (int j = 16; j < 32; ++j) v[j] = 0.f;
          }
          epi_store_chunk<BN, EPI, TRANS>(args, v, BN >= 32 ? 32 : 16, m, tn * BN + c);
        }
        tc_fence_before();
        mbar_arrive(&tempty_bar[ab]);
      } else {
        float* ws = args.workspace + ((long)tile * args.splits + sp) * (kBM * BN);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          if (BN >= 32) {
            tmem_ld32(tbase + c, v);
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(ws + (long)row * BN + c + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
          } else {
            float h[16];
            tmem_ld16(tbase + c, h);
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<float4*>(ws + (long)row * BN + c + j) = make_float4(h[j], h[j + 1], h[j + 2], h[j + 3]);
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty_bar[ab]);
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          const int t = atomicAdd(&args.tickets[tile], 1);
          *ticket_bcast = t;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int t = *ticket_bcast;
        if (t == args.splits - 1) {
          __threadfence();
          const float* base = args.workspace + (long)tile * args.splits * (kBM * BN);
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
            const int w = BN >= 32 ? 32 : 16;
            for (int s2 = 0; s2 < args.splits; ++s2) {
              const float* p = base + (long)s2 * (kBM * BN) + (long)row * BN + c;
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                if (j < w) {
                  const float4 x = __ldcg(reinterpret_cast<const float4*>(p + j));
                  v[j] += x.x;
                  v[j + 1] += x.y;
                  v[j + 2] += x.z;
                  v[j + 3] += x.w;
                }
              }
            }
            epi_store_chunk<BN, EPI, TRANS>(args, v, w, m, tn * BN + c);
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (threadIdx.x == 64) args.tickets[tile] = 0;  // re-arm for the next launch
        }
      }
    }
  }

  if ((EPI == kEpiSymm || EPI == kEpiSymmNorm) && warp >= 2) {
    // publish completion: the epilogue warps' stores precede one thread's
    // system-scope fence (named barrier), then the ticket; the last CTA bumps
    // the epoch and release-stores it to all ranks
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (threadIdx.x == 64) {
      // the epoch this launch publishes, read before this CTA's ticket (the
      // last ticket of the grid is what bumps it)
      *ticket_bcast = *args.sig.epoch + 1;
      __threadfence();
      const int t = atomicAdd(args.sig.done_ticket, 1);
      if (t == (int)gridDim.x - 1) {
        *args.sig.done_ticket = 0;
        fence_acq_rel_sys();
        const unsigned e = (unsigned)(*args.sig.epoch) + 1u;
        *args.sig.epoch = (int)e;
        for (int r = 0; r < args.sig.world; ++r) st_relaxed_sys_u32(args.sig.peer_flags[r] + args.sig.rank, e);
      }
    }
  }
  // Teardown (the producer already drained its in-flight copies on abort).
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
  if (EPI == kEpiSymmNorm) gemm_ar_tail(args, (unsigned)*ticket_bcast);
}

// ---------------------------------------------------------------------------
// host launcher
// ---------------------------------------------------------------------------
template <int BN, int EPI, bool TRANS, int MAJ>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid,
                        cudaStream_t stream) {
  using C = GemmCfg<BN, (MAJ & 4) != 0>;
  auto k = gemm_bf16_tc_kernel<BN, EPI, TRANS, MAJ>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    BWN_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
    attr_set[dev & 63] = true;
  }
  launch_k(k, dim3(grid), dim3(kGemmThreads), C::kSmemBytes, stream, ta, tb, a);
}

template <int EPI, bool TRANS>
static void dispatch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid,
                        cudaStream_t st, bool small = false) {
  if (TRANS && small) {  // decode: small ring
    switch (bn) {
      case 16: launch_gemm<16, EPI, TRANS, 4>(ta, tb, a, grid, st); return;
      case 32: launch_gemm<32, EPI, TRANS, 4>(ta, tb, a, grid, st); return;
      default: break;
    }
  }
  switch (bn) {
    case 16: launch_gemm<16, EPI, TRANS, 0>(ta, tb, a, grid, st); break;
    case 32: launch_gemm<32, EPI, TRANS, 0>(ta, tb, a, grid, st); break;
    case 64: launch_gemm<64, EPI, TRANS, 0>(ta, tb, a, grid, st); break;
    case 128: launch_gemm<128, EPI, TRANS, 0>(ta, tb, a, grid, st); break;
    case 256: launch_gemm<256, EPI, TRANS, 0>(ta, tb, a, grid, st); break;
    default: BWN_FAIL("gemm: unsupported BN %d", bn);
  }
}

template <int EPI, int MAJ>
static void dispatch_mn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid,
                        cudaStream_t st) {
  switch (bn) {
    case 64: launch_gemm<64, EPI, false, MAJ>(ta, tb, a, grid, st); break;
    case 128: launch_gemm<128, EPI, false, MAJ>(ta, tb, a, grid, st); break;
    case 256: launch_gemm<256, EPI, false, MAJ>(ta, tb, a, grid, st); break;
    default: BWN_FAIL("gemm: MN-major operands need BN in {64,128,256}, got %d", bn);
  }
}

int gemm_pick_bn(int n) {
  if (n <= 16) return 16;
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  if (n <= 128) return 128;
  return 256;
}

void gemm_bf16(const GemmProblem& p, cudaStream_t stream) {
  BWN_CHECK(p.K % 8 == 0, "gemm: K must be a multiple of 8 (TMA 16-byte stride rule)");
  BWN_CHECK(p.lda % 8 == 0 && p.ldb % 8 == 0, "gemm: lda/ldb must be multiples of 8");
  BWN_CHECK((reinterpret_cast<uintptr_t>(p.A) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.B) & 15) == 0,
            "gemm: A/B must be 16-byte aligned");
  const int maj = (p.a_mn ? 1 : 0) | (p.b_mn ? 2 : 0);
  int bn = p.bn > 0 ? p.bn : gemm_pick_bn(p.N);
  if (maj && bn < 64) bn = 64;
  CUtensorMap ta, tb;
  if (p.a_mn)
    make_tmap_2d_bf16(&ta, p.A, p.K, p.M, p.lda, kBK, 64);  // stored [K, M]
  else
    make_tmap_2d_bf16(&ta, p.A, p.M, p.K, p.lda, kBM, kBK);
  if (p.b_mn)
    make_tmap_2d_bf16(&tb, p.B, p.K, p.N, p.ldb, kBK, 64);  // stored [K, N]
  else
    make_tmap_2d_bf16(&tb, p.B, p.N, p.K, p.ldb, bn, kBK);
  GemmArgs a{};
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  if (p.ag.flags) {
    BWN_CHECK(!p.trans_out && !p.a_mn && p.ag.rows % kBM == 0 && p.ag.world >= 1 && p.ag.world <= 32 &&
                  (long)p.ag.rows * p.ag.world == p.M,
              "gemm: all-gathered A needs the normal orientation and 128-row shards covering M");
    a.ag = p.ag;
  }
  a.tiles_m = (p.M + kBM - 1) / kBM;
  a.tiles_n = (p.N + bn - 1) / bn;
  a.num_kb = (p.K + kBK - 1) / kBK;
  const int tiles = a.tiles_m * a.tiles_n;
  const int sms = num_sms();
  // Split-K when the output tiles cannot fill the SMs: one wave of
  // tiles*splits <= #SM CTAs, each with >= 4 k-blocks.  (Several split units
  // per persistent CTA measured ~2x slower on decode shapes: each unit's
  // partial round trip and fence serialises the CTA.)
  int splits = 1;
  if (p.allow_split && tiles < sms && p.workspace && p.tickets && tiles <= p.tickets_len) {
    splits = sms / tiles;
    if (splits > a.num_kb / 4) splits = a.num_kb / 4 > 0 ? a.num_kb / 4 : 1;
    static const int max_splits = [] {
      const char* e = getenv("BWN_GEMM_MAX_SPLITS");
      const int v = e ? atoi(e) : 16;
      return v >= 1 && v <= 16 ? v : 16;
    }();
    if (splits > max_splits) splits = max_splits;
    if ((long)tiles * splits * kBM * bn > p.workspace_floats) splits = 1;
  }
  a.splits = splits;
  a.kb_per_split = (a.num_kb + splits - 1) / splits;
  a.splits = (a.num_kb + a.kb_per_split - 1) / a.kb_per_split;  // drop empty splits
  a.out = p.out;
  a.ldo = p.ldo;
  a.resid = p.resid;
  a.ldr = p.ldr;
  a.workspace = p.workspace;
  a.tickets = p.tickets;
  a.status = p.status;
  a.sig = p.sig;
  a.tail = p.tail;
  const int units = tiles * a.splits;
  const int grid = units < sms ? units : sms;
  const bool tr = p.trans_out;
  static const bool small_ok = [] {
    const char* e = getenv("BWN_GEMM_SMALL_RING");
    return !(e && e[0] == '0');
  }();
  const bool small = small_ok && tr && !maj && bn <= 32 && a.kb_per_split <= 8;
  if (maj) {
    BWN_CHECK(!tr && (p.epi == kEpiBF16 || p.epi == kEpiF32), "gemm: MN-major operands support bf16/f32 epilogues");
    const bool f32 = p.epi == kEpiF32;
    switch (maj) {
      case 1: f32 ? dispatch_mn<kEpiF32, 1>(bn, ta, tb, a, grid, stream) : dispatch_mn<kEpiBF16, 1>(bn, ta, tb, a, grid, stream); break;
      case 2: f32 ? dispatch_mn<kEpiF32, 2>(bn, ta, tb, a, grid, stream) : dispatch_mn<kEpiBF16, 2>(bn, ta, tb, a, grid, stream); break;
      default: f32 ? dispatch_mn<kEpiF32, 3>(bn, ta, tb, a, grid, stream) : dispatch_mn<kEpiBF16, 3>(bn, ta, tb, a, grid, stream); break;
    }
    return;
  }
  switch (p.epi) {
    case kEpiBF16:
      tr ? dispatch_bn<kEpiBF16, true>(bn, ta, tb, a, grid, stream, small) : dispatch_bn<kEpiBF16, false>(bn, ta, tb, a, grid, stream);
      break;
    case kEpiResid:
      tr ? dispatch_bn<kEpiResid, true>(bn, ta, tb, a, grid, stream, small) : dispatch_bn<kEpiResid, false>(bn, ta, tb, a, grid, stream);
      break;
    case kEpiSwiGLU:
      tr ? dispatch_bn<kEpiSwiGLU, true>(bn, ta, tb, a, grid, stream, small) : dispatch_bn<kEpiSwiGLU, false>(bn, ta, tb, a, grid, stream);
      break;
    case kEpiF32:
      tr ? dispatch_bn<kEpiF32, true>(bn, ta, tb, a, grid, stream, small) : dispatch_bn<kEpiF32, false>(bn, ta, tb, a, grid, stream);
      break;
    case kEpiSymm:
      BWN_CHECK(p.sig.epoch && p.sig.done_ticket && p.sig.world >= 1 && p.sig.world <= 8, "gemm: bad comm signal");
      tr ? dispatch_bn<kEpiSymm, true>(bn, ta, tb, a, grid, stream, small) : dispatch_bn<kEpiSymm, false>(bn, ta, tb, a, grid, stream);
      break;
    case kEpiSymmNorm:
      BWN_CHECK(p.sig.epoch && p.sig.done_ticket && p.sig.world >= 1 && p.sig.world <= 8, "gemm: bad comm signal");
      BWN_CHECK(p.tail.mc_base && p.tail.flags && p.tail.sel && p.tail.resid && p.tail.w && p.tail.out &&
                    p.tail.cols % 8 == 0 && p.tail.cols <= kGemmThreads * 8 * kTailVec && p.tail.ldr % 8 == 0 &&
                    p.tail.ldo % 8 == 0,
                "gemm: bad reduction tail (hidden a multiple of 8, at most %d)", kGemmThreads * 8 * kTailVec);
      tr ? dispatch_bn<kEpiSymmNorm, true>(bn, ta, tb, a, grid, stream, small)
         : dispatch_bn<kEpiSymmNorm, false>(bn, ta, tb, a, grid, stream);
      break;
    default: BWN_FAIL("gemm: bad epilogue %d", p.epi);
  }
}

}  // namespace bwn
