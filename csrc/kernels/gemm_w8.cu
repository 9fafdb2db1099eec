// FP8 W8A16 GEMM for sm_100a (the reference's fp8 W8A16 matmul,
// contrib/qwen3.6-27b/kernels/fp8_matmul.py:55-184, with the 128x128 block
// scales of the official FP8 checkpoints, contrib/qwen3.6-35b-a3b/moe_w8.py:139):
//
//   out[t, n] = sum_k x[t, k] * (w8[n, k] * scale[n / 128, k / 128])
//
// Orientation is swap-AB: the fp8 weight is the 128-row MMA "A" operand, the
// bf16 token rows are "B", the store is transposed.  Per 128-deep K block:
//   warp 0      TMA: fp8 weight tile [128 x 128 B] (SW128) + bf16 token tile
//   warps 6-13  converters: the fp8 weight tile to f16 with the hardware
//               e4m3x2 -> f16x2 conversion (exact for every e4m3 value),
//               stored straight into tensor memory (two warps per TMEM lane
//               quadrant, one K half each), and the bf16 token tile to f16
//               scaled by this tile's 128x128 block scale (W x^T = w8 (s x)^T:
//               each CTA owns one scale block row) in the SW128 K-major layout
//               the MMA reads from shared memory
//   warp 1      tcgen05.mma kind::f16 (f16 x f16 -> fp32 TMEM) with A read
//               from tensor memory, 8 per block
//   warps 2-5   epilogue (shared with the bf16 GEMM: bf16 / residual /
//               SwiGLU / fp32 / NVLS multimem reduction)
// Split-K and the completion signalling are the same as the bf16 GEMM.
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "common/host.h"
#include "common/sm100.cuh"
#include "common/launch.cuh"
#include "kernels/gemm_epilogue.cuh"
#include "kernels/gemm_w8.h"

namespace bwn {

constexpr int kW8BM = 128;
constexpr int kW8BK = 128;  // fp8 elements (bytes) per row per stage
constexpr int kW8Threads = 448;
constexpr int kW8SlotCol0 = 256;  // TMEM columns [0, 256): the two accumulators

template <int BN>
struct W8Cfg {
  static constexpr int kA8 = kW8BM * kW8BK;        // 16 KB fp8 weight tile
  static constexpr int kB = BN * kW8BK * 2;        // token tile (two SW128 boxes), bf16 in / f16 out
  static constexpr int kL = kA8 + kB;              // TMA ring stage
  static constexpr int kSlots = BN <= 64 ? 4 : 2;  // converted stages: A in TMEM (64 columns), B in smem
  static constexpr int kNLRaw = (208 * 1024 - kSlots * kB) / kL;
  static constexpr int kNL = kNLRaw > 8 ? 8 : kNLRaw;
  static constexpr int kMaxKb = 512;  // scales staged per unit
  static constexpr int kSmem = kNL * kL + kSlots * kB + 1024 + 512 + kMaxKb * 4;
  static_assert(kNL >= 2, "gemm_w8: shared memory ring does not fit");
  static_assert(2 * BN <= kW8SlotCol0, "gemm_w8: accumulators overlap the A slots");
};

// four e4m3 bytes -> two f16x2 words (bytes 0,1 -> lo; bytes 2,3 -> hi), exactly
__device__ __forceinline__ void e4m3x4_to_f16x4(uint32_t v, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 l, h;\n\t"
      "mov.b32 {l, h}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, l;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(v));
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kW8Threads, 1)
    gemm_w8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs args,
                   const float* __restrict__ scales, int lds) {
  using C = W8Cfg<BN>;
  constexpr int S = C::kNL;      // TMA ring depth
  constexpr int SL = C::kSlots;  // converted stages
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sA8 = smem;                    // [S][kA8]
  uint8_t* sB = sA8 + S * C::kA8;         // [S][kB]   bf16 tokens
  uint8_t* sB16 = sB + S * C::kB;         // [SL][kB]  f16 tokens * scale
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sB16 + SL * C::kB);  // [S]  TMA landed
  uint64_t* lempty_bar = full_bar + S;    // [S]  converters done reading
  uint64_t* cvt_bar = lempty_bar + S;     // [SL] converted stage ready (A in TMEM, B in smem)
  uint64_t* empty_bar = cvt_bar + SL;     // [SL] MMA done with the stage
  uint64_t* tfull_bar = empty_bar + SL;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* ticket_bcast = reinterpret_cast<int*>(tmem_slot + 2);
  float* s_scale = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full_bar) + 512);  // [kMaxKb]
  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&lempty_bar[i], 256);
    }
    for (int i = 0; i < SL; ++i) {
      mbar_init(&cvt_bar[i], 256);
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
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  const uint32_t tmem_base = *tmem_slot;
  const int tiles = args.tiles_m * args.tiles_n;
  const int units = tiles * args.splits;

  if (warp == 0) {
    if (elect_one()) {
      const uint64_t polA = l2_policy_evict_first(), polB = l2_policy_evict_last();
      int s = 0;
      uint32_t ph = 0, issued_mask = 0, issued_ph = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        const int tile = u / args.splits, sp = u % args.splits;
        const int tm = tile % args.tiles_m, tn = tile / args.tiles_m;
        const int kb0 = sp * args.kb_per_split, kb1 = min(args.num_kb, kb0 + args.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&lempty_bar[s], ph ^ 1)) {
            set_status(args.status, kStatusMbarTimeout);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[s], C::kA8 + C::kB);
          tma_load_2d_hint(&tmA, &full_bar[s], sA8 + s * C::kA8, kb * kW8BK, tm * kW8BM, polA);
          tma_load_2d_hint(&tmB, &full_bar[s], sB + s * C::kB, kb * kW8BK, tn * BN, polB);
          tma_load_2d_hint(&tmB, &full_bar[s], sB + s * C::kB + BN * 128, kb * kW8BK + 64, tn * BN, polB);
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
  } else if (warp >= 6) {
    // ------------------------------ converters ------------------------------
    // two warps per TMEM lane quadrant (one K half each): the thread of weight
    // row r turns its 64 fp8 bytes into f16 (exact) and stores them into its
    // own TMEM lane of the stage's A slot; all 256 threads scale the token tile
    // by the block scale into f16 in the SW128 layout the MMA reads as B
    const int c = threadIdx.x - 6 * 32;  // 0..255
    const int q = warp & 3, half = (warp - 6) >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    int s = 0, sl = 0;
    uint32_t ph = 0, ph2 = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      // all 256 converter threads leave together after an abort (the named
      // barrier below needs every one of them)
      if (bar_any(2, 256, *abort_flag != 0)) break;
      const int tile = u / args.splits, sp = u % args.splits;
      const int tm = tile % args.tiles_m;
      const int kb0 = sp * args.kb_per_split, kb1 = min(args.num_kb, kb0 + args.kb_per_split);
      // stage this unit's block scales once (a per-block global load would put
      // an L2 round trip in front of every conversion)
      for (int j = c; j < kb1 - kb0; j += 256) s_scale[j] = scales[(long)tm * lds + kb0 + j];
      asm volatile("bar.sync 2, 256;" ::: "memory");
      for (int kb = kb0; kb < kb1; ++kb) {
        if (*abort_flag || !mbar_wait(&full_bar[s], ph) || !mbar_wait(&empty_bar[sl], ph2 ^ 1)) {
          set_status(args.status, kStatusMbarTimeout);
          *abort_flag = 1;
          break;
        }
        const float sc = s_scale[kb - kb0];
        const uint8_t* a8 = sA8 + s * C::kA8 + r * 128;
        uint32_t o[32];
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const int cc = half * 4 + qq;  // 16-byte fp8 chunk = 16 k
          const uint4 raw8 = *reinterpret_cast<const uint4*>(a8 + ((cc ^ (r & 7)) << 4));
          const uint32_t w[4] = {raw8.x, raw8.y, raw8.z, raw8.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) e4m3x4_to_f16x4(w[j], o[qq * 8 + 2 * j], o[qq * 8 + 2 * j + 1]);
        }
        // column c of the slot holds k = 2c, 2c+1 of this row
        tmem_st32u(tmem_base + lane_addr + kW8SlotCol0 + sl * 64 + half * 32, o);
        {  // token tile: bf16 -> f16 * block scale, same swizzled positions
          const uint32_t* b32 = reinterpret_cast<const uint32_t*>(sB + s * C::kB);
          uint32_t* o32 = reinterpret_cast<uint32_t*>(sB16 + sl * C::kB);
          for (int i = c; i < C::kB / 4; i += 256) {
            const uint32_t v = b32[i];
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
            __half2 h = __floats2half2_rn(f.x * sc, f.y * sc);
            o32[i] = *reinterpret_cast<uint32_t*>(&h);
          }
        }
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&cvt_bar[sl]);
        mbar_arrive(&lempty_bar[s]);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
        if (++sl == SL) {
          sl = 0;
          ph2 ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      // kind::f16 with A = B = f16 (format 0), D = f32; A read from TMEM
      const uint32_t idesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kW8BM >> 4) << 24);
      int s = 0, i = 0;
      uint32_t ph = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x, ++i) {
        const int sp = u % args.splits;
        const int kb0 = sp * args.kb_per_split, kb1 = min(args.num_kb, kb0 + args.kb_per_split);
        const int ab = i & 1;
        if (!mbar_wait(&tempty_bar[ab], ((i >> 1) & 1) ^ 1)) {
          set_status(args.status, kStatusMbarTimeout);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + ab * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&cvt_bar[s], ph)) {
            set_status(args.status, kStatusMbarTimeout);
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint32_t at = tmem_base + kW8SlotCol0 + s * 64;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const uint64_t db = smem_desc_sw128(smem_u32(sB16 + s * C::kB + t * (BN * 128)));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_f16_ts(d, at + t * 32 + kk * 8, db + 2 * kk, idesc, (kb > kb0 || t > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[s]);
          if (++s == SL) {
            s = 0;
            ph ^= 1;
          }
        }
        umma_commit(&tfull_bar[ab]);
      }
    }
  } else {
    // ------------------------------ epilogue (warps 2-5) ---------------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    int i = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++i) {
      const int tile = u / args.splits, sp = u % args.splits;
      const int tm = tile % args.tiles_m, tn = tile / args.tiles_m;
      const int ab = i & 1;
      if (!mbar_wait(&tfull_bar[ab], (i >> 1) & 1)) {
        set_status(args.status, kStatusMbarTimeout);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + ab * BN;
      const int m = tm * kW8BM + row;
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
          epi_store_chunk<BN, EPI, true>(args, v, BN >= 32 ? 32 : 16, m, tn * BN + c);
        }
        tc_fence_before();
        mbar_arrive(&tempty_bar[ab]);
      } else {
        float* ws = args.workspace + ((long)tile * args.splits + sp) * (kW8BM * BN);
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          float h[16];
          tmem_ld16(tbase + c, h);
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            *reinterpret_cast<float4*>(ws + (long)row * BN + c + j) = make_float4(h[j], h[j + 1], h[j + 2], h[j + 3]);
        }
        tc_fence_before();
        mbar_arrive(&tempty_bar[ab]);
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 64) *ticket_bcast = atomicAdd(&args.tickets[tile], 1);
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (*ticket_bcast == args.splits - 1) {
          __threadfence();
          const float* base = args.workspace + (long)tile * args.splits * (kW8BM * BN);
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
            const int w = BN >= 32 ? 32 : 16;
            for (int s2 = 0; s2 < args.splits; ++s2) {
              const float* pp = base + (long)s2 * (kW8BM * BN) + (long)row * BN + c;
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                if (j < w) {
                  const float4 x = __ldcg(reinterpret_cast<const float4*>(pp + j));
                  v[j] += x.x;
                  v[j + 1] += x.y;
                  v[j + 2] += x.z;
                  v[j + 3] += x.w;
                }
            }
            epi_store_chunk<BN, EPI, true>(args, v, w, m, tn * BN + c);
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (threadIdx.x == 64) args.tickets[tile] = 0;
        }
      }
    }
    if (EPI == kEpiSymm) {
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) {
        __threadfence();
        const int t = atomicAdd(args.sig.done_ticket, 1);
        if (t == (int)gridDim.x - 1) {
          *args.sig.done_ticket = 0;
          fence_acq_rel_sys();
          const unsigned e = (unsigned)(*args.sig.epoch) + 1u;
          *args.sig.epoch = (int)e;
          for (int r2 = 0; r2 < args.sig.world; ++r2) st_relaxed_sys_u32(args.sig.peer_flags[r2] + args.sig.rank, e);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <int BN, int EPI>
static void launch_w8(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, const float* scales, int lds,
                      int grid, cudaStream_t st) {
  using C = W8Cfg<BN>;
  auto k = gemm_w8_kernel<BN, EPI>;
  static bool set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    BWN_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    set[dev & 63] = true;
  }
  launch_k(k, dim3(grid), dim3(kW8Threads), C::kSmem, st, ta, tb, a, scales, lds);
}

template <int EPI>
static void w8_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, const float* sc, int lds,
                  int grid, cudaStream_t st) {
  switch (bn) {
    case 16: launch_w8<16, EPI>(ta, tb, a, sc, lds, grid, st); break;
    case 32: launch_w8<32, EPI>(ta, tb, a, sc, lds, grid, st); break;
    case 64: launch_w8<64, EPI>(ta, tb, a, sc, lds, grid, st); break;
    default: launch_w8<128, EPI>(ta, tb, a, sc, lds, grid, st); break;
  }
}

void gemm_w8(const GemmW8Problem& p, cudaStream_t stream) {
  BWN_CHECK(p.K % 16 == 0, "gemm_w8: K must be a multiple of 16");
  BWN_CHECK(p.ldb % 8 == 0 && p.lda % 16 == 0, "gemm_w8: strides (16-byte TMA rule)");
  int bn = 16;
  while (bn < p.N && bn < 128) bn *= 2;
  CUtensorMap ta, tb;
  make_tmap_2d_u8(&ta, p.A, p.M, p.K, p.lda, kW8BM, kW8BK);
  make_tmap_2d_bf16(&tb, p.B, p.N, p.K, p.ldb, bn, 64);
  GemmArgs a{};
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.tiles_m = (p.M + kW8BM - 1) / kW8BM;
  a.tiles_n = (p.N + bn - 1) / bn;
  a.num_kb = (p.K + kW8BK - 1) / kW8BK;
  const int tiles = a.tiles_m * a.tiles_n, sms = num_sms();
  int splits = 1;
  if (tiles < sms && p.workspace && p.tickets && tiles <= p.tickets_len) {
    splits = sms / tiles;
    if (splits > a.num_kb / 2) splits = a.num_kb / 2 > 0 ? a.num_kb / 2 : 1;
    if (splits > 16) splits = 16;
    if ((long)tiles * splits * kW8BM * bn > p.workspace_floats) splits = 1;
  }
  a.kb_per_split = (a.num_kb + splits - 1) / splits;
  a.splits = (a.num_kb + a.kb_per_split - 1) / a.kb_per_split;
  BWN_CHECK(a.kb_per_split <= 512, "gemm_w8: K too large for the staged scales (%d blocks)", a.kb_per_split);
  a.out = p.out;
  a.ldo = p.ldo;
  a.resid = p.resid;
  a.ldr = p.ldr;
  a.workspace = p.workspace;
  a.tickets = p.tickets;
  a.status = p.status;
  a.sig = p.sig;
  const int units = tiles * a.splits;
  const int grid = units < sms ? units : sms;
  switch (p.epi) {
    case kEpiBF16: w8_bn<kEpiBF16>(bn, ta, tb, a, p.scales, p.lds, grid, stream); break;
    case kEpiResid: w8_bn<kEpiResid>(bn, ta, tb, a, p.scales, p.lds, grid, stream); break;
    case kEpiSwiGLU: w8_bn<kEpiSwiGLU>(bn, ta, tb, a, p.scales, p.lds, grid, stream); break;
    case kEpiF32: w8_bn<kEpiF32>(bn, ta, tb, a, p.scales, p.lds, grid, stream); break;
    case kEpiSymm: w8_bn<kEpiSymm>(bn, ta, tb, a, p.scales, p.lds, grid, stream); break;
    default: BWN_FAIL("gemm_w8: bad epilogue");
  }
}

}  // namespace bwn
