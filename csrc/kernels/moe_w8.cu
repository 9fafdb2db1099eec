// Grouped expert GEMM with block-scaled E4M3FN weights for sm_100a: the
// reference's fused all-expert W8 MoE and FP8 grouped matvec
// (contrib/qwen3.6-35b-a3b/kernels/moe_fused_w8_35b.py:345-940,
// kernels/fp8_group_matvec.py:47-105) on the tensor cores, with bf16
// activations (W8A16).
//
// Same schedule as the bf16 grouped GEMM (csrc/kernels/moe.cu): swap-AB, one
// work unit = (expert e, 128 weight rows, BN token rows of e), units compacted
// over the device row counts so one launch shape serves every routing.  The
// weight stays fp8 in HBM (half the bytes of bf16).  Converter warps turn each
// fp8 tile into bf16 (hardware e4m3x2 -> f16x2, exact; times the row group's
// block scale in fp32; rounded to bf16, the same rounding as dequantizing at
// load) and store it straight into tensor memory, where tcgen05.mma reads its
// A operand; the token tile is the B operand in shared memory as TMA loaded
// it.  Scales are kept per 16 weight rows (scales16, see moe.h) so the gate/up
// interleave of a 128-row tile needs no re-quantization.
#include <cuda_fp16.h>

#include "common/host.h"
#include "common/launch.cuh"
#include "common/sm100.cuh"
#include "kernels/grouped_units.cuh"
#include "kernels/moe.h"

namespace bwn {

namespace {

constexpr int kXBM = 128;    // weight rows per tile
constexpr int kXBK = 128;    // fp8 columns (bytes) per K block
constexpr int kXCvtWarps = 8;                    // two per TMEM lane quadrant
constexpr int kXThreads = (6 + kXCvtWarps) * 32;
constexpr int kXSlots = 4;                       // converted A tiles in TMEM, 64 columns each
constexpr int kXSlotCol0 = 256;                  // TMEM columns [0, 256): the two accumulators
constexpr int kXMaxScales = 1024;                // 8 row groups x K blocks staged per unit

template <int BN>
struct XCfg {
  static constexpr int kA8 = kXBM * kXBK;       // 16 KB fp8 weight tile
  static constexpr int kB = BN * kXBK * 2;      // bf16 token tile (two SW128 boxes)
  static constexpr int kL = kA8 + kB;           // TMA ring stage
  static constexpr int kNLRaw = (208 * 1024) / kL;
  static constexpr int kNL = kNLRaw > 8 ? 8 : kNLRaw;
  static constexpr int kSmem = kNL * kL + 1024 + 512 + kXMaxScales * 4;
  static_assert(kNL >= 2, "fp8 grouped GEMM: shared memory ring does not fit");
  static_assert(2 * BN <= kXSlotCol0, "fp8 grouped GEMM: accumulators overlap the A slots");
};

struct GroupedW8Args {
  GroupedArgs g;
  const float* scales16;
  int nkb;  // K blocks of 128
};

// four e4m3 bytes -> two f16x2 words (bytes 0,1 -> lo; bytes 2,3 -> hi), exactly
__device__ __forceinline__ void e4m3x4_to_f16x4_g(uint32_t v, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 l, h;\n\t"
      "mov.b32 {l, h}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, l;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(v));
}

// f16x2 (exact fp8 values) * scale -> bf16x2
__device__ __forceinline__ uint32_t scale_to_bf16x2(uint32_t h2, float s) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
  const __nv_bfloat162 b = __floats2bfloat162_rn(f.x * s, f.y * s);
  return *reinterpret_cast<const uint32_t*>(&b);
}

// Pipeline per 128-deep K block j of a unit (TMA stage s = j mod kNL, TMEM
// slot t = j mod kXSlots):
//   warp 0      TMA: fp8 weight tile [128 rows x 128 B] + bf16 token tile into
//               stage s (full_bar[s]), after the MMAs of the stage's last use
//               retired (empty_bar[s])
//   warps 6-13  converters, two per TMEM lane quadrant (one K half each): the
//               thread of weight row r converts its 64 fp8 bytes to bf16 times
//               the row group's block scale and stores them into its own TMEM
//               lane of slot t (tcgen05.st), then arrives on cvt_full[t]
//   warp 1      tcgen05.mma with A read from TMEM slot t and the token tile from
//               stage s (8 MMAs of K 16), then commits empty_bar[s] and
//               cvt_empty[t]; after a unit's last block, the accumulator barrier
//   warps 2-5   epilogue from the double-buffered TMEM accumulator
// The converted weights never touch shared memory: per block the SM's shared
// memory carries the fp8 tile in and out once and the token tile.
template <int BN, bool SWIGLU>
__global__ void __launch_bounds__(kXThreads, 1)
    grouped_gemm_w8_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                           GroupedW8Args xa) {
  using C = XCfg<BN>;
  constexpr int S = C::kNL;
  const GroupedArgs& a = xa.g;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sA8 = smem;                   // [S][kA8]
  uint8_t* sB = sA8 + S * C::kA8;        // [S][kB]  bf16 tokens as loaded
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sB + S * C::kB);  // [S]  TMA landed
  uint64_t* empty_bar = full_bar + S;    // [S]  MMAs done with the stage
  uint64_t* cvt_full = empty_bar + S;    // [kXSlots] converted slot written
  uint64_t* cvt_empty = cvt_full + kXSlots;  // [kXSlots] MMAs done with the slot
  uint64_t* tfull_bar = cvt_empty + kXSlots;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_scale = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full_bar) + 512);  // [kXMaxScales]
  __shared__ GUnits gu;
  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < kXSlots; ++i) {
      mbar_init(&cvt_full[i], kXCvtWarps * 32);
      mbar_init(&cvt_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // the row counts and packed rows come from the previous kernel (PDL)
  pdl_trigger();
  pdl_wait();
  gunits_fill(a, gu, BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int units = gu.pref[a.groups];
  const int nkb = xa.nkb;

  if (warp == 0) {
    if (elect_one()) {
      const uint64_t polA = l2_policy_evict_first(), polB = l2_policy_evict_last();
      int s = 0;
      uint32_t ph = 0, issued_mask = 0, issued_ph = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int e, tm, tn, n0, nr;
        if (!gunit(a, gu, u, e, tm, tn, n0, nr, BN)) continue;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1)) {
            set_status(a.status, kStatusMbarTimeout);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[s], C::kA8 + C::kB);
          tma_load_2d_hint(&tmW, &full_bar[s], sA8 + s * C::kA8, kb * kXBK, e * a.N + tm * kXBM, polA);
          tma_load_2d_hint(&tmX, &full_bar[s], sB + s * C::kB, kb * kXBK, n0, polB);
          tma_load_2d_hint(&tmX, &full_bar[s], sB + s * C::kB + BN * 128, kb * kXBK + 64, n0, polB);
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
    const int c = threadIdx.x - 6 * 32;       // 0..255
    const int q = warp & 3;                   // TMEM lane quadrant this warp may access
    const int half = (warp - 6) >> 2;         // which 64 of the block's 128 K columns
    const int r = q * 32 + lane;              // weight row == TMEM lane
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    int s = 0, t = 0;
    uint32_t ph = 0, pht = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      // all converter threads leave together after an abort (the named
      // barriers below need every one of them)
      if (bar_any(2, kXCvtWarps * 32, *abort_flag != 0)) break;
      int e, tm, tn, n0, nr;
      if (!gunit(a, gu, u, e, tm, tn, n0, nr, BN)) continue;
      // this unit's scales: 8 consecutive row groups x nkb blocks, contiguous
      const float* src = xa.scales16 + ((long)e * (a.N >> 4) + (long)tm * 8) * nkb;
      for (int j = c; j < 8 * nkb; j += kXCvtWarps * 32) s_scale[j] = src[j];
      asm volatile("bar.sync 2, %0;" ::"n"(kXCvtWarps * 32) : "memory");
      for (int kb = 0; kb < nkb; ++kb) {
        if (*abort_flag || !mbar_wait(&full_bar[s], ph) || !mbar_wait(&cvt_empty[t], pht ^ 1)) {
          set_status(a.status, kStatusMbarTimeout);
          *abort_flag = 1;
          break;
        }
        const float sc = s_scale[(r >> 4) * nkb + kb];
        const uint8_t* a8 = sA8 + s * C::kA8 + r * 128;
        uint32_t o[32];
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const int cc = half * 4 + qq;  // 16-byte fp8 chunk = 16 k
          const uint4 raw8 = *reinterpret_cast<const uint4*>(a8 + ((cc ^ (r & 7)) << 4));
          const uint32_t w[4] = {raw8.x, raw8.y, raw8.z, raw8.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t lo, hi;
            e4m3x4_to_f16x4_g(w[j], lo, hi);
            o[qq * 8 + 2 * j] = scale_to_bf16x2(lo, sc);      // k = 16 cc + 4 j, +1
            o[qq * 8 + 2 * j + 1] = scale_to_bf16x2(hi, sc);  // k = 16 cc + 4 j + 2, +3
          }
        }
        // column c of the slot holds k = 2c, 2c+1 of this row
        tmem_st32u(tmem_base + lane_addr + kXSlotCol0 + t * 64 + half * 32, o);
        tc_fence_before();
        mbar_arrive(&cvt_full[t]);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
        if (++t == kXSlots) {
          t = 0;
          pht ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = idesc_bf16_f32(kXBM, BN);
      int s = 0, t = 0, i = 0;
      uint32_t ph = 0, pht = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        int e, tm, tn, n0, nr;
        if (!gunit(a, gu, u, e, tm, tn, n0, nr, BN)) continue;
        const int ab = i & 1;
        if (!mbar_wait(&tempty_bar[ab], ((i >> 1) & 1) ^ 1)) {
          set_status(a.status, kStatusMbarTimeout);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + ab * BN;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&cvt_full[t], pht) || !mbar_wait(&full_bar[s], ph)) {
            set_status(a.status, kStatusMbarTimeout);
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint32_t at = tmem_base + kXSlotCol0 + t * 64;
#pragma unroll
          for (int box = 0; box < 2; ++box) {
            const uint64_t db = smem_desc_sw128(smem_u32(sB + s * C::kB + box * (BN * 128)));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_f16_ts(d, at + box * 32 + kk * 8, db + 2 * kk, idesc, (kb > 0 || box > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[s]);
          umma_commit(&cvt_empty[t]);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
          if (++t == kXSlots) {
            t = 0;
            pht ^= 1;
          }
        }
        umma_commit(&tfull_bar[ab]);
        ++i;
      }
    }
  } else {
    // ------------------------------ epilogue (warps 2-5) ---------------------
    const int q = warp & 3;
    const int row = q * 32 + lane;  // weight row within the 128-row tile
    int i = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      int e, tm, tn, n0, nr;
      if (!gunit(a, gu, u, e, tm, tn, n0, nr, BN)) continue;
      const int ab = i & 1;
      if (!mbar_wait(&tfull_bar[ab], (i >> 1) & 1)) {
        set_status(a.status, kStatusMbarTimeout);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + ab * BN;
      const int f = tm * kXBM + row;  // output feature (or gate/up row)
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
      mbar_arrive(&tempty_bar[ab]);
      ++i;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <int BN, bool SW>
void launch_w8g(const CUtensorMap& tw, const CUtensorMap& tx, const GroupedW8Args& a, cudaStream_t st) {
  using C = XCfg<BN>;
  auto k = grouped_gemm_w8_kernel<BN, SW>;
  static bool set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    BWN_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    set[dev & 63] = true;
  }
  const int units = a.g.groups * a.g.tiles_m * a.g.max_tiles_n;
  const int sms = num_sms();
  launch_k(k, dim3(units < sms ? units : sms), dim3(kXThreads), C::kSmem, st, tw, tx, a);
}

}  // namespace

void grouped_gemm_w8(const GroupedW8Problem& p, cudaStream_t st) {
  BWN_CHECK(p.N % kXBM == 0, "grouped_gemm_w8: N_out must be a multiple of 128");
  BWN_CHECK(p.groups <= kGMaxGroups, "grouped_gemm_w8: at most %d groups", kGMaxGroups);
  BWN_CHECK(p.K % 16 == 0, "grouped_gemm_w8: K multiple of 16 (16-byte TMA rows)");
  if (p.swiglu) BWN_CHECK(p.N % 32 == 0, "grouped_gemm_w8: swiglu rows multiple of 32");
  const int nkb = (p.K + kXBK - 1) / kXBK;
  BWN_CHECK(8 * nkb <= kXMaxScales, "grouped_gemm_w8: K too large for the staged scales");
  int bn = 16;
  while (bn < p.max_rows_per_group && bn < 128) bn *= 2;
  if (p.max_rows_per_group > 128) bn = 128;
  CUtensorMap tw, tx;
  make_tmap_2d_u8(&tw, p.W, (long)p.groups * p.N, p.K, p.K, kXBM, kXBK);
  make_tmap_2d_bf16(&tx, p.X, p.rows_total > 0 ? p.rows_total : 1, p.K, p.K, bn, 64);
  GroupedW8Args a{};
  a.g.counts = p.counts;
  a.g.offsets = p.offsets;
  a.g.groups = p.groups;
  a.g.N = p.N;
  a.g.K = p.K;
  a.g.tiles_m = p.N / kXBM;
  a.g.max_tiles_n = (p.max_rows_per_group + bn - 1) / bn;
  a.g.out = p.out;
  a.g.ldo = p.ldo;
  a.g.status = p.status;
  a.g.swiglu_limit = p.swiglu_limit;
  a.scales16 = p.scales16;
  a.nkb = nkb;
  if (a.g.max_tiles_n == 0) return;
  switch (bn) {
    case 16: p.swiglu ? launch_w8g<16, true>(tw, tx, a, st) : launch_w8g<16, false>(tw, tx, a, st); break;
    case 32: p.swiglu ? launch_w8g<32, true>(tw, tx, a, st) : launch_w8g<32, false>(tw, tx, a, st); break;
    case 64: p.swiglu ? launch_w8g<64, true>(tw, tx, a, st) : launch_w8g<64, false>(tw, tx, a, st); break;
    default: p.swiglu ? launch_w8g<128, true>(tw, tx, a, st) : launch_w8g<128, false>(tw, tx, a, st); break;
  }
}

}  // namespace bwn
