// Chunked gated delta rule on the tensor cores (sm_100a): the reference's
// chunked DeltaNet prefill kernels (contrib/qwen3.6-27b/kernels/deltanet_chunked_v2.py:49-139,
// contrib/qwen3.6-35b-a3b/kernels/deltanet_chunked_prefill_35b.py:78-1002) and
// their oracle (the chunk rule of bwn/ops/reference.py).
//
// One CTA per (sequence, V-head) stream; 64-token chunks in sequence.  For a
// chunk with keys K, queries Q (normalised, scaled), values V, gates beta and
// cumulative log-decay G (G_C its last entry):
//   A  = strict_lower(-beta_i exp(G_i - G_j) k_i.k_j)      T = (I - A)^-1
//   U  = T (beta V)        W = T (beta e^G K)
//   Vn = U - W S           P = lower(exp(G_i - G_j) q_i.k_j)
//   O  = (e^G Q) S + P Vn   S' = e^G_C S + (e^(G_C - G) K)^T Vn
// Every product runs on tcgen05 with the value / key dimension (128) on the
// TMEM lanes ("transposed" orientation), so the fp32 state S^T, V-new^T and the
// outputs O^T live in tensor memory:
//   (a) [Q;K] K^T             one M=128 MMA: rows 0-63 Q K^T, rows 64-127 K K^T
//   (c) U^T = (bV)^T T^T,  W^T = (b e^G K)^T T^T            bf16, fp32 TMEM
//   (d) V-new^T = U^T + S^T (-W)^T    accumulated into U^T  bf16 (S^T copy)
//   (e) O^T = S^T (e^G Q)^T + V-new^T P^T                   bf16 + tf32, A of the
//                                                           second from TMEM
//   (f) S'^T = e^G_C S^T + V-new^T (e^(G_C-G) K)            tf32, A from TMEM,
//                                                           accumulated into S^T
// The triangular solve is forward substitution in fp32 on the CUDA cores (four
// threads per column).  The state stays fp32 in TMEM for the whole prompt; a
// bf16 copy in shared memory is the A operand of (d) and (e).
//
// Warp roles (10 warps): warp 0 TMA (Q, K, V tiles of a chunk, prefetched
// while the previous chunk finishes), warp 1 MMA issuer + TMEM owner, warps
// 2-9 compute (transposes, masks, the solve, TMEM epilogues; warps 2-5 own the
// four TMEM lane quadrants).  Every wait is bounded; on a timeout the kernel
// sets the status word, skips the rest and frees its TMEM.
#include "common/host.h"
#include "common/launch.cuh"
#include "common/sm100.cuh"
#include "kernels/prefill.h"

namespace bwn {

namespace {
constexpr int kC = 64;        // chunk length
constexpr int kD = 128;       // head dim (k and v)
constexpr int kThreads = 320;
constexpr int kCompute = 256;  // warps 2-9

// shared memory map (bytes from the 1024-aligned base); every MMA operand is a
// K-major SW128 tile: rows of 128 bytes in 8-row 1024-byte atoms, one "box"
// per 128 bytes of K
constexpr int kOffQK = 0;                    // bf16 [128 rows][128]: Q rows 0-63, K rows 64-127 (2 boxes x 16 KB)
constexpr int kOffV = kOffQK + 32768;        // bf16 [64][128] (2 boxes x 8 KB)
constexpr int kOffVbT = kOffV + 16384;       // bf16 [128 v][64 j]  (beta V)^T
constexpr int kOffKbT = kOffVbT + 16384;     // bf16 [128 d][64 j]  (beta e^G K)^T
constexpr int kOffKtT = kOffKbT + 16384;     // fp32 [128 d][64 j]  (e^(G_C-G) K)^T (2 boxes x 16 KB)
constexpr int kOffT = kOffKtT + 32768;       // bf16 [64 i][64 j]   T
constexpr int kOffP = kOffT + 8192;          // fp32 [64 i][64 j]   P (2 boxes x 8 KB)
constexpr int kOffW = kOffP + 16384;         // bf16 [64 i][128 d]  -W (2 boxes x 8 KB)
constexpr int kOffS = kOffW + 16384;         // bf16 [128 v][128 d] S^T (2 boxes x 16 KB)
constexpr int kOffA = kOffS + 32768;         // fp32 [64][65] A (solve); then bf16 [64 i][128 d] e^G Q (MMA B)
constexpr int kOffTf = kOffA + 64 * 65 * 4;  // fp32 [64][65] T (solve)
constexpr int kOffVec = kOffTf + 64 * 65 * 4;  // G, beta, e^G, e^(G_C-G): 4 x 64 fp32; norm partials [4][64]
constexpr int kOffBar = kOffVec + 8 * 64 * 4;
constexpr int kSmemBytes = kOffBar + 256 + 1024;

// TMEM columns
constexpr uint32_t kTa = 0, kTu = 64, kTw = 128, kTo = 192, kTs = 256;

// byte offset of element (r, c) in a K-major SW128 tile of `eb`-byte elements
// whose boxes (128 bytes of K each) are `box_bytes` apart
__device__ __forceinline__ int swz(int r, int c, int eb, int box_bytes) {
  const int per = 128 / eb;  // elements per 128-byte row
  const int box = c / per, cc = c % per;
  const int byte = cc * eb;
  return box * box_bytes + r * 128 + ((((byte >> 4) ^ (r & 7))) << 4) + (byte & 15);
}

__device__ __forceinline__ bool wait_or_flag(uint64_t* bar, uint32_t parity, volatile int* abort, int* status) {
  if (*abort) return false;
  if (!mbar_wait(bar, parity)) {
    set_status(status, kStatusMbarTimeout);
    *abort = 1;
    return false;
  }
  return true;
}
}  // namespace

template <typename StateT>
__global__ void __launch_bounds__(kThreads, 1)
    dn_chunk_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, DnPrefillArgs p, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  float* sG = reinterpret_cast<float*>(sm + kOffVec);
  float* sBeta = sG + 64;
  float* sEg = sBeta + 64;
  float* sEgc = sEg + 64;                       // e^(G_C - G_j)
  float* sNorm = sEgc + 64;                     // [4 warps][64 tokens] partial sums of squares
  float* sA = reinterpret_cast<float*>(sm + kOffA);
  float* sTf = reinterpret_cast<float*>(sm + kOffTf);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint64_t* bar_tma = bars + 0;   // TMA landed (tx)
  uint64_t* bar_free = bars + 1;  // compute done with the Q/K/V tiles (1 arrival)
  uint64_t* bar_a = bars + 2;     // MMA (a) retired
  uint64_t* bar_T = bars + 3;     // T, (bV)^T, (b e^G K)^T, e^G Q, (e^(G_C-G) K)^T, P written (1 arrival)
  uint64_t* bar_c = bars + 4;     // MMA (c) retired
  uint64_t* bar_W = bars + 5;     // -W written, S^T scaled by e^G_C (1 arrival)
  uint64_t* bar_d = bars + 6;     // MMA (d), (e1) retired
  uint64_t* bar_f = bars + 7;     // MMA (e2), (f) retired
  uint64_t* bar_S = bars + 8;     // S^T bf16 copy written for the next chunk (1 arrival)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int h = blockIdx.x, b = blockIdx.y;
  const int warp = warp_id(), lane = lane_id();
  const int rep = p.v_heads / p.k_heads, kh = h / rep;
  const long qk_row0 = ((long)b * p.k_heads + kh) * p.S_pad;
  const long v_row0 = ((long)b * p.v_heads + h) * p.S_pad;
  const int nchunks = (p.S + kC - 1) / kC;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 10; ++i) mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (elect_one()) {
      int issued = 0;
      for (int c = 0; c < nchunks && !*abort_flag; ++c) {
        if (c > 0 && !wait_or_flag(bar_free, (c - 1) & 1, abort_flag, status)) break;
        ++issued;
        mbar_arrive_expect_tx(bar_tma, 3 * kC * kD * 2);
        const int r0 = c * kC;
        for (int bx = 0; bx < 2; ++bx) {
          tma_load_2d(&tmQ, bar_tma, sm + kOffQK + bx * 16384, bx * 64, (int)(qk_row0 + r0));
          tma_load_2d(&tmK, bar_tma, sm + kOffQK + bx * 16384 + 8192, bx * 64, (int)(qk_row0 + r0));
          tma_load_2d(&tmV, bar_tma, sm + kOffV + bx * 8192, bx * 64, (int)(v_row0 + r0));
        }
      }
      // drain: the last issued load must land before the CTA leaves
      if (*abort_flag && issued > 0) mbar_wait(bar_tma, (issued - 1) & 1, 100000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (elect_one()) {
      const uint32_t id_a = idesc_bf16_f32(128, 64);
      const uint32_t id_n64 = idesc_bf16_f32(128, 64);
      const uint32_t id_tf64 = idesc_tf32_f32(128, 64);
      const uint32_t id_tf128 = idesc_tf32_f32(128, 128);
      for (int c = 0; c < nchunks; ++c) {
        const uint32_t ph = c & 1;
        // (a) [Q;K] K^T
        if (!wait_or_flag(bar_tma, ph, abort_flag, status)) break;
        tc_fence_after();
        for (int bx = 0; bx < 2; ++bx) {
          const uint64_t da = smem_desc_sw128(smem_u32(sm + kOffQK + bx * 16384));
          const uint64_t db = smem_desc_sw128(smem_u32(sm + kOffQK + bx * 16384 + 8192));
          for (int kk = 0; kk < 4; ++kk) umma_f16(tmem + kTa, da + 2 * kk, db + 2 * kk, id_a, (bx | kk) ? 1u : 0u);
        }
        umma_commit(bar_a);
        // (c) U^T = (bV)^T T^T, W^T = (b e^G K)^T T^T
        if (!wait_or_flag(bar_T, ph, abort_flag, status)) break;
        tc_fence_after();
        {
          const uint64_t dt = smem_desc_sw128(smem_u32(sm + kOffT));
          const uint64_t dv = smem_desc_sw128(smem_u32(sm + kOffVbT));
          const uint64_t dk = smem_desc_sw128(smem_u32(sm + kOffKbT));
          for (int kk = 0; kk < 4; ++kk) umma_f16(tmem + kTu, dv + 2 * kk, dt + 2 * kk, id_n64, kk ? 1u : 0u);
          for (int kk = 0; kk < 4; ++kk) umma_f16(tmem + kTw, dk + 2 * kk, dt + 2 * kk, id_n64, kk ? 1u : 0u);
        }
        umma_commit(bar_c);
        // (d) V-new^T = U^T + S^T (-W)^T ;  (e1) O^T = S^T (e^G Q)^T
        if (!wait_or_flag(bar_W, ph, abort_flag, status)) break;
        if (c > 0 && !wait_or_flag(bar_S, (c - 1) & 1, abort_flag, status)) break;
        tc_fence_after();
        for (int bx = 0; bx < 2; ++bx) {
          const uint64_t ds = smem_desc_sw128(smem_u32(sm + kOffS + bx * 16384));
          const uint64_t dw = smem_desc_sw128(smem_u32(sm + kOffW + bx * 8192));
          const uint64_t dq = smem_desc_sw128(smem_u32(sm + kOffA + bx * 8192));
          for (int kk = 0; kk < 4; ++kk) umma_f16(tmem + kTu, ds + 2 * kk, dw + 2 * kk, id_n64, 1u);
          for (int kk = 0; kk < 4; ++kk) umma_f16(tmem + kTo, ds + 2 * kk, dq + 2 * kk, id_n64, (bx | kk) ? 1u : 0u);
        }
        umma_commit(bar_d);
        // (e2) O^T += V-new^T P^T ; (f) S^T += V-new^T (e^(G_C-G) K), A from TMEM (V-new^T)
        if (!wait_or_flag(bar_d, ph, abort_flag, status)) break;
        tc_fence_after();
        for (int kk = 0; kk < 8; ++kk) {  // K = 64 tokens, 8 per instruction
          const int bx = kk >> 2, off = (kk & 3) * 2;
          const uint64_t dp = smem_desc_sw128(smem_u32(sm + kOffP + bx * 8192)) + off;
          const uint64_t dk = smem_desc_sw128(smem_u32(sm + kOffKtT + bx * 16384)) + off;
          umma_tf32_ts(tmem + kTo, tmem + kTu + kk * 8, dp, id_tf64, 1u);
          umma_tf32_ts(tmem + kTs, tmem + kTu + kk * 8, dk, id_tf128, 1u);
        }
        umma_commit(bar_f);
      }
      if (*abort_flag) {  // every issued MMA retires before the TMEM is freed
        umma_commit(bars + 9);
        mbar_wait(bars + 9, 0, 100000000ull);
      }
    }
  } else {
    // ------------------------------ compute warps -----------------------------
    const int ct = threadIdx.x - 64;  // 0..255
    const bool tmem_warp = warp < 6;  // warps 2-5: one TMEM lane quadrant each
    const int q = warp & 3;
    const int row = q * 32 + lane;    // TMEM lane of this thread (warps 2-5)
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    StateT* gS = reinterpret_cast<StateT*>(p.state) + ((long)b * p.v_heads + h) * kD * kD;
    auto cbar = [] { asm volatile("bar.sync 1, 256;" ::: "memory"); };
    // a bounded wait of every compute thread; they leave together (the named
    // barriers need all 256) if any of them gave up
    auto cwait = [&](uint64_t* bar, uint32_t parity) {
      const bool ok = wait_or_flag(bar, parity, abort_flag, status);
      return !bar_any(1, kCompute, !ok);
    };
    // initial state: S^T (lane v, column d) into TMEM, bf16 copy into smem
    if (tmem_warp) {
      float sv[32];
      for (int c0 = 0; c0 < kD; c0 += 32) {
        for (int j = 0; j < 32; ++j) sv[j] = to_f(gS[(long)(c0 + j) * kD + row]);
        tmem_st32(tmem + lane_addr + kTs + c0, sv);
        for (int j = 0; j < 32; j += 8) {
          alignas(16) __nv_bfloat16 o8[8];
          for (int e = 0; e < 8; ++e) o8[e] = __float2bfloat16(sv[j + e]);
          *reinterpret_cast<uint4*>(sm + kOffS + swz(row, c0 + j, 2, 16384)) = *reinterpret_cast<uint4*>(o8);
        }
      }
      tc_fence_before();
    }
    fence_async_smem();
    cbar();
    for (int c = 0; c < nchunks; ++c) {
      const uint32_t ph = c & 1;
      const int t0 = c * kC;
      // ---- gates: cumulative log-decay G, beta, exponentials ----
      if (ct < 32) {
        const long gi = v_row0 + t0 + 2 * ct;
        const float g0 = p.g_out[gi], g1 = p.g_out[gi + 1];
        float s2 = g0 + g1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float n = __shfl_up_sync(0xffffffffu, s2, o);
          if (ct >= o) s2 += n;
        }
        sG[2 * ct] = s2 - g1;
        sG[2 * ct + 1] = s2;
        sBeta[2 * ct] = p.beta_out[gi];
        sBeta[2 * ct + 1] = p.beta_out[gi + 1];
      }
      cbar();
      if (ct < 64) {
        sEg[ct] = __expf(sG[ct]);
        sEgc[ct] = __expf(sG[kC - 1] - sG[ct]);
      }
      if (!cwait(bar_tma, ph)) break;
      cbar();
      // ---- transposes of the chunk's K and V (bf16 tiles from TMA) ----
      {
        const int col = ct & 127;  // v (threads 0-127) or d (128-255)
        if (ct < 128) {
          for (int j0 = 0; j0 < kC; j0 += 8) {
            alignas(16) __nv_bfloat16 o8[8];
            for (int e = 0; e < 8; ++e) {
              const int j = j0 + e;
              const float v = __bfloat162float(
                  *reinterpret_cast<const __nv_bfloat16*>(sm + kOffV + swz(j, col, 2, 8192)));
              o8[e] = __float2bfloat16(sBeta[j] * v);
            }
            *reinterpret_cast<uint4*>(sm + kOffVbT + swz(col, j0, 2, 16384)) = *reinterpret_cast<uint4*>(o8);
          }
        } else {
          for (int j0 = 0; j0 < kC; j0 += 8) {
            alignas(16) __nv_bfloat16 o8[8];
            float f8[8];
            for (int e = 0; e < 8; ++e) {
              const int j = j0 + e;
              const float k = __bfloat162float(
                  *reinterpret_cast<const __nv_bfloat16*>(sm + kOffQK + swz(64 + j, col, 2, 16384)));
              o8[e] = __float2bfloat16(sBeta[j] * sEg[j] * k);
              f8[e] = sEgc[j] * k;
            }
            *reinterpret_cast<uint4*>(sm + kOffKbT + swz(col, j0, 2, 16384)) = *reinterpret_cast<uint4*>(o8);
            *reinterpret_cast<float4*>(sm + kOffKtT + swz(col, j0, 4, 16384)) = make_float4(f8[0], f8[1], f8[2], f8[3]);
            *reinterpret_cast<float4*>(sm + kOffKtT + swz(col, j0 + 4, 4, 16384)) =
                make_float4(f8[4], f8[5], f8[6], f8[7]);
          }
        }
      }
      // ---- masks of [Q;K] K^T: P (fp32 operand) and A (fp32, for the solve) ----
      if (!cwait(bar_a, ph)) break;
      tc_fence_after();
      if (tmem_warp) {
        float v[64];
        tmem_ld32(tmem + lane_addr + kTa, *reinterpret_cast<float(*)[32]>(v));
        tmem_ld32(tmem + lane_addr + kTa + 32, *reinterpret_cast<float(*)[32]>(v + 32));
        if (row < kC) {  // P row i = row
          const int i = row;
          const float gi = sG[i];
#pragma unroll
          for (int j0 = 0; j0 < kC; j0 += 4) {
            float o4[4];
            for (int e = 0; e < 4; ++e) {
              const int j = j0 + e;
              o4[e] = j <= i ? __expf(gi - sG[j]) * v[j] : 0.f;
            }
            *reinterpret_cast<float4*>(sm + kOffP + swz(i, j0, 4, 8192)) = make_float4(o4[0], o4[1], o4[2], o4[3]);
          }
        } else {  // A row i = row - 64
          const int i = row - kC;
          const float gi = sG[i], bi = sBeta[i];
#pragma unroll
          for (int j = 0; j < kC; ++j) sA[i * 65 + j] = j < i ? -bi * __expf(gi - sG[j]) * v[j] : 0.f;
        }
        tc_fence_before();
      }
      cbar();
      // ---- T = (I - A)^-1 by forward substitution (fp32), four threads per column ----
      {
        const int col = ct >> 2, qq = ct & 3;
        for (int i = 0; i < kC; ++i) {
          float part = 0.f;
          if (i > col)
            for (int j = col + 1 + qq; j < i; j += 4) part += sA[i * 65 + j] * sTf[j * 65 + col];
          part += __shfl_xor_sync(0xffffffffu, part, 1);
          part += __shfl_xor_sync(0xffffffffu, part, 2);
          if (qq == 0) sTf[i * 65 + col] = i == col ? 1.f : (i > col ? sA[i * 65 + col] + part : 0.f);
          __syncwarp();
        }
      }
      cbar();
      // T (bf16 operand); e^G Q (bf16 operand, over the dead A); chunk inputs consumed
      for (int idx = ct; idx < kC * kC / 8; idx += kCompute) {
        const int i = idx >> 3, j0 = (idx & 7) * 8;
        alignas(16) __nv_bfloat16 o8[8];
        for (int e = 0; e < 8; ++e) o8[e] = __float2bfloat16(sTf[i * 65 + j0 + e]);
        *reinterpret_cast<uint4*>(sm + kOffT + swz(i, j0, 2, 8192)) = *reinterpret_cast<uint4*>(o8);
      }
      for (int idx = ct; idx < kC * kD / 8; idx += kCompute) {
        const int i = idx >> 4, d0 = (idx & 15) * 8;
        const uint4 qv = *reinterpret_cast<const uint4*>(sm + kOffQK + swz(i, d0, 2, 16384));
        const __nv_bfloat16* q8 = reinterpret_cast<const __nv_bfloat16*>(&qv);
        alignas(16) __nv_bfloat16 o8[8];
        for (int e = 0; e < 8; ++e) o8[e] = __float2bfloat16(__bfloat162float(q8[e]) * sEg[i]);
        *reinterpret_cast<uint4*>(sm + kOffA + swz(i, d0, 2, 8192)) = *reinterpret_cast<uint4*>(o8);
      }
      fence_async_smem();
      cbar();
      if (ct == 0) {
        mbar_arrive(bar_T);
        mbar_arrive(bar_free);  // the TMA may load the next chunk into the Q/K/V tiles
      }
      // ---- -W (bf16 operand) from W^T; S^T *= e^G_C in TMEM ----
      if (!cwait(bar_c, ph)) break;
      tc_fence_after();
      if (tmem_warp) {
        float w[64];
        tmem_ld32(tmem + lane_addr + kTw, *reinterpret_cast<float(*)[32]>(w));
        tmem_ld32(tmem + lane_addr + kTw + 32, *reinterpret_cast<float(*)[32]>(w + 32));
#pragma unroll
        for (int i = 0; i < kC; ++i)  // lane d writes column d of -W [i][d]
          *reinterpret_cast<__nv_bfloat16*>(sm + kOffW + swz(i, row, 2, 8192)) = __float2bfloat16(-w[i]);
        const float egc = __expf(sG[kC - 1]);
        for (int c0 = 0; c0 < kD; c0 += 32) {
          float sv[32];
          tmem_ld32(tmem + lane_addr + kTs + c0, sv);
          for (int j = 0; j < 32; ++j) sv[j] *= egc;
          tmem_st32(tmem + lane_addr + kTs + c0, sv);
        }
        tc_fence_before();
      }
      fence_async_smem();
      cbar();
      if (ct == 0) mbar_arrive(bar_W);
      // ---- outputs: O^T (lane v, column i) -> gated RMSNorm -> out; S^T copy ----
      if (!cwait(bar_f, ph)) break;
      tc_fence_after();
      if (tmem_warp) {
        float o[64];
        tmem_ld32(tmem + lane_addr + kTo, *reinterpret_cast<float(*)[32]>(o));
        tmem_ld32(tmem + lane_addr + kTo + 32, *reinterpret_cast<float(*)[32]>(o + 32));
#pragma unroll
        for (int i = 0; i < kC; ++i) {
          const float ss = warp_sum(o[i] * o[i]);
          if (lane == 0) sNorm[q * 64 + i] = ss;
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");
        const float nw = p.norm_w[row];
#pragma unroll
        for (int i = 0; i < kC; ++i) {
          const int t = t0 + i;
          if (t >= p.S) continue;
          const float tot = sNorm[i] + sNorm[64 + i] + sNorm[128 + i] + sNorm[192 + i];
          const float inv = rsqrtf(tot / kD + p.norm_eps);
          const float z = __bfloat162float(p.z[((long)b * p.S + t) * p.z_row + h * kD + row]);
          p.out[((long)b * p.S + t) * p.out_row + h * kD + row] = __float2bfloat16(o[i] * inv * nw * silu_f(z));
        }
        for (int c0 = 0; c0 < kD; c0 += 32) {
          float sv[32];
          tmem_ld32(tmem + lane_addr + kTs + c0, sv);
          for (int j = 0; j < 32; j += 8) {
            alignas(16) __nv_bfloat16 o8[8];
            for (int e = 0; e < 8; ++e) o8[e] = __float2bfloat16(sv[j + e]);
            *reinterpret_cast<uint4*>(sm + kOffS + swz(row, c0 + j, 2, 16384)) = *reinterpret_cast<uint4*>(o8);
          }
        }
        tc_fence_before();
      }
      fence_async_smem();
      cbar();
      if (ct == 0) mbar_arrive(bar_S);
    }
    // final state back to global
    if (tmem_warp && !*abort_flag) {
      tc_fence_after();
      for (int c0 = 0; c0 < kD; c0 += 32) {
        float sv[32];
        tmem_ld32(tmem + lane_addr + kTs + c0, sv);
        for (int j = 0; j < 32; ++j) gS[(long)(c0 + j) * kD + row] = from_f<StateT>(sv[j]);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool deltanet_chunk_tc_supported(const DnPrefillArgs& p) { return p.S_pad % kC == 0 && p.v_heads % p.k_heads == 0; }

void deltanet_chunk_tc(const DnPrefillArgs& p, int* status, cudaStream_t stream) {
  CUtensorMap tq, tk, tv;
  make_tmap_2d_bf16(&tq, p.q_out, (long)p.batch * p.k_heads * p.S_pad, kD, kD, kC, 64);
  make_tmap_2d_bf16(&tk, p.k_out, (long)p.batch * p.k_heads * p.S_pad, kD, kD, kC, 64);
  make_tmap_2d_bf16(&tv, p.v_out, (long)p.batch * p.v_heads * p.S_pad, kD, kD, kC, 64);
  static bool set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    BWN_CUDA_CHECK(cudaFuncSetAttribute(dn_chunk_tc_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kSmemBytes));
    BWN_CUDA_CHECK(cudaFuncSetAttribute(dn_chunk_tc_kernel<__nv_bfloat16>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    set[dev & 63] = true;
  }
  const dim3 grid(p.v_heads, p.batch);
  if (p.state_bf16)
    dn_chunk_tc_kernel<__nv_bfloat16><<<grid, kThreads, kSmemBytes, stream>>>(tq, tk, tv, p, status);
  else
    dn_chunk_tc_kernel<float><<<grid, kThreads, kSmemBytes, stream>>>(tq, tk, tv, p, status);
  BWN_CUDA_CHECK(cudaGetLastError());
}

}  // namespace bwn
