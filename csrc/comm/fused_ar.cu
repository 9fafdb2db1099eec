// Fused collective kernels over NVLink / NVSwitch for tensor parallelism.
//
// Row-parallel projections (o_proj, out_proj, down_proj) are followed by an
// all-reduce in the reference (functional_all_reduce after every row-parallel
// GEMM, contrib/qwen3.6-27b/static_decode.py:798-961; static_decode_35b.py:1972,
// 2110, 1278).  Here it is a one-shot reduction through the switch:
//
//  * the tcgen05 GEMM epilogue (csrc/kernels/gemm_tc.cu, kEpiSymm) stores its
//    bf16 partial into this rank's slot of a symmetric buffer pair -- plain
//    local stores -- and its last CTA release-stores an epoch flag into every
//    rank's flag array; symm_put_signal_kernel does the same for a partial
//    already in memory (MoE output);
//  * ar_add_norm_kernel waits (bounded) for every rank's flag, reads the sum of
//    all ranks' partials with multimem.ld_reduce on the multicast address (the
//    NVSwitch adds the eight copies with fp32 accumulation, 16 bytes per
//    request), adds the residual, RMSNorm(1+w)s the row, and flips the slot
//    selector once all its CTAs have read;
//  * greedy_allmax_kernel exchanges per-rank packed (logit, id) argmax keys by
//    peer stores and takes the max: the sharded greedy of
//    static_decode_35b.py:1534-1564 in one launch.
// Two slots alternate under a device-side selector so a CUDA graph replays the
// same launches; a slot is rewritten only after every rank has passed the next
// flag barrier, i.e. after every rank finished reading it.  Every wait gives up
// after a bounded time and sets a status bit instead of hanging the GPU.
#include <climits>

#include "comm/fused.h"
#include "comm/signal.cuh"
#include "common/host.h"
#include "common/launch.cuh"
#include "common/sm100.cuh"

namespace bwn {

// Thread r (< world) waits for rank r's flag to reach `epoch`; all ranks' flags
// are polled in parallel.  Callers follow with a CTA barrier.
__device__ __forceinline__ bool wait_flag_lane(const unsigned* flags, int world, unsigned epoch, int* status,
                                               uint64_t limit_ns) {
  const int r = threadIdx.x;
  if (r >= world) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while ((int)(ld_acquire_sys(flags + r) - epoch) < 0) {
    if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) {
      set_status(status, kStatusPeerTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ bool wait_flags(const unsigned* flags, int world, unsigned epoch, int* status,
                                           uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (int r = 0; r < world; ++r) {
    uint32_t spins = 0;
    while ((int)(ld_acquire_sys(flags + r) - epoch) < 0) {
      if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) {
        set_status(status, kStatusPeerTimeout);
        return false;
      }
    }
  }
  return true;
}

__global__ void __launch_bounds__(256) symm_put_signal_kernel(const __nv_bfloat16* __restrict__ x, long ldx, int rows,
                                                              int cols, __nv_bfloat16* local_base, CommSignal sig) {
  pdl_trigger();
  pdl_wait();
  __nv_bfloat16* dst = local_base + (long)((*sig.sel) & 1) * sig.buf_stride;
  const int c8 = cols >> 3;
  const long n = (long)rows * c8;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long r = i / c8, c = (i % c8) * 8;
    *reinterpret_cast<uint4*>(dst + r * cols + c) = *reinterpret_cast<const uint4*>(x + r * ldx + c);
  }
  __syncthreads();  // the CTA's stores precede thread 0's system-scope fence in signal_done
  if (threadIdx.x == 0) signal_done(sig);
}

__global__ void __launch_bounds__(256) ar_add_norm_kernel(const __nv_bfloat16* mc_base, long buf_stride, int* sel,
                                                          const unsigned* flags, int world, const int* epoch,
                                                          __nv_bfloat16* __restrict__ resid, long ldr,
                                                          const float* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                                          long ldo, int cols, float eps, int* status,
                                                          unsigned long long limit_ns) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  __shared__ float red[8];
  const bool arrived = wait_flag_lane(flags, world, (unsigned)(*epoch), status, limit_ns);
  // a peer that never signalled: its partial may not exist, so nothing is read
  // or written (the status word carries the timeout to the host)
  if (!__syncthreads_and(arrived)) return;
  const __nv_bfloat16* buf = mc_base + (long)((*sel) & 1) * buf_stride + (long)row * cols;
  constexpr int kMaxVec = 4;  // 8 columns per vector, 256 threads: cols <= 8192
  float v[kMaxVec][8];
  float ss = 0.f;
  // issue every reduction load first so their switch round trips overlap
#pragma unroll
  for (int n = 0; n < kMaxVec; ++n) {
    const int c = (threadIdx.x + n * blockDim.x) * 8;
    if (c < cols) mc_ld_reduce_bf16x8(buf + c, v[n]);
  }
#pragma unroll
  for (int n = 0; n < kMaxVec; ++n) {
    const int c = (threadIdx.x + n * blockDim.x) * 8;
    if (c >= cols) continue;
    const uint4 rr = *reinterpret_cast<const uint4*>(resid + (long)row * ldr + c);
    const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rr);
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 rf = __bfloat1622float2(r2[e]);
      const __nv_bfloat162 nb = __floats2bfloat162_rn(rf.x + v[n][2 * e], rf.y + v[n][2 * e + 1]);
      o2[e] = nb;
      const float2 nf = __bfloat1622float2(nb);
      v[n][2 * e] = nf.x;
      v[n][2 * e + 1] = nf.y;
      ss += nf.x * nf.x + nf.y * nf.y;
    }
    *reinterpret_cast<uint4*>(resid + (long)row * ldr + c) = o;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = rsqrtf(tot / cols + eps);
#pragma unroll
  for (int n = 0; n < kMaxVec; ++n) {
    const int c = (threadIdx.x + n * blockDim.x) * 8;
    if (c >= cols) continue;
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e)
      o2[e] = __floats2bfloat162_rn(v[n][2 * e] * inv * (1.f + w[c + 2 * e]), v[n][2 * e + 1] * inv * (1.f + w[c + 2 * e + 1]));
    *reinterpret_cast<uint4*>(out + (long)row * ldo + c) = o;
  }
  // flip the slot selector once every CTA has read it: last CTA (ticket)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int t = atomicAdd(sel + 1, 1);
    if (t == (int)gridDim.x - 1) {
      sel[1] = 0;
      sel[0] = sel[0] + 1;
    }
  }
}

// One CTA per token: the partial rows of every rank summed through the switch
// (multimem.ld_reduce, fp32), rounded to bf16 as the unfused all-reduce output
// is, then DeepSeek V4's hyper-connection post-mix of the residual streams
// (hc_post of csrc/kernels/deepseek.cu; the reference's all-reduce followed by
// hc_post, contrib/deepseek-v4-flash/run_deepseek_v4_tp.py:541-556, 564-583).
template <int HC, int kMaxVec>  // kMaxVec: 8-column vectors per thread, cols <= 2048 * kMaxVec
__global__ void __launch_bounds__(256) ar_hc_post_kernel(ArHcArgs a) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int cols = a.cols;
  __shared__ float s_post[HC], s_comb[HC * HC];
  if (threadIdx.x < HC) s_post[threadIdx.x] = a.post[(long)t * HC + threadIdx.x];
  if (threadIdx.x < HC * HC) s_comb[threadIdx.x] = a.comb[(long)t * HC * HC + threadIdx.x];
  const bool arrived = wait_flag_lane(a.flags, a.world, (unsigned)(*a.epoch), a.status, a.limit_ns);
  // (the barrier also publishes s_post / s_comb)  a timed-out wait reads and writes nothing
  if (!__syncthreads_and(arrived)) return;
  const __nv_bfloat16* buf = a.mc_base + (long)((*a.sel) & 1) * a.buf_stride + (long)t * cols;
  float v[kMaxVec][8];
#pragma unroll
  for (int n = 0; n < kMaxVec; ++n) {
    const int c = (threadIdx.x + n * blockDim.x) * 8;
    if (c < cols) mc_ld_reduce_bf16x8(buf + c, v[n]);
  }
#pragma unroll
  for (int n = 0; n < kMaxVec; ++n) {
    const int c = (threadIdx.x + n * blockDim.x) * 8;
    if (c >= cols) continue;
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = __bfloat162float(__float2bfloat16(v[n][e]));
    // acc[j] = post[j] * x + sum_i comb[i][j] * resid[i], one residual stream live at a time
    float acc[HC][8];
#pragma unroll
    for (int j = 0; j < HC; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[j][e] = s_post[j] * x[e];
#pragma unroll
    for (int i = 0; i < HC; ++i) {
      const uint4 rr = *reinterpret_cast<const uint4*>(a.resid + ((long)t * HC + i) * cols + c);
      const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rr);
      float r[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(r2[e]);
        r[2 * e] = f.x;
        r[2 * e + 1] = f.y;
      }
#pragma unroll
      for (int j = 0; j < HC; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[j][e] += s_comb[i * HC + j] * r[e];
    }
#pragma unroll
    for (int j = 0; j < HC; ++j) {
      uint4 w;
      __nv_bfloat162* w2 = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
      for (int e = 0; e < 4; ++e) w2[e] = __floats2bfloat162_rn(acc[j][2 * e], acc[j][2 * e + 1]);
      *reinterpret_cast<uint4*>(a.out + ((long)t * HC + j) * cols + c) = w;
    }
  }
  // flip the slot selector once every CTA has read it: last CTA (ticket)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int tk = atomicAdd(a.sel + 1, 1);
    if (tk == (int)gridDim.x - 1) {
      a.sel[1] = 0;
      a.sel[0] = a.sel[0] + 1;
    }
  }
}

// One CTA per shard row: (sum of every rank's partial row through the switch |
// a local addend) + residual -> RMSNorm(1+w) -> multicast store of the normed
// row into every rank's gathered buffer; the last CTA flips the partial slot
// and publishes the gather flag.  The next column-parallel GEMM waits for that
// flag per owner before reading the owner's rows (gemm_tc.cu, AgWait).
__global__ void __launch_bounds__(256) sp_norm_gather_kernel(SpNormArgs a) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  const int cols = a.cols;
  const long grow = (long)a.rank * a.rows + i;
  __shared__ float red[8];
  const bool arrived = !a.mc_partial || wait_flag_lane(a.flags, a.world, (unsigned)(*a.epoch), a.status, a.limit_ns);
  if (!__syncthreads_and(arrived)) return;  // timed out: read and write nothing
  constexpr int kMaxVec = 4;
  float v[kMaxVec][8];
#pragma unroll
  for (int n = 0; n < kMaxVec; ++n) {
    const int c = (threadIdx.x + n * blockDim.x) * 8;
    if (c >= cols) continue;
    if (a.mc_partial) {
      mc_ld_reduce_bf16x8(a.mc_partial + (long)((*a.sel) & 1) * a.buf_stride + grow * cols + c, v[n]);
    } else {
      const uint4 p = *reinterpret_cast<const uint4*>(a.local_partial + (long)i * a.ldp + c);
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&p);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(p2[e]);
        v[n][2 * e] = f.x;
        v[n][2 * e + 1] = f.y;
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int n = 0; n < kMaxVec; ++n) {
    const int c = (threadIdx.x + n * blockDim.x) * 8;
    if (c >= cols) continue;
    __nv_bfloat16* xr = a.x + (long)i * a.ldx + c;
    const uint4 rr = *reinterpret_cast<const uint4*>(xr);
    const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rr);
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 rf = __bfloat1622float2(r2[e]);
      const __nv_bfloat162 nb = __floats2bfloat162_rn(rf.x + v[n][2 * e], rf.y + v[n][2 * e + 1]);
      o2[e] = nb;
      const float2 nf = __bfloat1622float2(nb);
      v[n][2 * e] = nf.x;
      v[n][2 * e + 1] = nf.y;
      ss += nf.x * nf.x + nf.y * nf.y;
    }
    *reinterpret_cast<uint4*>(xr) = o;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int k = 0; k < (int)(blockDim.x >> 5); ++k) tot += red[k];
  const float inv = rsqrtf(tot / cols + a.eps);
#pragma unroll
  for (int n = 0; n < kMaxVec; ++n) {
    const int c = (threadIdx.x + n * blockDim.x) * 8;
    if (c >= cols) continue;
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = v[n][e] * inv * (1.f + a.w[c + e]);
    mc_st_bf16x8(a.h_mc + grow * cols + c, o);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int t = atomicAdd(a.ticket, 1);
    if (t == (int)gridDim.x - 1) {
      *a.ticket = 0;
      if (a.mc_partial) a.sel[0] = a.sel[0] + 1;
      fence_acq_rel_sys();
      const unsigned e = (unsigned)(*a.ag_epoch) + 1u;
      *a.ag_epoch = (int)e;
      for (int r = 0; r < a.world; ++r) st_relaxed_sys_u32(a.ag_peer_flags[r] + a.rank, e);
    }
  }
}

void sp_norm_gather(const SpNormArgs& a, cudaStream_t st) {
  BWN_CHECK(a.cols % 8 == 0 && a.cols <= 256 * 8 * 4, "sp_norm_gather: hidden must be a multiple of 8, at most 8192");
  BWN_CHECK(a.world >= 1 && a.world <= 8 && a.rows > 0, "sp_norm_gather: bad shape");
  launch_k(sp_norm_gather_kernel, dim3(a.rows), dim3(256), 0, st, a);
}

__global__ void greedy_allmax_kernel(GreedyArgs a) {
  pdl_trigger();
  pdl_wait();
  const int64_t* keys = a.keys;
  const int rows = a.rows, world = a.world, rank = a.rank;
  int64_t* const* peer_slots = a.peer_slots;
  unsigned* const* peer_flags = a.peer_flags;
  const unsigned* flags = a.flags;
  int* epoch = a.epoch;
  int* ids_out = a.ids_out;
  int* status = a.status;
  const unsigned long long limit_ns = a.limit_ns;
  // one CTA: scatter this rank's keys into every rank's slot [rank][rows]
  for (int r = 0; r < world; ++r)
    for (int i = threadIdx.x; i < rows; i += blockDim.x) {
      unsigned long long* dst = reinterpret_cast<unsigned long long*>(peer_slots[r]) + (long)rank * rows + i;
      asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst), "l"((unsigned long long)keys[i]) : "memory");
    }
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    const unsigned e = (unsigned)(*epoch) + 1u;
    *epoch = (int)e;
    for (int r = 0; r < world; ++r) st_release_sys(peer_flags[r] + rank, e);
    wait_flags(flags, world, e, status, limit_ns);
  }
  __syncthreads();
  const unsigned long long* mine = reinterpret_cast<const unsigned long long*>(peer_slots[rank]);
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    long long best = LLONG_MIN;  // keys order as signed int64 (argmax_packed)
    for (int r = 0; r < world; ++r) {
      unsigned long long k;
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(k) : "l"(mine + (long)r * rows + i) : "memory");
      best = (long long)k > best ? (long long)k : best;
    }
    ids_out[i] = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
  }
}

void symm_put_signal(const __nv_bfloat16* x, long ldx, int rows, int cols, __nv_bfloat16* local_base,
                     const CommSignal& sig, cudaStream_t st) {
  BWN_CHECK(cols % 8 == 0 && ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0,
            "symm_put_signal: 16-byte aligned rows");
  const long n = (long)rows * cols / 8;
  int grid = (int)std::min<long>((n + 255) / 256, num_sms());
  if (grid < 1) grid = 1;
  launch_k(symm_put_signal_kernel, dim3(grid), dim3(256), 0, st, x, ldx, rows, cols, local_base, sig);
}

void ar_add_norm(const ArNormArgs& a, cudaStream_t st) {
  BWN_CHECK(a.cols % 8 == 0 && a.cols <= 256 * 8 * 4, "ar_add_norm: hidden must be a multiple of 8, at most 8192");
  BWN_CHECK(a.ldr % 8 == 0 && a.ldo % 8 == 0, "ar_add_norm: 16-byte aligned rows");
  launch_k(ar_add_norm_kernel, dim3(a.rows), dim3(256), 0, st, a.mc_base, a.buf_stride, a.sel, a.flags, a.world,
           a.epoch, a.resid, a.ldr, a.w, a.out, a.ldo, a.cols, a.eps, a.status, a.limit_ns);
}

void ar_hc_post(const ArHcArgs& a, cudaStream_t st) {
  BWN_CHECK(a.hc == 4, "ar_hc_post: hc_mult 4 supported");
  BWN_CHECK(a.cols % 8 == 0 && a.cols <= 256 * 8 * 4, "ar_hc_post: dim must be a multiple of 8, at most 8192");
  // as few register vectors as the row needs (DeepSeek V4 Flash, dim 4096: two)
  if (a.cols <= 2048)
    launch_k(ar_hc_post_kernel<4, 1>, dim3(a.rows), dim3(256), 0, st, a);
  else if (a.cols <= 4096)
    launch_k(ar_hc_post_kernel<4, 2>, dim3(a.rows), dim3(256), 0, st, a);
  else
    launch_k(ar_hc_post_kernel<4, 4>, dim3(a.rows), dim3(256), 0, st, a);
}

void greedy_allmax(const GreedyArgs& a, cudaStream_t st) {
  BWN_CHECK(a.world >= 1 && a.world <= 8, "greedy_allmax: world size 1..8");
  launch_k(greedy_allmax_kernel, dim3(1), dim3(256), 0, st, a);
}

}  // namespace bwn
