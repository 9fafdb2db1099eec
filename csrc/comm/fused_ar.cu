// Fused collective kernels over NVLink / NVSwitch for tensor parallelism.
//
// Row-parallel projections (o_proj, out_proj, down_proj) are followed by an
// all-reduce in the reference (functional_all_reduce after every row-parallel
// GEMM, contrib/qwen3.6-27b/static_decode.py:798-961; static_decode_35b.py:1972,
// 2110, 1278).  Here the tcgen05 GEMM epilogue reduces its fp32 partial tiles
// straight into an NVLS multicast buffer (multimem.red; csrc/kernels/gemm_tc.cu,
// kEpiMcRed) and publishes an epoch flag to every rank; the kernels below
//
//  * mc_red_signal_kernel  do the same for a partial that is already in memory
//                          (MoE output, embedding), and
//  * ar_add_norm_kernel    wait for all ranks' flags (bounded), add the reduced
//                          row to the residual stream, RMSNorm(1+w) it, and zero
//                          the local copy for its next use (two buffers
//                          alternate under a device-side selector, so a CUDA
//                          graph replays the same launches), and
//  * greedy_allmax_kernel  exchange per-rank packed (logit, id) argmax keys by
//                          peer stores and take the max: the sharded greedy of
//                          static_decode_35b.py:1534-1564 in one launch.
// Every wait gives up after a bounded time and sets a status bit instead of
// hanging the GPU.
#include "comm/fused.h"
#include "common/host.h"
#include "common/launch.cuh"
#include "common/sm100.cuh"

namespace bwn {

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

__device__ __forceinline__ void signal_done(const CommSignal& sig) {
  // caller: one thread per CTA, after a CTA-wide barrier
  fence_acq_rel_sys();
  const int t = atomicAdd(sig.done_ticket, 1);
  if (t == (int)gridDim.x - 1) {
    *sig.done_ticket = 0;
    fence_acq_rel_sys();
    const unsigned e = (unsigned)(*sig.epoch) + 1u;
    *sig.epoch = (int)e;
    for (int r = 0; r < sig.world; ++r) st_release_sys(sig.peer_flags[r] + sig.rank, e);
  }
}

__global__ void __launch_bounds__(256) mc_red_signal_kernel(const __nv_bfloat16* __restrict__ x, long ldx, int rows,
                                                            int cols, float* mc_base, CommSignal sig) {
  pdl_trigger();
  pdl_wait();
  float* mc = mc_base + (long)((*sig.sel) & 1) * sig.buf_stride;
  const long n = (long)rows * cols;
  for (long i = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 2; i < n; i += (long)gridDim.x * blockDim.x * 2) {
    const long r = i / cols, c = i % cols;
    const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(x + r * ldx + c));
    mc_red_add_f32(mc + r * cols + c, v.x);
    mc_red_add_f32(mc + r * cols + c + 1, v.y);
  }
  fence_acq_rel_sys();
  __syncthreads();
  if (threadIdx.x == 0) signal_done(sig);
}

__global__ void __launch_bounds__(256) ar_add_norm_kernel(float* local_base, long buf_stride, int* sel,
                                                          const unsigned* flags, int world, const int* epoch,
                                                          __nv_bfloat16* __restrict__ resid, long ldr,
                                                          const float* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                                          long ldo, int cols, float eps, int* status,
                                                          unsigned long long limit_ns) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  __shared__ float red[8];
  if (threadIdx.x == 0) wait_flags(flags, world, (unsigned)(*epoch), status, limit_ns);
  __syncthreads();
  float* buf = local_base + (long)((*sel) & 1) * buf_stride + (long)row * cols;
  float ss = 0.f;
  constexpr int kMaxPerThread = 32;
  float v[kMaxPerThread];
  int n = 0;
  for (int c = threadIdx.x; c < cols && n < kMaxPerThread; c += blockDim.x, ++n) {
    const float x = __ldcg(buf + c);
    const float r = __bfloat162float(__float2bfloat16(__bfloat162float(resid[(long)row * ldr + c]) + x));
    resid[(long)row * ldr + c] = __float2bfloat16(r);
    buf[c] = 0.f;  // ready for this buffer's next use
    v[n] = r;
    ss += r * r;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = rsqrtf(tot / cols + eps);
  n = 0;
  for (int c = threadIdx.x; c < cols && n < kMaxPerThread; c += blockDim.x, ++n)
    out[(long)row * ldo + c] = __float2bfloat16(v[n] * inv * (1.f + w[c]));
  // flip the buffer selector once every CTA has read it: last CTA (ticket)
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
  fence_acq_rel_sys();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned e = (unsigned)(*epoch) + 1u;
    *epoch = (int)e;
    for (int r = 0; r < world; ++r) st_release_sys(peer_flags[r] + rank, e);
    wait_flags(flags, world, e, status, limit_ns);
  }
  __syncthreads();
  const unsigned long long* mine = reinterpret_cast<const unsigned long long*>(peer_slots[rank]);
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    unsigned long long best = 0;
    for (int r = 0; r < world; ++r) {
      unsigned long long k;
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(k) : "l"(mine + (long)r * rows + i) : "memory");
      best = k > best ? k : best;
    }
    ids_out[i] = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
  }
}

void mc_red_signal(const __nv_bfloat16* x, long ldx, int rows, int cols, float* mc_base, const CommSignal& sig,
                   cudaStream_t st) {
  BWN_CHECK(cols % 2 == 0 && ldx % 2 == 0, "mc_red_signal: even columns");
  long n = (long)rows * cols / 2;
  int grid = (int)std::min<long>((n + 255) / 256, num_sms());
  if (grid < 1) grid = 1;
  launch_k(mc_red_signal_kernel, dim3(grid), dim3(256), 0, st, x, ldx, rows, cols, mc_base, sig);
}

void ar_add_norm(const ArNormArgs& a, cudaStream_t st) {
  BWN_CHECK(a.cols <= 256 * 32, "ar_add_norm: hidden too wide");
  launch_k(ar_add_norm_kernel, dim3(a.rows), dim3(256), 0, st, a.local_base, a.buf_stride, a.sel, a.flags, a.world,
           a.epoch, a.resid, a.ldr, a.w, a.out, a.ldo, a.cols, a.eps, a.status, a.limit_ns);
}

void greedy_allmax(const GreedyArgs& a, cudaStream_t st) {
  BWN_CHECK(a.world >= 1 && a.world <= 8, "greedy_allmax: world size 1..8");
  launch_k(greedy_allmax_kernel, dim3(1), dim3(256), 0, st, a);
}

}  // namespace bwn
