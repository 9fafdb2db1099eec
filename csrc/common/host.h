// Host-side helpers shared by every kernel launcher: error checks, driver entry
// points (resolved at run time, so nothing links against libcuda), TMA tensor
// maps, device properties, the host-mapped status word, and the launch
// descriptors the torch bindings fill in.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <stdexcept>
#include <string>

namespace bwn {

[[noreturn]] void fail(const char* file, int line, const char* fmt, ...);

#define BWN_FAIL(...) ::bwn::fail(__FILE__, __LINE__, __VA_ARGS__)
#define BWN_CHECK(cond, ...)          \
  do {                                \
    if (!(cond)) BWN_FAIL(__VA_ARGS__); \
  } while (0)
#define BWN_CUDA_CHECK(expr)                                                        \
  do {                                                                              \
    cudaError_t _e = (expr);                                                        \
    if (_e != cudaSuccess) BWN_FAIL("CUDA error %s: %s", #expr, cudaGetErrorString(_e)); \
  } while (0)

// ---- device info / status -------------------------------------------------
int num_sms();
// Device pointer (into host-mapped pinned memory) of this device's status word.
int* status_dev_ptr();
// Host view of the status word; read after a synchronize.
int status_read();
void status_clear();

// ---- TMA tensor maps --------------------------------------------------------
// 2-D bf16 row-major matrix [rows, cols] with leading dimension `ld` elements;
// box = [box_rows, box_cols] with the 128-byte swizzle (box_cols*2 must be 128).
void make_tmap_2d_bf16(CUtensorMap* m, const void* base, long rows, long cols, long ld, int box_rows,
                       int box_cols);
// Same for an 8-bit element type (fp8 e4m3 weights); box_cols must be 128.
void make_tmap_2d_u8(CUtensorMap* m, const void* base, long rows, long cols, long ld, int box_rows, int box_cols);

// Driver API entry point by name (cudaGetDriverEntryPoint).
void* driver_fn(const char* name);

// ---- GEMM -----------------------------------------------------------------
enum GemmEpilogue : int {
  kEpiBF16 = 0,    // out = bf16(acc)
  kEpiResid = 1,   // out = bf16(acc + resid)
  kEpiSwiGLU = 2,  // out = bf16(silu(gate) * up), gate/up interleaved in blocks of 16
  kEpiF32 = 3,     // out = acc (fp32)
  kEpiSymm = 4,    // bf16 partial into this rank's symmetric buffer slot, then signal every peer
  kEpiSymmNorm = 5,  // kEpiSymm, then (same launch) the NVLS sum over ranks + residual add + RMSNorm (ArTail)
};

// Completion signalling of a fused compute + collective launch: the last CTA to
// finish bumps *epoch and release-stores it into every rank's flag slot.
struct CommSignal {
  unsigned* peer_flags[8] = {nullptr};  // flag array of each rank (slot = this rank)
  int world = 1, rank = 0;
  int* epoch = nullptr;                  // local epoch counter
  int* done_ticket = nullptr;            // grid completion ticket (re-armed)
  const int* sel = nullptr;              // device buffer selector: buffer (*sel & 1)
  long buf_stride = 0;                   // elements between the two alternating buffers
};

// All-gathered A operand: rows [r*rows, (r+1)*rows) of A are written by rank r
// into this rank's copy; the producer waits for flags[r] >= *epoch before
// loading them, and visits this rank's own rows first.
struct AgWait {
  const unsigned* flags = nullptr;
  const int* epoch = nullptr;
  int rows = 0;  // rows per rank, a multiple of 128
  int rank = 0;
  int world = 0;
  unsigned long long limit_ns = 0;
};

// The reduction tail of a kEpiSymmNorm GEMM: once every rank's completion flag
// has arrived, the CTAs read the sum of all ranks' partial rows through the
// multicast address (multimem.ld_reduce), add it to the residual (bf16, in
// place) and write RMSNorm(residual) * (1 + w); the last CTA flips the slot
// selector.
struct ArTail {
  const __nv_bfloat16* mc_base = nullptr;  // multicast address of the two partial slots
  const unsigned* flags = nullptr;         // this rank's flag array (slot r written by rank r)
  int* sel = nullptr;                      // [2]: slot selector, CTA ticket
  __nv_bfloat16* resid = nullptr;
  long ldr = 0;
  const float* w = nullptr;
  __nv_bfloat16* out = nullptr;
  long ldo = 0;
  int rows = 0, cols = 0;
  float eps = 1e-6f;
  unsigned long long limit_ns = 0;
};

struct GemmProblem {
  // D[M, N] = A[M, K] . B[N, K]^T ; A, B bf16 K-major
  const void* A = nullptr;
  long lda = 0;
  const void* B = nullptr;
  long ldb = 0;
  int M = 0, N = 0, K = 0;
  void* out = nullptr;
  long ldo = 0;
  bool trans_out = false;  // store D^T (out[n, m]); used for swap-AB decode GEMMs
  bool a_mn = false;       // A stored [K, M] (MN-major) instead of [M, K]
  bool b_mn = false;       // B stored [K, N] (MN-major) instead of [N, K]
  int epi = kEpiBF16;
  const __nv_bfloat16* resid = nullptr;
  long ldr = 0;
  int bn = 0;  // 0 = pick from N
  bool allow_split = true;
  float* workspace = nullptr;
  long workspace_floats = 0;
  int* tickets = nullptr;
  int tickets_len = 0;
  int* status = nullptr;
  CommSignal sig;  // kEpiSymm / kEpiSymmNorm
  AgWait ag;       // A all-gathered by peers (normal orientation only)
  ArTail tail;     // kEpiSymmNorm only
};

void gemm_bf16(const GemmProblem& p, cudaStream_t stream);
int gemm_pick_bn(int n);

}  // namespace bwn
