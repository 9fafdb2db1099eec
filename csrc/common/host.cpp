#include "common/host.h"

#include <cstdarg>
#include <mutex>

namespace bwn {

void fail(const char* file, int line, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  char msg[1200];
  snprintf(msg, sizeof(msg), "[bwn] %s (%s:%d)", buf, file, line);
  throw std::runtime_error(msg);
}

static constexpr int kMaxDev = 64;

int num_sms() {
  static int cache[kMaxDev] = {0};
  int dev = 0;
  BWN_CUDA_CHECK(cudaGetDevice(&dev));
  if (!cache[dev]) {
    int v = 0;
    BWN_CUDA_CHECK(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
    cache[dev] = v;
  }
  return cache[dev];
}

static int* g_status_host[kMaxDev] = {nullptr};
static int* g_status_dev[kMaxDev] = {nullptr};
static std::mutex g_status_mu;

static void status_init(int dev) {
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (g_status_host[dev]) return;
  int* h = nullptr;
  BWN_CUDA_CHECK(cudaHostAlloc(reinterpret_cast<void**>(&h), 64, cudaHostAllocMapped | cudaHostAllocPortable));
  *h = 0;
  int* d = nullptr;
  BWN_CUDA_CHECK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d), h, 0));
  g_status_host[dev] = h;
  g_status_dev[dev] = d;
}

int* status_dev_ptr() {
  int dev = 0;
  BWN_CUDA_CHECK(cudaGetDevice(&dev));
  if (!g_status_host[dev]) status_init(dev);
  return g_status_dev[dev];
}

int status_read() {
  int dev = 0;
  BWN_CUDA_CHECK(cudaGetDevice(&dev));
  if (!g_status_host[dev]) return 0;
  return *reinterpret_cast<volatile int*>(g_status_host[dev]);
}

void status_clear() {
  int dev = 0;
  BWN_CUDA_CHECK(cudaGetDevice(&dev));
  if (g_status_host[dev]) *reinterpret_cast<volatile int*>(g_status_host[dev]) = 0;
}

void* driver_fn(const char* name) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  BWN_CUDA_CHECK(cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q));
  BWN_CHECK(fn != nullptr && q == cudaDriverEntryPointSuccess, "driver entry point %s not found", name);
  return fn;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn f = nullptr;
  if (!f) f = reinterpret_cast<EncodeTiledFn>(driver_fn("cuTensorMapEncodeTiled"));
  return f;
}

static void make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, long rows, long cols,
                         long ld, int box_rows, int box_cols) {
  BWN_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  BWN_CHECK((ld * esize) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  BWN_CHECK(box_cols * esize == 128, "TMA box inner extent must be 128 bytes for SWIZZLE_128B");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * esize)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  BWN_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d): rows=%ld cols=%ld ld=%ld box=%dx%d", (int)r,
            rows, cols, ld, box_rows, box_cols);
}

void make_tmap_2d_bf16(CUtensorMap* m, const void* base, long rows, long cols, long ld, int box_rows, int box_cols) {
  make_tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, rows, cols, ld, box_rows, box_cols);
}

void make_tmap_2d_u8(CUtensorMap* m, const void* base, long rows, long cols, long ld, int box_rows, int box_cols) {
  make_tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, rows, cols, ld, box_rows, box_cols);
}

}  // namespace bwn
