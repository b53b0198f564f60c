// qik_api.cu -- library-wide entry points: version, error reporting, device
// properties, TMA descriptor encoding, and the bounded-wait self-test.
#include <string.h>

#include <mutex>

#include "qik_device.cuh"
#include "qik_host.h"

namespace qik {

namespace {
thread_local char g_err[512] = "";

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

const char* last_error() { return g_err; }

int sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t cols, uint64_t rows,
                 uint64_t row_pitch_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(QIK_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(QIK_ERR_CUDA, "cuTensorMapEncodeTiled(2d) failed (%d): cols=%llu rows=%llu pitch=%llu box=%ux%u",
                     static_cast<int>(r), (unsigned long long)cols, (unsigned long long)rows,
                     (unsigned long long)row_pitch_bytes, box_cols, box_rows);
  return QIK_OK;
}

int make_tmap_nd(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(QIK_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (rank < 1 || rank > 5) return set_error(QIK_ERR_INVALID, "tensor map rank %d out of range", rank);
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, st, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(QIK_ERR_CUDA, "cuTensorMapEncodeTiled(%dd) failed (%d)", rank, static_cast<int>(r));
  return QIK_OK;
}

// One CTA waits on an mbarrier that nothing arrives at; the bounded wait gives up
// after `wait_ns` and records the timeout.
__global__ void selftest_wait_kernel(int* status, uint64_t wait_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer();
    bool done = false;
    while (!done) {
      done = mbar_try_wait(&bar, 0);
      if (!done && globaltimer() - t0 > wait_ns) break;
    }
    atomicExch(status, done ? QIK_DEV_OK : QIK_DEV_TIMEOUT);
  }
}

}  // namespace qik

extern "C" {

int qik_version(void) { return 100; }

const char* qik_last_error(void) { return qik::last_error(); }

int qik_selftest_wait_timeout(int* status, uint64_t wait_ns, void* stream) {
  QIK_REQUIRE(status != nullptr, "qik_selftest_wait_timeout: status is NULL");
  QIK_REQUIRE(wait_ns <= 10ull * 1000 * 1000 * 1000, "qik_selftest_wait_timeout: wait_ns above 10 s");
  qik::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, wait_ns);
  return qik::check_launch("selftest_wait_kernel");
}

}  // extern "C"
