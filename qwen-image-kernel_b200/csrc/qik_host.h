// qik_host.h -- host-side helpers shared by the qik entry points: status codes,
// the per-thread error message, CUDA error mapping and TMA descriptor encoding.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/qik.h"

namespace qik {

int set_error(int code, const char* fmt, ...);
const char* last_error();

// Map a CUDA runtime error to QIK_ERR_CUDA with a message naming the call site.
inline int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return QIK_OK;
  return set_error(QIK_ERR_CUDA, "%s: %s (%d)", what, cudaGetErrorString(e), static_cast<int>(e));
}

#define QIK_TRY_CUDA(call)                                  \
  do {                                                      \
    cudaError_t qik_e_ = (call);                            \
    if (qik_e_ != cudaSuccess) return ::qik::cuda_status(qik_e_, #call); \
  } while (0)

#define QIK_REQUIRE(cond, ...)                                        \
  do {                                                                \
    if (!(cond)) return ::qik::set_error(QIK_ERR_INVALID, __VA_ARGS__); \
  } while (0)

// After a launch: report launch-configuration errors without synchronizing.
inline int check_launch(const char* what) { return cuda_status(cudaGetLastError(), what); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Number of SMs of the current device (cached per device).
int sm_count();

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
// 2-D map over a row-major [rows, cols] matrix with `row_pitch_bytes`, box
// {box_cols, box_rows}, 128-byte swizzle, out-of-bounds elements read as zero.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t cols, uint64_t rows,
                 uint64_t row_pitch_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle);

// rank-D map (dims innermost first, rank <= 5) with byte strides for dims 1..rank-1.
int make_tmap_nd(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// Kernel launch with optional programmatic dependent launch (the kernel may start
// while its stream predecessor finishes; it must call pdl_wait() before reading
// the predecessor's results).
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                          Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Internal launchers shared by the C entry points (pdl: chain onto the previous
// kernel in the stream).
int launch_amax(const void* x, int dtype, int64_t n, uint32_t* amax_bits, cudaStream_t st, bool pdl);
int launch_pack_act(const void* x, int64_t n, const uint32_t* amax_bits, uint8_t* q, float* scale_out,
                    cudaStream_t st, bool pdl, bool backward = false);
// Single-pass activation quantizer (one cooperative kernel; x, q and ws 16-byte aligned):
// ws is its 1 KB workspace (qik_quant_workspace_bytes), whose barrier word must be
// zero before the first call and is left ready for the next call by each call that
// completes; clear_bar zeroes that word on the stream first.
struct QuantWs;
int launch_quant_single_pass(const void* x, int64_t n, uint8_t* q, float* scale_out, QuantWs* ws, cudaStream_t st,
                             bool clear_bar);
int launch_fp8_gemm(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                    const float* scale_a, const float* scale_b, const void* bias, void* C, int64_t ldc, int out_dtype,
                    int epilogue, uint32_t* amax_out, int* status, cudaStream_t st, bool pdl,
                    bool keep_out_l2 = false);

}  // namespace qik
