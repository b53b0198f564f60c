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

}  // namespace qik
