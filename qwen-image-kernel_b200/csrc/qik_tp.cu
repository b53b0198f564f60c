// qik_tp.cu -- row-parallel reduction over peer memory for the tensor-parallel block
// stack (one process per GPU, NVLink peers mapped with CUDA IPC).
//
// The row-parallel linears of the TP stack (attention-out, FFN-down) each produce an
// fp32 partial product per rank that must be summed over the ranks.  Instead of a
// GEMM followed by an NCCL all-reduce, qik_fp8_gemm_scatter (qik_gemm.cu) stores each
// finished tile of the partial product straight into the receive slot of the rank
// that owns those rows, while the GEMM goes on with the next tile.  Then:
//   tp_reduce_gather_kernel  the owner waits for every rank's tiles of its rows, sums
//                            them in rank order (the order of a 2-rank all-reduce:
//                            fp32 addition of two terms commutes), adds the bias and
//                            stores the bf16 rows into every rank's output;
//   tp_wait_kernel           each rank waits for every owner's rows.
// Release / acquire at system scope: the writer's stores, a CTA barrier, one
// __threadfence_system and a system-scope atomic add; the reader polls with
// ld.acquire.sys and passes a CTA barrier.  Every poll is bounded by QIK_WAIT_NS and
// records QIK_DEV_TIMEOUT in the status word when it gives up.
#include <string.h>

#include "qik_device.cuh"
#include "qik_host.h"

namespace qik {
namespace {

constexpr int kTpThreads = 256;

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Polls until every counter reached target (signed 32-bit distance, so the counters may
// wrap); false after QIK_WAIT_NS.
__device__ bool wait_counters(const uint32_t* cnt, int n, uint32_t target, int* status) {
  const uint64_t t0 = globaltimer();
  for (int i = 0; i < n; ++i) {
    for (uint32_t it = 0;; ++it) {
      if (static_cast<int32_t>(ld_acquire_sys(cnt + i) - target) >= 0) break;
      if ((it & 255u) == 255u && globaltimer() - t0 > QIK_WAIT_NS) {
        if (status) atomicExch(status, QIK_DEV_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}

struct ReduceArgs {
  const float* recv;  // world slots of R x N fp32 (this owner's receive area, one call parity)
  const uint32_t* cnt_in;
  uint32_t cnt_target;
  int world, owner, M, N, R;
  const __nv_bfloat16* bias;
  __nv_bfloat16* out[QIK_TP_MAX_WORLD];
  uint32_t* gcnt[QIK_TP_MAX_WORLD];
  int* status;
};

__global__ void __launch_bounds__(kTpThreads) tp_reduce_gather_kernel(const ReduceArgs a) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) ok_s = wait_counters(a.cnt_in, a.world, a.cnt_target, a.status) ? 1 : 0;
  __syncthreads();
  if (ok_s) {
    const int row0 = a.owner * a.R;
    const int rows = max(0, min(a.R, a.M - row0));
    const int64_t groups = static_cast<int64_t>(rows) * (a.N / 8);  // 8 columns per thread step
    const int64_t slot = static_cast<int64_t>(a.R) * a.N;
    for (int64_t gi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gi < groups;
         gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int64_t r = gi / (a.N / 8);
      const int c = static_cast<int>(gi - r * (a.N / 8)) * 8;
      const float* src = a.recv + r * a.N + c;
      float acc[8];
      {
        const float4 u = __ldcg(reinterpret_cast<const float4*>(src));
        const float4 v = __ldcg(reinterpret_cast<const float4*>(src + 4));
        acc[0] = u.x, acc[1] = u.y, acc[2] = u.z, acc[3] = u.w, acc[4] = v.x, acc[5] = v.y, acc[6] = v.z, acc[7] = v.w;
      }
      for (int s = 1; s < a.world; ++s) {
        const float4 u = __ldcg(reinterpret_cast<const float4*>(src + s * slot));
        const float4 v = __ldcg(reinterpret_cast<const float4*>(src + s * slot + 4));
        acc[0] += u.x, acc[1] += u.y, acc[2] += u.z, acc[3] += u.w;
        acc[4] += v.x, acc[5] += v.y, acc[6] += v.z, acc[7] += v.w;
      }
      if (a.bias) {
        const uint4 bb = __ldg(reinterpret_cast<const uint4*>(a.bias + c));
        const uint32_t bw[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          acc[2 * t] += __uint_as_float(bw[t] << 16);
          acc[2 * t + 1] += __uint_as_float(bw[t] & 0xFFFF0000u);
        }
      }
      const uint4 w = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                 pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
      const int64_t off = (row0 + r) * static_cast<int64_t>(a.N) + c;
      for (int p = 0; p < a.world; ++p) *reinterpret_cast<uint4*>(a.out[p] + off) = w;
    }
  }
  // every CTA counts itself at every rank (also after a timeout, so the others' waits
  // end on their own limit rather than on a missing arrival of this one)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < a.world; ++p) atomicAdd_system(a.gcnt[p], 1u);
  }
}

// out = bf16(x + bias) for the rows of x [rows, N] fp32 (this rank's rows of a summed
// row-parallel product), and max|out| into *amax_out (fp32 bits, atomic max) for the
// next FP8 linear's dynamic scale.  8 columns per thread step.
__global__ void __launch_bounds__(kTpThreads) rows_bias_bf16_kernel(const float* __restrict__ x, int64_t rows, int N,
                                                                    const __nv_bfloat16* __restrict__ bias,
                                                                    __nv_bfloat16* __restrict__ out,
                                                                    uint32_t* __restrict__ amax_out) {
  const int64_t groups = rows * (N / 8);
  uint32_t m2 = 0;
  for (int64_t gi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gi < groups;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = gi / (N / 8);
    const int c = static_cast<int>(gi - r * (N / 8)) * 8;
    const float4 u = __ldcs(reinterpret_cast<const float4*>(x + r * N + c));
    const float4 v = __ldcs(reinterpret_cast<const float4*>(x + r * N + c + 4));
    float acc[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
    if (bias) {
      const uint4 bb = __ldg(reinterpret_cast<const uint4*>(bias + c));
      const uint32_t bw[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        acc[2 * t] += __uint_as_float(bw[t] << 16);
        acc[2 * t + 1] += __uint_as_float(bw[t] & 0xFFFF0000u);
      }
    }
    const uint4 w = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                               pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
    m2 = __vmaxu2(m2, __vmaxu2(__vmaxu2(w.x & 0x7FFF7FFFu, w.y & 0x7FFF7FFFu),
                               __vmaxu2(w.z & 0x7FFF7FFFu, w.w & 0x7FFF7FFFu)));
    *reinterpret_cast<uint4*>(out + r * N + c) = w;
  }
  if (amax_out) {
    const uint32_t m = __reduce_max_sync(0xffffffffu, max(m2 & 0xFFFFu, m2 >> 16));
    if ((threadIdx.x & 31) == 0 && m != 0u) atomicMax(amax_out, m << 16);
  }
}

__global__ void tp_wait_kernel(const uint32_t* gcnt, uint32_t target, int world, int* status) {
  if (threadIdx.x == 0) {
    wait_counters(gcnt, world, target, status);
    __threadfence_system();
  }
}

}  // namespace
}  // namespace qik

using namespace qik;

extern "C" size_t qik_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int qik_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  QIK_REQUIRE(ptr && handle_out && offset_out, "qik_ipc_export: NULL argument");
  cudaIpcMemHandle_t h;
  QIK_TRY_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)));
  CUdeviceptr base = 0;
  size_t size = 0;
  // the allocation's base: through the runtime's driver entry point (no -lcuda)
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  QIK_TRY_CUDA(cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q));
  QIK_REQUIRE(fn && q == cudaDriverEntryPointSuccess, "qik_ipc_export: cuMemGetAddressRange unavailable");
  using Fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  const CUresult r = reinterpret_cast<Fn>(fn)(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  QIK_REQUIRE(r == CUDA_SUCCESS, "qik_ipc_export: cuMemGetAddressRange failed (%d)", static_cast<int>(r));
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return QIK_OK;
}

extern "C" int qik_ipc_open(const void* handle, void** base_out) {
  QIK_REQUIRE(handle && base_out, "qik_ipc_open: NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  QIK_TRY_CUDA(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess));
  return QIK_OK;
}

extern "C" int qik_ipc_close(void* base) {
  QIK_REQUIRE(base, "qik_ipc_close: NULL base");
  QIK_TRY_CUDA(cudaIpcCloseMemHandle(base));
  return QIK_OK;
}

extern "C" int qik_tp_reduce_gather(const float* recv, const uint32_t* cnt_in, uint32_t cnt_target, int world,
                                    int owner, int64_t M, int64_t N, int64_t rows_per_owner, const void* bias,
                                    void* const* out, uint32_t* const* gcnt, int ctas, int* status, void* stream) {
  QIK_REQUIRE(world >= 1 && world <= QIK_TP_MAX_WORLD && owner >= 0 && owner < world,
              "qik_tp_reduce_gather: owner %d / world %d out of range", owner, world);
  QIK_REQUIRE(recv && cnt_in && out && gcnt, "qik_tp_reduce_gather: NULL argument");
  QIK_REQUIRE(M > 0 && N > 0 && N % 8 == 0 && rows_per_owner > 0 && rows_per_owner * world >= M &&
                  M <= (1ll << 31) - 1 && rows_per_owner * N <= (1ll << 40),
              "qik_tp_reduce_gather: bad sizes (N a multiple of 8, world x rows per owner >= M)");
  QIK_REQUIRE(ctas >= 1 && ctas <= 65535, "qik_tp_reduce_gather: ctas %d out of range", ctas);
  QIK_REQUIRE(aligned16(recv) && (!bias || aligned16(bias)), "qik_tp_reduce_gather: recv / bias must be 16-byte aligned");
  ReduceArgs a;
  memset(&a, 0, sizeof(a));
  a.recv = recv;
  a.cnt_in = cnt_in;
  a.cnt_target = cnt_target;
  a.world = world;
  a.owner = owner;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.R = static_cast<int>(rows_per_owner);
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  for (int p = 0; p < world; ++p) {
    QIK_REQUIRE(out[p] && gcnt[p] && aligned16(out[p]), "qik_tp_reduce_gather: out[%d] / gcnt[%d] NULL or unaligned",
                p, p);
    a.out[p] = static_cast<__nv_bfloat16*>(out[p]);
    a.gcnt[p] = gcnt[p];
  }
  a.status = status;
  tp_reduce_gather_kernel<<<ctas, kTpThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("tp_reduce_gather_kernel");
}

extern "C" int qik_tp_wait(const uint32_t* gcnt, uint32_t target, int world, int* status, void* stream) {
  QIK_REQUIRE(gcnt && world >= 1 && world <= QIK_TP_MAX_WORLD, "qik_tp_wait: bad arguments");
  tp_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(gcnt, target, world, status);
  return check_launch("tp_wait_kernel");
}

extern "C" int qik_rows_bias_bf16(const float* x, int64_t rows, int64_t N, const void* bias, void* out,
                                  uint32_t* amax_out, void* stream) {
  QIK_REQUIRE(rows >= 0 && N > 0 && N % 8 == 0 && N <= (1ll << 30), "qik_rows_bias_bf16: N=%lld must be a positive "
              "multiple of 8", (long long)N);
  if (rows == 0) return QIK_OK;
  QIK_REQUIRE(x && out, "qik_rows_bias_bf16: NULL x / out");
  QIK_REQUIRE(aligned16(x) && aligned16(out) && (!bias || aligned16(bias)),
              "qik_rows_bias_bf16: x, out and bias must be 16-byte aligned");
  const int64_t groups = rows * (N / 8);
  const int64_t want = (groups + kTpThreads - 1) / kTpThreads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  const int grid = static_cast<int>(want < cap ? want : cap);
  rows_bias_bf16_kernel<<<grid, kTpThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, rows, static_cast<int>(N), static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(out),
      amax_out);
  return check_launch("rows_bias_bf16_kernel");
}
