// qik_quant.cu -- per-tensor e4m3 quantizers and the prefix-KV slab store.
//
// HBM-bound byte work: 16-byte vector loads/stores, grids sized to a multiple of
// the SM count, one atomic per CTA for the global amax.  Scales are computed on
// the device exactly as the reference's torch expressions evaluate on CUDA:
//   s   = clamp_min(fl32(amax) * fl32(1/448), 1e-12)     (fp8.py:24-26; a CUDA
//         division by a host scalar is a multiplication by its fp32 reciprocal)
//   act:    q = e4m3_rn_satfinite(fl32(x) * inv), inv = 1/s  (fp8.py:39-41)
//   weight: q = e4m3(clamp(fl32(w) / s, -448, 448))          (fp8.py:59, IEEE div)
//   slab V: per (b, h), as weight                              (kv_cache.py:36-42)
// The amax is kept as the fp32 bit pattern of |x|: for non-negative floats the
// unsigned order is the numeric order and NaN patterns sort above +inf, so an
// integer atomicMax reproduces torch.amax including NaN propagation.
#include <mutex>

#include "qik_device.cuh"
#include "qik_host.h"

namespace qik {

// The workspace (QuantWs) and its grid-wide amax exchange are in qik_device.cuh.
constexpr int kQuantThreads = 256;

__device__ __forceinline__ uint32_t block_max_u32(uint32_t v) {
  __shared__ uint32_t red[32];
  v = __reduce_max_sync(0xffffffffu, v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (blockDim.x >> 5) ? red[lane] : 0u;
    v = __reduce_max_sync(0xffffffffu, v);
  }
  return v;  // valid in warp 0
}

// ---------------------------------------------------------------- amax
// bf16: |x| as 16-bit patterns; __vmaxu2 takes the halfword max of two at once.
__global__ void __launch_bounds__(kQuantThreads) amax_bf16_kernel(const uint16_t* __restrict__ x, int64_t n,
                                                                  uint32_t* __restrict__ amax_bits) {
  pdl_wait();
  uint32_t m2 = 0;  // two running halfword maxima
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  int64_t done = 0;
  if (vec) {
    const int64_t nvec = n >> 3;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    int64_t i = tid;
    for (; i + 3 * nthreads < nvec; i += 4 * nthreads) {
      uint4 a = __ldg(xv + i), b = __ldg(xv + i + nthreads), c = __ldg(xv + i + 2 * nthreads),
            d = __ldg(xv + i + 3 * nthreads);
      m2 = __vmaxu2(m2, __vmaxu2(__vmaxu2(a.x & 0x7FFF7FFFu, a.y & 0x7FFF7FFFu),
                                 __vmaxu2(a.z & 0x7FFF7FFFu, a.w & 0x7FFF7FFFu)));
      m2 = __vmaxu2(m2, __vmaxu2(__vmaxu2(b.x & 0x7FFF7FFFu, b.y & 0x7FFF7FFFu),
                                 __vmaxu2(b.z & 0x7FFF7FFFu, b.w & 0x7FFF7FFFu)));
      m2 = __vmaxu2(m2, __vmaxu2(__vmaxu2(c.x & 0x7FFF7FFFu, c.y & 0x7FFF7FFFu),
                                 __vmaxu2(c.z & 0x7FFF7FFFu, c.w & 0x7FFF7FFFu)));
      m2 = __vmaxu2(m2, __vmaxu2(__vmaxu2(d.x & 0x7FFF7FFFu, d.y & 0x7FFF7FFFu),
                                 __vmaxu2(d.z & 0x7FFF7FFFu, d.w & 0x7FFF7FFFu)));
    }
    for (; i < nvec; i += nthreads) {
      uint4 a = __ldg(xv + i);
      m2 = __vmaxu2(m2, __vmaxu2(__vmaxu2(a.x & 0x7FFF7FFFu, a.y & 0x7FFF7FFFu),
                                 __vmaxu2(a.z & 0x7FFF7FFFu, a.w & 0x7FFF7FFFu)));
    }
    done = nvec << 3;
  }
  for (int64_t i = done + tid; i < n; i += nthreads) m2 = __vmaxu2(m2, static_cast<uint32_t>(x[i] & 0x7FFFu));
  uint32_t m = max(m2 & 0xFFFFu, m2 >> 16);
  m = block_max_u32(m);
  if (threadIdx.x == 0 && m != 0u) atomicMax(amax_bits, m << 16);
  pdl_trigger();
}

__global__ void __launch_bounds__(kQuantThreads) amax_f32_kernel(const float* __restrict__ x, int64_t n,
                                                                 uint32_t* __restrict__ amax_bits) {
  uint32_t m = 0;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t done = 0;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
    const int64_t nvec = n >> 2;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    for (int64_t i = tid; i < nvec; i += nthreads) {
      uint4 a = __ldg(xv + i);
      m = max(max(max(m, a.x & 0x7FFFFFFFu), max(a.y & 0x7FFFFFFFu, a.z & 0x7FFFFFFFu)), a.w & 0x7FFFFFFFu);
    }
    done = nvec << 2;
  }
  for (int64_t i = done + tid; i < n; i += nthreads) m = max(m, __float_as_uint(x[i]) & 0x7FFFFFFFu);
  m = block_max_u32(m);
  if (threadIdx.x == 0 && m != 0u) atomicMax(amax_bits, m);
}

__global__ void scale_finalize_kernel(const uint32_t* __restrict__ amax_bits, float* __restrict__ scale_out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) scale_out[0] = scale_from_amax_bits(*amax_bits);
}

// ---------------------------------------------------------------- packs
// Activation: 16 bf16 -> 16 e4m3 per thread iteration (two 16-byte loads, one
// 16-byte store).
// backward: the 16-element vectors are visited from the last one down (same codes).
// For an x its producer has just written in row order and that L2 kept only in part,
// the lines written last are read first, while they are still in L2; a forward walk
// over such an x misses on nearly every line.
__global__ void __launch_bounds__(kQuantThreads) pack_act_kernel(const uint16_t* __restrict__ x, int64_t n,
                                                                 const uint32_t* __restrict__ amax_bits,
                                                                 uint8_t* __restrict__ q,
                                                                 float* __restrict__ scale_out, int backward) {
  pdl_wait();
  const float s = scale_from_amax_bits(__ldg(amax_bits));
  const float inv = act_inverse(s);
  if (blockIdx.x == 0 && threadIdx.x == 0 && scale_out) scale_out[0] = s;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t done = 0;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(q) & 15u) == 0) {
    const int64_t nvec = n >> 4;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    uint4* qv = reinterpret_cast<uint4*>(q);
    for (int64_t k = tid; k < nvec; k += nthreads) {
      const int64_t i = backward ? nvec - 1 - k : k;
      const uint4 a = __ldg(xv + 2 * i), b = __ldg(xv + 2 * i + 1);
      uint4 o;
      o.x = pack8_e4m3(a, inv, o.y);
      o.z = pack8_e4m3(b, inv, o.w);
      qv[i] = o;
    }
    done = nvec << 4;
  }
  for (int64_t i = done + tid; i < n; i += nthreads) {
    const float v = __uint_as_float(static_cast<uint32_t>(x[i]) << 16) * inv;
    q[i] = static_cast<uint8_t>(cvt_e4m3x2(v, 0.0f) & 0xFFu);
  }
  pdl_trigger();
}

// Weight / slab V element: clamp(w / s) then round to e4m3; NaN keeps its sign
// like c10's conversion (after the clamp every other value is finite).
__device__ __forceinline__ uint8_t weight_code(float w, float s) {
  float v = __fdiv_rn(w, s);
  if (v != v) return static_cast<uint8_t>(0x7Fu | ((__float_as_uint(v) >> 24) & 0x80u));
  v = fminf(fmaxf(v, -448.0f), 448.0f);
  return static_cast<uint8_t>(cvt_e4m3x2(v, 0.0f) & 0xFFu);
}

template <typename T>
__device__ __forceinline__ float load_as_f32(const T* p, int64_t i);
template <>
__device__ __forceinline__ float load_as_f32<uint16_t>(const uint16_t* p, int64_t i) {
  return __uint_as_float(static_cast<uint32_t>(__ldg(p + i)) << 16);
}
template <>
__device__ __forceinline__ float load_as_f32<float>(const float* p, int64_t i) {
  return __ldg(p + i);
}

template <typename T>
__global__ void __launch_bounds__(kQuantThreads) pack_weight_kernel(const T* __restrict__ w, int64_t n,
                                                                    const uint32_t* __restrict__ amax_bits,
                                                                    uint8_t* __restrict__ q,
                                                                    float* __restrict__ scale_out) {
  const float s = scale_from_amax_bits(__ldg(amax_bits));
  if (blockIdx.x == 0 && threadIdx.x == 0) scale_out[0] = s;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  // 4 elements per thread iteration, one 4-byte store.
  const int64_t n4 = ((reinterpret_cast<uintptr_t>(q) & 3u) == 0) ? (n >> 2) : 0;
  for (int64_t i = tid; i < n4; i += nthreads) {
    const uint32_t o = static_cast<uint32_t>(weight_code(load_as_f32(w, 4 * i), s)) |
                       (static_cast<uint32_t>(weight_code(load_as_f32(w, 4 * i + 1), s)) << 8) |
                       (static_cast<uint32_t>(weight_code(load_as_f32(w, 4 * i + 2), s)) << 16) |
                       (static_cast<uint32_t>(weight_code(load_as_f32(w, 4 * i + 3), s)) << 24);
    reinterpret_cast<uint32_t*>(q)[i] = o;
  }
  for (int64_t i = (n4 << 2) + tid; i < n; i += nthreads) q[i] = weight_code(load_as_f32(w, i), s);
}

// ---------------------------------------------------------------- slab store
// grid (row chunks, B*H); rows of D contiguous elements.
__global__ void __launch_bounds__(kQuantThreads) kv_amax_kernel(const uint16_t* __restrict__ v, int64_t P, int64_t H,
                                                                int64_t D, int64_t sb, int64_t sp, int64_t sh,
                                                                int rows_per_block, uint32_t* __restrict__ amax_bits) {
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / H, h = bh % H;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  const int64_t p1 = min(P, p0 + rows_per_block);
  const uint16_t* base = v + b * sb + h * sh;
  uint32_t m = 0;
  const int64_t cnt = (p1 - p0) * D;
  for (int64_t e = threadIdx.x; e < cnt; e += blockDim.x) {
    const int64_t p = p0 + e / D, d = e % D;
    m = max(m, static_cast<uint32_t>(base[p * sp + d] & 0x7FFFu));
  }
  m = block_max_u32(m);
  if (threadIdx.x == 0 && m != 0u) atomicMax(amax_bits + bh, m << 16);
}

__global__ void __launch_bounds__(kQuantThreads) kv_store_kernel(
    const uint16_t* __restrict__ k, const uint16_t* __restrict__ v, int64_t P, int64_t H, int64_t D, int64_t k_sb,
    int64_t k_sp, int64_t k_sh, int64_t v_sb, int64_t v_sp, int64_t v_sh, uint16_t* __restrict__ k_layer,
    void* __restrict__ v_layer, int64_t pmax, int v_fp8, const uint32_t* __restrict__ amax_bits,
    float* __restrict__ v_scale_layer, int rows_per_block) {
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / H, h = bh % H;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  const int64_t p1 = min(P, p0 + rows_per_block);
  const uint16_t* kb = k + b * k_sb + h * k_sh;
  const uint16_t* vb = v + b * v_sb + h * v_sh;
  const int64_t dst0 = bh * pmax * D;
  const int64_t cnt = (p1 - p0) * D;
  float s = 1.0f;
  if (v_fp8) {
    s = scale_from_amax_bits(__ldg(amax_bits + bh));
    if (blockIdx.x == 0 && threadIdx.x == 0) v_scale_layer[bh] = s;
  }
  for (int64_t e = threadIdx.x; e < cnt; e += blockDim.x) {
    const int64_t p = p0 + e / D, d = e % D;
    const int64_t dst = dst0 + p * D + d;
    k_layer[dst] = kb[p * k_sp + d];
    const uint16_t vv = vb[p * v_sp + d];
    if (v_fp8)
      static_cast<uint8_t*>(v_layer)[dst] = weight_code(__uint_as_float(static_cast<uint32_t>(vv) << 16), s);
    else
      static_cast<uint16_t*>(v_layer)[dst] = vv;
  }
}

// ---------------------------------------------------------------- single-pass activation quantizer
// One CTA per SM, launched cooperatively (all CTAs resident at once).  Phase 1: each
// CTA streams the first kQfSmemBytes of its contiguous slice into shared memory with
// bulk copies (16 KB chunks, each on its own mbarrier, all issued up front so the
// copy engine keeps the whole slice in flight) while its threads read any remainder of
// the slice with plain loads (8 per thread in flight), then reduces max|x| over the
// chunks as they land.  Its maximum goes to its slot of the workspace, and a grid
// barrier (one 64-bit atomic per CTA; the waits bounded by QIK_WAIT_NS) makes every
// slot visible.  Phase 2: each CTA reduces the slots to the global amax and packs its
// slice, from shared memory where it was kept, so a tensor up to ~33 MB (148 x 224 KB)
// is read from HBM exactly once: 2 B read + 1 B written per element.  A remainder is
// read with an L2 evict-last policy in phase 1 and re-read (from L2 while it stays
// there) with evict-first in phase 2; while a remainder exists the codes are stored
// with evict-first too, so they do not push it out of L2.
// If any CTA's copy or barrier wait gives up, every CTA that sees it writes no codes
// and CTA 0 writes a NaN scale; the workspace must then be zeroed again before reuse.
constexpr int kQfThreads = 512;
constexpr int kQfChunkVecs = 1024;  // 16 KB per bulk copy
constexpr int kQfChunks = 14;
constexpr int kQfSmemVecs = kQfChunkVecs * kQfChunks;
constexpr int kQfSmemBytes = kQfSmemVecs * 16;

__device__ __forceinline__ uint32_t absmax8(uint32_t m2, const uint4 a) {
  return __vmaxu2(m2, __vmaxu2(__vmaxu2(a.x & 0x7FFF7FFFu, a.y & 0x7FFF7FFFu),
                               __vmaxu2(a.z & 0x7FFF7FFFu, a.w & 0x7FFF7FFFu)));
}

__global__ void __launch_bounds__(kQfThreads, 1) quant_act_single_pass_kernel(const uint16_t* __restrict__ x,
                                                                              int64_t n, uint8_t* __restrict__ q,
                                                                              float* __restrict__ scale_out,
                                                                              QuantWs* __restrict__ ws) {
  extern __shared__ __align__(16) uint4 stage[];
  __shared__ __align__(8) uint64_t bars[kQfChunks];
  __shared__ int abort_cta;
  __shared__ uint32_t amax_all;
  const int64_t nvec = n >> 3;
  const int64_t chunk = (nvec + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = min(nvec, static_cast<int64_t>(blockIdx.x) * chunk);
  const int64_t v1 = min(nvec, v0 + chunk);
  const int64_t cnt = v1 - v0;
  const int64_t nkeep = min(cnt, static_cast<int64_t>(kQfSmemVecs));
  const bool has_rem = cnt > nkeep;
  const int nch = static_cast<int>((nkeep + kQfChunkVecs - 1) / kQfChunkVecs);
  const uint4* xv = reinterpret_cast<const uint4*>(x) + v0;
  const uint64_t pol_once = l2_evict_first_policy();
  if (threadIdx.x == 0) {
    abort_cta = 0;
    for (int c = 0; c < nch; ++c) mbar_init(&bars[c], 1);
    fence_mbar_init();
    for (int c = 0; c < nch; ++c) {
      const int64_t a = static_cast<int64_t>(c) * kQfChunkVecs;
      const uint32_t bytes = static_cast<uint32_t>(min(static_cast<int64_t>(kQfChunkVecs), nkeep - a) * 16);
      mbar_arrive_expect_tx(&bars[c], bytes);
      bulk_load_hint(stage + a, xv + a, bytes, &bars[c], pol_once);
    }
  }
  __syncthreads();
  // phase 1: amax of the slice (bf16 |x| as halfword maxima); the remainder beyond
  // shared memory first, so its loads overlap the bulk copies in flight
  uint32_t m2 = 0;
  if (has_rem) {
    // 16 loads of 16 B in flight per thread (128 KB per CTA) keep HBM busy once the
    // bulk copies have landed
    const uint64_t pol_keep = l2_evict_last_policy();
    for (int64_t base = nkeep; base < cnt; base += 16 * kQfThreads) {
      uint4 r[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int64_t i = base + k * kQfThreads + threadIdx.x;
        r[k] = i < cnt ? ld_nc_hint(xv + i, pol_keep) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) m2 = absmax8(m2, r[k]);
    }
  }
  bool ok = true;
  for (int c = 0; c < nch && ok; ++c) {
    ok = mbar_wait(&bars[c], 0, &abort_cta, nullptr);
    const int64_t a = static_cast<int64_t>(c) * kQfChunkVecs;
    const int64_t b = min(a + kQfChunkVecs, nkeep);
    for (int64_t i = a + threadIdx.x; ok && i < b; i += kQfThreads) m2 = absmax8(m2, stage[i]);
  }
  if (blockIdx.x == 0)  // the n % 8 tail elements
    for (int64_t i = (nvec << 3) + threadIdx.x; i < n; i += kQfThreads)
      m2 = __vmaxu2(m2, static_cast<uint32_t>(x[i] & 0x7FFFu));
  uint32_t m = block_max_u32(max(m2 & 0xFFFFu, m2 >> 16)) << 16;
  if (threadIdx.x == 0) {
    if (abort_cta) m = kQuantAbortMark;  // a chunk never landed: poison the amax
    // grid barrier: every CTA is resident (cooperative launch); the wait is bounded
    if (!grid_max_publish_wait(ws, m)) abort_cta = 1;
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // the global amax from every CTA's slot
    const uint32_t g = grid_max_collect(ws);
    if (threadIdx.x == 0) amax_all = abort_cta ? kQuantAbortMark : g;
  }
  __syncthreads();
  if (amax_all == kQuantAbortMark) {  // some CTA's copy or barrier wait gave up
    if (blockIdx.x == 0 && threadIdx.x == 0) scale_out[0] = __int_as_float(0x7fc00000);
    return;
  }
  // phase 2: scale from the complete amax, codes from shared memory (the remainder
  // re-read, from L2 while it is there)
  const float s = scale_from_amax_bits(amax_all);
  const float inv = act_inverse(s);
  if (blockIdx.x == 0 && threadIdx.x == 0) scale_out[0] = s;
  uint2* qv = reinterpret_cast<uint2*>(q) + v0;
  if (has_rem) {
    for (int64_t base = nkeep; base < cnt; base += 8 * kQfThreads) {
      uint4 r[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int64_t i = base + k * kQfThreads + threadIdx.x;
        r[k] = i < cnt ? ld_nc_hint(xv + i, pol_once) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int64_t i = base + k * kQfThreads + threadIdx.x;
        if (i < cnt) {
          uint32_t hi;
          const uint32_t lo = pack8_e4m3(r[k], inv, hi);
          st_v2_hint(qv + i, lo, hi, pol_once);
        }
      }
    }
    for (int64_t i = threadIdx.x; i < nkeep; i += kQfThreads) {
      uint32_t hi;
      const uint32_t lo = pack8_e4m3(stage[i], inv, hi);
      st_v2_hint(qv + i, lo, hi, pol_once);
    }
  } else {
    for (int64_t i = threadIdx.x; i < nkeep; i += kQfThreads) {
      uint32_t hi;
      const uint32_t lo = pack8_e4m3(stage[i], inv, hi);
      qv[i] = make_uint2(lo, hi);
    }
  }
  if (blockIdx.x == 0)
    for (int64_t i = (nvec << 3) + threadIdx.x; i < n; i += kQfThreads) {
      const float v = __uint_as_float(static_cast<uint32_t>(x[i]) << 16) * inv;
      q[i] = static_cast<uint8_t>(cvt_e4m3x2(v, 0.0f) & 0xFFu);
    }
}

// Cooperative launch of the single-pass quantizer.  ws->bar must hold a consistent
// barrier state (zero once, then as each call leaves it); clear_bar zeroes it on the
// stream first (for callers that cannot keep the workspace between calls).
int launch_quant_single_pass(const void* x, int64_t n, uint8_t* q, float* scale_out, QuantWs* ws,
                             cudaStream_t st, bool clear_bar) {
  static std::once_flag attr_once[64];
  int dev = 0;
  QIK_TRY_CUDA(cudaGetDevice(&dev));
  QIK_REQUIRE(dev >= 0 && dev < 64, "qik_quantize_act: device ordinal %d out of range", dev);
  cudaError_t attr_rc = cudaSuccess;
  std::call_once(attr_once[dev], [&] {
    attr_rc = cudaFuncSetAttribute(quant_act_single_pass_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kQfSmemBytes);
  });
  QIK_TRY_CUDA(attr_rc);
  const int64_t nvec = n >> 3;
  int64_t grid = (nvec + 4 * kQfThreads - 1) / (4 * kQfThreads);
  const int64_t sms = min(static_cast<int64_t>(sm_count()), static_cast<int64_t>(kQuantMaxCtas));
  grid = grid < 1 ? 1 : (grid > sms ? sms : grid);
  const int64_t chunk = (nvec + grid - 1) / grid;
  const size_t smem = static_cast<size_t>(chunk < kQfSmemVecs ? chunk : kQfSmemVecs) * 16;
  if (clear_bar) QIK_TRY_CUDA(cudaMemsetAsync(&ws->bar, 0, sizeof(ws->bar), st));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kQfThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QIK_TRY_CUDA(cudaLaunchKernelEx(&cfg, quant_act_single_pass_kernel, static_cast<const uint16_t*>(x), n, q,
                                  scale_out, ws));
  return check_launch("quant_act_single_pass_kernel");
}

static int grid_for(int64_t work_items, int per_thread) {
  const int64_t want = (work_items + static_cast<int64_t>(kQuantThreads) * per_thread - 1) /
                       (static_cast<int64_t>(kQuantThreads) * per_thread);
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  int64_t g = want < cap ? want : cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

int launch_amax(const void* x, int dtype, int64_t n, uint32_t* amax_bits, cudaStream_t st, bool pdl) {
  if (n <= 0) return QIK_OK;
  if (dtype == QIK_DTYPE_BF16) {
    QIK_TRY_CUDA(launch_kernel(amax_bf16_kernel, dim3(grid_for(n, 32)), dim3(kQuantThreads), 0, st, pdl,
                               static_cast<const uint16_t*>(x), n, amax_bits));
  } else {
    amax_f32_kernel<<<grid_for(n, 16), kQuantThreads, 0, st>>>(static_cast<const float*>(x), n, amax_bits);
  }
  return check_launch("amax kernel");
}

int launch_pack_act(const void* x, int64_t n, const uint32_t* amax_bits, uint8_t* q, float* scale_out,
                    cudaStream_t st, bool pdl, bool backward) {
  QIK_TRY_CUDA(launch_kernel(pack_act_kernel, dim3(grid_for(n, 16)), dim3(kQuantThreads), 0, st, pdl,
                             static_cast<const uint16_t*>(x), n, amax_bits, q, scale_out, backward ? 1 : 0));
  return check_launch("pack_act_kernel");
}

}  // namespace qik

using namespace qik;

extern "C" {

size_t qik_quant_workspace_bytes(void) { return sizeof(QuantWs); }

int qik_compute_scale(const void* x, int dtype, int64_t n, float* scale_out, void* ws, void* stream) {
  QIK_REQUIRE(x || n == 0, "qik_compute_scale: x is NULL");
  QIK_REQUIRE(scale_out && ws, "qik_compute_scale: scale_out/ws is NULL");
  QIK_REQUIRE(dtype == QIK_DTYPE_BF16 || dtype == QIK_DTYPE_F32, "qik_compute_scale: dtype must be BF16 or F32");
  QIK_REQUIRE(n >= 0, "qik_compute_scale: negative n");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  QuantWs* w = static_cast<QuantWs*>(ws);
  QIK_TRY_CUDA(cudaMemsetAsync(&w->amax_bits, 0, sizeof(uint32_t), st));
  int rc = launch_amax(x, dtype, n, &w->amax_bits, st, false);
  if (rc) return rc;
  scale_finalize_kernel<<<1, 32, 0, st>>>(&w->amax_bits, scale_out);
  return check_launch("scale_finalize_kernel");
}

int qik_amax(const void* x, int dtype, int64_t n, uint32_t* amax_bits, void* stream) {
  QIK_REQUIRE(x || n == 0, "qik_amax: x is NULL");
  QIK_REQUIRE(amax_bits, "qik_amax: amax_bits is NULL");
  QIK_REQUIRE(dtype == QIK_DTYPE_BF16 || dtype == QIK_DTYPE_F32, "qik_amax: dtype must be BF16 or F32");
  QIK_REQUIRE(n >= 0, "qik_amax: negative n");
  return launch_amax(x, dtype, n, amax_bits, static_cast<cudaStream_t>(stream), false);
}

int qik_quantize_act_from_amax(const void* x, int64_t n, const uint32_t* amax_bits, uint8_t* q, float* scale_out,
                               void* stream) {
  QIK_REQUIRE((x && q) || n == 0, "qik_quantize_act_from_amax: x/q is NULL");
  QIK_REQUIRE(amax_bits, "qik_quantize_act_from_amax: amax_bits is NULL");
  QIK_REQUIRE(n >= 0, "qik_quantize_act_from_amax: negative n");
  // backward: x is typically the output its producer (GEMM, attention, SwiGLU) has just
  // written, and whatever part of it L2 kept is the part written last
  return launch_pack_act(x, n, amax_bits, q, scale_out, static_cast<cudaStream_t>(stream), true, true);
}

static int quantize_act_impl(const void* x, int64_t n, uint8_t* q, float* scale_out, void* ws, cudaStream_t st,
                             bool clear_bar) {
  QuantWs* w = static_cast<QuantWs*>(ws);
  // one pass over HBM (16-byte aligned operands); otherwise an amax pass then a pack pass
  if (aligned16(x) && aligned16(q) && aligned16(ws)) return launch_quant_single_pass(x, n, q, scale_out, w, st, clear_bar);
  QIK_TRY_CUDA(cudaMemsetAsync(&w->amax_bits, 0, sizeof(uint32_t), st));
  int rc = launch_amax(x, QIK_DTYPE_BF16, n, &w->amax_bits, st, false);
  if (rc) return rc;
  return launch_pack_act(x, n, &w->amax_bits, q, scale_out, st, false);
}

int qik_quantize_act(const void* x, int64_t n, uint8_t* q, float* scale_out, void* ws, void* stream) {
  QIK_REQUIRE(ws && scale_out, "qik_quantize_act: ws/scale_out is NULL");
  QIK_REQUIRE((x && q) || n == 0, "qik_quantize_act: x/q is NULL");
  QIK_REQUIRE(n >= 0, "qik_quantize_act: negative n");
  return quantize_act_impl(x, n, q, scale_out, ws, static_cast<cudaStream_t>(stream), false);
}

int qik_quantize_weight(const void* w, int dtype, int64_t n, uint8_t* q, float* scale_out, void* ws, void* stream) {
  QIK_REQUIRE(ws && scale_out, "qik_quantize_weight: ws/scale_out is NULL");
  QIK_REQUIRE((w && q) || n == 0, "qik_quantize_weight: w/q is NULL");
  QIK_REQUIRE(dtype == QIK_DTYPE_BF16 || dtype == QIK_DTYPE_F32, "qik_quantize_weight: dtype must be BF16 or F32");
  QIK_REQUIRE(n >= 0, "qik_quantize_weight: negative n");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  QuantWs* ws_ = static_cast<QuantWs*>(ws);
  QIK_TRY_CUDA(cudaMemsetAsync(&ws_->amax_bits, 0, sizeof(uint32_t), st));
  int rc = launch_amax(w, dtype, n, &ws_->amax_bits, st, false);
  if (rc) return rc;
  const int g = grid_for(n, 4);
  if (dtype == QIK_DTYPE_BF16)
    pack_weight_kernel<uint16_t><<<g, kQuantThreads, 0, st>>>(static_cast<const uint16_t*>(w), n, &ws_->amax_bits,
                                                               q, scale_out);
  else
    pack_weight_kernel<float><<<g, kQuantThreads, 0, st>>>(static_cast<const float*>(w), n, &ws_->amax_bits, q,
                                                            scale_out);
  return check_launch("pack_weight_kernel");
}

int qik_kv_store(const void* k, const void* v, int64_t B, int64_t P, int64_t H, int64_t D, int64_t k_sb,
                 int64_t k_sp, int64_t k_sh, int64_t v_sb, int64_t v_sp, int64_t v_sh, void* k_layer, void* v_layer,
                 int64_t pmax, int v_fp8, float* v_scale_layer, void* ws, void* stream) {
  QIK_REQUIRE(B >= 0 && P >= 0 && H >= 0 && D >= 0, "qik_kv_store: negative size");
  QIK_REQUIRE(P <= pmax, "qik_kv_store: P=%lld exceeds slab capacity %lld", (long long)P, (long long)pmax);
  if (B == 0 || H == 0 || P == 0 || D == 0) return QIK_OK;
  QIK_REQUIRE(k && v && k_layer && v_layer, "qik_kv_store: NULL tensor");
  QIK_REQUIRE(!v_fp8 || (v_scale_layer && ws), "qik_kv_store: fp8 V needs v_scale_layer and ws");
  QIK_REQUIRE(B * H <= 65535, "qik_kv_store: B*H above 65535");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t rows_want = 8192 / D;
  const int rows = static_cast<int>(rows_want < 1 ? 1 : (rows_want > P ? P : rows_want));
  dim3 grid(static_cast<unsigned>((P + rows - 1) / rows), static_cast<unsigned>(B * H));
  uint32_t* amax = static_cast<uint32_t*>(ws);
  if (v_fp8) {
    QIK_TRY_CUDA(cudaMemsetAsync(amax, 0, sizeof(uint32_t) * B * H, st));
    kv_amax_kernel<<<grid, kQuantThreads, 0, st>>>(static_cast<const uint16_t*>(v), P, H, D, v_sb, v_sp, v_sh, rows,
                                                   amax);
    int rc = check_launch("kv_amax_kernel");
    if (rc) return rc;
  }
  kv_store_kernel<<<grid, kQuantThreads, 0, st>>>(static_cast<const uint16_t*>(k), static_cast<const uint16_t*>(v), P,
                                                  H, D, k_sb, k_sp, k_sh, v_sb, v_sp, v_sh,
                                                  static_cast<uint16_t*>(k_layer), v_layer, pmax, v_fp8, amax,
                                                  v_scale_layer, rows);
  return check_launch("kv_store_kernel");
}

}  // extern "C"

// ---------------------------------------------------------------- no-alloc variant
// Scratch of qik_quantize_act_noalloc, for callers that cannot allocate device
// memory.  Host code cannot use the array's name as a device pointer (on the host
// it names a stand-in object), so its device address is looked up once per
// device with cudaGetSymbolAddress, with that device current, and passed to the
// kernels like any workspace.
static __device__ __align__(256) uint8_t qik_noalloc_scratch[QIK_NOALLOC_SCRATCH_BYTES];

namespace qik {
namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {nullptr};

int noalloc_scratch_ptr(void** out) {
  int dev = 0;
  QIK_TRY_CUDA(cudaGetDevice(&dev));
  QIK_REQUIRE(dev >= 0 && dev < 64, "qik_quantize_act_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, qik_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(qik_noalloc_scratch)");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return QIK_OK;
}
}  // namespace
}  // namespace qik

extern "C" int qik_quantize_act_noalloc(const void* x, int64_t n, uint8_t* q, float* scale_out, void* stream) {
  QIK_REQUIRE(scale_out, "qik_quantize_act_noalloc: scale_out is NULL");
  QIK_REQUIRE((x && q) || n == 0, "qik_quantize_act_noalloc: x/q is NULL");
  QIK_REQUIRE(n >= 0, "qik_quantize_act_noalloc: negative n");
  const size_t need = qik_quant_workspace_bytes();
  QIK_REQUIRE(need <= QIK_NOALLOC_SCRATCH_BYTES,
              "qik_quantize_act_noalloc: needs %zu bytes of scratch, the static array holds %d", need,
              QIK_NOALLOC_SCRATCH_BYTES);
  void* ws = nullptr;
  const int rc = qik::noalloc_scratch_ptr(&ws);
  if (rc) return rc;
  // The barrier word is cleared on the stream at the start of every call, so a call
  // that failed earlier leaves nothing behind; the per-CTA slots need no clearing.
  return quantize_act_impl(x, n, q, scale_out, ws, static_cast<cudaStream_t>(stream), true);
}
