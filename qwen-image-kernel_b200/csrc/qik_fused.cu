// qik_fused.cu -- the elementwise / normalization kernels of the DiT block.
//
// Restatements of the reference's fused Triton kernels
// (qwen_image_kernel/triton_fused.py) with the same rounding points:
//   rms_norm_rope    per-head RMSNorm (fp32 weight multiply, one bf16 rounding) +
//                    complex RoPE on (even, odd) pairs             (:28-69)
//   layer_norm_mod   LayerNorm without affine, bf16, times bf16(1 + scale) with the
//                    per-position modulation row map              (:111-138)
// The two norms stream their rows through shared memory (bulk copies into a ring,
// see "row streaming"); RMSNorm + RoPE keeps a register-only form for layouts whose
// heads are not contiguous within a token.
//   gate_residual    x + bf16(tanh(gate)) * f                      (:183-209)
//   swiglu           bf16(silu(g)) * up                            (:237-249)
// All four are HBM-bound: 16-byte vector loads and stores, grids a multiple of the
// SM count with grid-stride loops.  Layer norm and SwiGLU can also accumulate the
// amax of their bf16 output (fp32 bit patterns, atomicMax), which is the reduction
// the next FP8 linear's dynamic quantizer needs, so that linear can skip its own
// amax pass (qik_quantize_act_from_amax); the layer norm can also emit that linear's
// e4m3 input itself (ln_modulate_e4m3_kernel, qik_layer_norm_modulate_e4m3).
#include <mutex>

#include "qik_device.cuh"
#include "qik_host.h"

namespace qik {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ uint32_t absmax_bf16x2(uint32_t m, uint32_t w) { return __vmaxu2(m, w & 0x7FFF7FFFu); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ float4 ldg16f(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Block-wide max of u32 values; one atomicMax per CTA into *dst (skipped for 0).
__device__ __forceinline__ void block_atomic_max(uint32_t v, uint32_t* dst) {
  __shared__ uint32_t red[32];
  v = __reduce_max_sync(0xffffffffu, v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (blockDim.x >> 5) ? red[lane] : 0u;
    v = __reduce_max_sync(0xffffffffu, v);
    if (lane == 0 && v != 0u) atomicMax(dst, v);
  }
}

// ---------------------------------------------------------------- RMSNorm + RoPE
// G = D / 8 lanes per (b, s, h) row, 8 consecutive elements (4 rotation pairs) per
// lane; 32 / G rows per warp and kRopeUnroll row groups per warp iteration, whose
// loads (x and the RoPE table rows) are all issued before any arithmetic.  Two groups
// (measured at the t2i shape: 1 -> 34.7 us, 2 -> 30.7, 4 -> 33.8, 8 -> 47.3): more
// groups per warp cost registers, hence resident warps, and lose more than they gain.
constexpr int kRopeUnroll = 2;

template <int G>
__global__ void __launch_bounds__(kThreads) rms_rope_kernel(const uint16_t* __restrict__ x, int64_t x_sb,
                                                            int64_t x_ss, int64_t x_sh, uint16_t* __restrict__ out,
                                                            int64_t o_sb, int64_t o_ss, int64_t o_sh,
                                                            const float* __restrict__ w, const float* __restrict__ cs,
                                                            const float* __restrict__ sn, int64_t S, int64_t H,
                                                            int64_t nrows, float eps) {
  constexpr int D = 8 * G, HALF = D / 2, RPW = 32 / G, U = kRopeUnroll;
  const uint32_t S32 = static_cast<uint32_t>(S), H32 = static_cast<uint32_t>(H);
  const int lane = threadIdx.x & 31;
  const int sub = lane / G, gl = lane % G;
  // weights of this lane's 8 columns: loop invariant
  const float4 w0 = ldg16f(w + gl * 8), w1 = ldg16f(w + gl * 8 + 4);
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t groups = (nrows + RPW - 1) / RPW;
  for (int64_t wg0 = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * U; wg0 < groups;
       wg0 += warps_total * U) {
    uint4 v[U];
    float4 c4[U], s4[U];
    int64_t dst[U];
    bool live[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t row = (wg0 + u) * RPW + sub;
      live[u] = row < nrows;
      const uint32_t r = live[u] ? static_cast<uint32_t>(row) : 0u;  // nrows < 2^31 (host check)
      const uint32_t bs = r / H32, h = r - bs * H32;
      const uint32_t b = bs / S32, s = bs - b * S32;
      v[u] = live[u] ? ldg16(x + b * x_sb + s * x_ss + h * x_sh + gl * 8) : make_uint4(0u, 0u, 0u, 0u);
      c4[u] = ldg16f(cs + static_cast<int64_t>(s) * HALF + gl * 4);
      s4[u] = ldg16f(sn + static_cast<int64_t>(s) * HALF + gl * 4);
      dst[u] = b * o_sb + s * o_ss + h * o_sh + gl * 8;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t uu[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      float xe[4], xo[4];
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        xe[i] = bf_lo(uu[i]);
        xo[i] = bf_hi(uu[i]);
        ss = fmaf(xe[i], xe[i], ss);
        ss = fmaf(xo[i], xo[i], ss);
      }
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rrms = rsqrtf(ss / static_cast<float>(D) + eps);
      const float cv[4] = {c4[u].x, c4[u].y, c4[u].z, c4[u].w}, sv[4] = {s4[u].x, s4[u].y, s4[u].z, s4[u].w};
      uint32_t o4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // fp32 norm, one rounding to bf16, back to fp32 for the rotation
        const float ne = round_bf16((xe[i] * rrms) * wv[2 * i]);
        const float no = round_bf16((xo[i] * rrms) * wv[2 * i + 1]);
        // (e + i o)(c + i s) = (e c - o s) + i (e s + o c)
        o4[i] = pack_bf16x2(ne * cv[i] - no * sv[i], ne * sv[i] + no * cv[i]);
      }
      if (live[u]) *reinterpret_cast<uint4*>(out + dst[u]) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
    }
  }
}

// ---------------------------------------------------------------- row streaming
// Register-resident norms issue a row's loads only when the warp reaches the row, so
// only a few KB per warp are in flight and they wait on memory latency (~0.5 of HBM).
// The streaming forms decouple the loads: one CTA per SM, one producer thread issuing
// bulk copies (cp.async.bulk) of 8-row groups into a ring of shared-memory stages, and
// two sets of 8 consumer warps taking alternate stages, one row of a stage per warp.
// The consumers read their row from shared memory in every pass (mean, variance,
// output), which keeps them at ~40 registers so 16 of them fit beside the producer.  A
// stage is released once its 8 warps arrive on its empty barrier.  Every wait is
// bounded.
constexpr int kStreamWarps = 8;                    // rows per stage = consumer warps per set
constexpr int kStreamSets = 2;                     // consumer sets, taking alternate stages
constexpr int kStreamThreads = 32 * (kStreamWarps * kStreamSets + 1);
constexpr int kStreamMaxStages = 8;
constexpr int kStreamRingBytes = 216 * 1024;  // ring + table, below the 227 KB per CTA

__device__ __forceinline__ void stream_bars_init(uint64_t* full, uint64_t* empty, int stages, int* abort_flag) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kStreamWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
}

// bf16(1 + scale) of the first mod_rows modulation rows into `table` (nv vectors a row).
__device__ __forceinline__ void ln_modulate_table(uint4* table, const uint16_t* __restrict__ mod, int64_t mod_stride,
                                                  int64_t scale_off, int mod_rows, int nv) {
  for (int e = threadIdx.x; e < mod_rows * nv; e += blockDim.x) {
    const int r = e / nv, c = e - r * nv;
    const uint4 m = ldg16(mod + r * mod_stride + scale_off + c * 8);
    const uint32_t w[4] = {m.x, m.y, m.z, m.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = f2_to_bf2(fadd2(bf2_to_f2(w[k]), f2_pack(1.0f, 1.0f)));
    table[e] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// LayerNorm + modulation of one row held in shared memory, by one warp, in two steps:
// ln_row_stats gives (-mean, -mean) and (rstd, rstd) as fp32 pairs (fp32 mean and
// centred variance), ln_row_out computes y = bf16((x - mean) * rstd) and out =
// bf16(y * bf16(1 + scale)) -- one packed bf16 multiply, the product of two bf16 values
// being exact in fp32 -- and hands emit(idx, o) the 8 outputs of vector idx as four
// bf16x2 words.
__device__ __forceinline__ void ln_row_stats(const uint4* xr, int nv, int D, float eps, int lane, uint64_t& nm2,
                                             uint64_t& r2) {
  uint64_t acc = 0ull;  // (0.f, 0.f)
  for (int idx = lane; idx < nv; idx += 32) {
    const uint4 v = xr[idx];
    acc = fadd2(fadd2(acc, bf2_to_f2(v.x)), bf2_to_f2(v.y));
    acc = fadd2(fadd2(acc, bf2_to_f2(v.z)), bf2_to_f2(v.w));
  }
  const float mean = warp_sum(f2_sum(acc)) / static_cast<float>(D);
  nm2 = f2_pack(-mean, -mean);
  acc = 0ull;
  for (int idx = lane; idx < nv; idx += 32) {
    const uint4 v = xr[idx];
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint64_t d = fadd2(bf2_to_f2(u[k]), nm2);
      acc = ffma2(d, d, acc);
    }
  }
  const float var = warp_sum(f2_sum(acc)) / static_cast<float>(D);
  r2 = f2_pack(rsqrtf(var + eps), rsqrtf(var + eps));
}

template <typename Emit>
__device__ __forceinline__ void ln_row_out(const uint4* xr, const uint4* tr, int nv, uint64_t nm2, uint64_t r2,
                                           int lane, Emit emit) {
#pragma unroll 2
  for (int idx = lane; idx < nv; idx += 32) {
    const uint4 v = xr[idx], sv = tr[idx];
    const uint32_t u[4] = {v.x, v.y, v.z, v.w}, m[4] = {sv.x, sv.y, sv.z, sv.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = mul_bf16x2(f2_to_bf2(fmul2(fadd2(bf2_to_f2(u[k]), nm2), r2)), m[k]);
    emit(idx, o);
  }
}

__global__ void __launch_bounds__(kStreamThreads, 1)
    ln_modulate_stream_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ mod, int64_t mod_stride,
                              int64_t scale_off, const uint8_t* __restrict__ tmask, uint16_t* __restrict__ out,
                              int64_t B, int64_t S, int D, float eps, uint32_t* __restrict__ amax_out, int stages,
                              int mod_rows) {
  // [stages][kStreamWarps rows][nv] ring, then bf16(1 + scale) for each used modulation row
  extern __shared__ __align__(128) uint4 ring[];
  __shared__ __align__(8) uint64_t full[kStreamMaxStages], empty[kStreamMaxStages];
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = D >> 3;  // 16-byte vectors per row; a stage holds kStreamWarps rows = 8 nv vectors
  uint4* table = ring + static_cast<int64_t>(stages) * kStreamWarps * nv;
  ln_modulate_table(table, mod, mod_stride, scale_off, mod_rows, nv);
  stream_bars_init(full, empty, stages, &abort_flag);  // (its barrier also publishes the table)
  const int64_t nrows = B * S;
  const int64_t ngroups = (nrows + kStreamWarps - 1) / kStreamWarps;
  uint32_t am2 = 0;
  if (warp == 0) {
    if (lane == 0) {
      int i = 0;
      for (int64_t g = blockIdx.x; g < ngroups; g += gridDim.x, ++i) {
        const int st = i % stages;
        if (!mbar_wait(&empty[st], ((i / stages) & 1) ^ 1u, &abort_flag, nullptr)) break;
        const int64_t r0 = g * kStreamWarps;
        const int64_t rows = min(static_cast<int64_t>(kStreamWarps), nrows - r0);
        const uint32_t bytes = static_cast<uint32_t>(rows * D * 2);
        mbar_arrive_expect_tx(&full[st], bytes);
        bulk_load(ring + static_cast<int64_t>(st) * kStreamWarps * nv, x + r0 * D, bytes, &full[st]);
      }
    }
  } else {
    const int set = (warp - 1) / kStreamWarps, cw = (warp - 1) % kStreamWarps;
    int i = set;
    for (int64_t g = blockIdx.x + static_cast<int64_t>(set) * gridDim.x; g < ngroups;
         g += static_cast<int64_t>(kStreamSets) * gridDim.x, i += kStreamSets) {
      const int st = i % stages;
      if (!__all_sync(0xffffffffu, mbar_wait(&full[st], (i / stages) & 1, &abort_flag, nullptr))) break;
      const int64_t row = g * kStreamWarps + cw;
      if (row < nrows) {
        const int64_t b = row / S, s = row % S;
        // target positions use their own sample's row b, the others row B + b
        const int64_t mrow = (tmask == nullptr || tmask[s] != 0) ? b : B + b;
        uint16_t* orow = out + row * D;
        const uint4* xr = ring + (static_cast<int64_t>(st) * kStreamWarps + cw) * nv;
        uint64_t nm2, r2;
        ln_row_stats(xr, nv, D, eps, lane, nm2, r2);
        ln_row_out(xr, table + mrow * nv, nv, nm2, r2, lane, [&](int idx, const uint32_t(&o)[4]) {
          am2 = absmax_bf16x2(absmax_bf16x2(am2, o[0]), o[1]);
          am2 = absmax_bf16x2(absmax_bf16x2(am2, o[2]), o[3]);
          *reinterpret_cast<uint4*>(orow + idx * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        });
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  }
  if (amax_out) block_atomic_max(max(am2 & 0xFFFFu, am2 >> 16) << 16, amax_out);
}

// LayerNorm + modulation emitting e4m3 codes with the output's own dynamic per-tensor
// scale (fused_layer_norm_modulate followed by quantize_tensorwise, without the bf16
// output ever reaching memory).  The scale needs max|out| over the whole tensor before
// the first code, so the kernel makes two passes over the same rows, launched
// cooperatively (one CTA per SM, every CTA resident): pass 0 streams the CTA's row
// groups through the ring (L2 evict-last), reduces max|out| and keeps each row's mean
// and rstd in shared memory; a grid-wide exchange (grid_max_publish_wait) gives every
// CTA the global amax; pass 1 streams the same groups again (evict-first, from L2 while
// they are there), recomputes the identical outputs from the kept statistics and
// stores fl32(out) * (1/s) as e4m3.  The producer runs straight on into
// pass 1 while the consumers wait at the exchange.  HBM traffic: x once (2 B per
// element while x fits in L2) and the codes (1 B).  On a failed wait every CTA skips
// its stores (still draining the ring), CTA 0 writes a NaN scale and `status` records
// the timeout; the workspace must then be zeroed again before reuse.
constexpr int kStreamConsumerThreads = 32 * kStreamWarps * kStreamSets;

__global__ void __launch_bounds__(kStreamThreads, 1)
    ln_modulate_e4m3_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ mod, int64_t mod_stride,
                            int64_t scale_off, const uint8_t* __restrict__ tmask, uint8_t* __restrict__ q,
                            float* __restrict__ scale_out, int64_t B, int64_t S, int D, float eps, int stages,
                            int mod_rows, QuantWs* __restrict__ ws, int* __restrict__ status) {
  extern __shared__ __align__(128) uint4 ring[];
  __shared__ __align__(8) uint64_t full[kStreamMaxStages], empty[kStreamMaxStages];
  __shared__ int abort_flag;
  __shared__ uint32_t warp_max[kStreamWarps * kStreamSets];
  __shared__ uint32_t amax_all;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = D >> 3;
  // [stages][8 rows][nv] ring, the modulation table, then (-mean, rstd) of each row of
  // this CTA (pass 0 computes them, pass 1 reuses them)
  uint4* table = ring + static_cast<int64_t>(stages) * kStreamWarps * nv;
  uint4* stats = table + static_cast<int64_t>(mod_rows) * nv;
  ln_modulate_table(table, mod, mod_stride, scale_off, mod_rows, nv);
  stream_bars_init(full, empty, stages, &abort_flag);
  const int64_t nrows = B * S;
  const int64_t ngroups = (nrows + kStreamWarps - 1) / kStreamWarps;
  // this CTA's groups: blockIdx.x + k * gridDim.x, k < mine; item j of the ring is
  // group j % mine of pass j / mine
  const int64_t mine = ngroups > blockIdx.x ? (ngroups - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_keep = l2_evict_last_policy(), pol_once = l2_evict_first_policy();
      for (int64_t j = 0; j < 2 * mine; ++j) {
        const int st = static_cast<int>(j % stages);
        if (!mbar_wait(&empty[st], static_cast<uint32_t>((j / stages) & 1) ^ 1u, &abort_flag, status)) break;
        const int64_t r0 = (blockIdx.x + (j % mine) * gridDim.x) * kStreamWarps;
        const int64_t rows = min(static_cast<int64_t>(kStreamWarps), nrows - r0);
        const uint32_t bytes = static_cast<uint32_t>(rows * D * 2);
        mbar_arrive_expect_tx(&full[st], bytes);
        bulk_load_hint(ring + static_cast<int64_t>(st) * kStreamWarps * nv, x + r0 * D, bytes, &full[st],
                       j < mine ? pol_keep : pol_once);
      }
    }
    return;
  }
  const int cwarp = warp - 1;
  const int set = cwarp / kStreamWarps, cw = cwarp % kStreamWarps;
  uint32_t am2 = 0;
  float inv = 0.0f;
  bool skip = false;  // pass 1 without stores: some CTA gave up
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      // grid-wide max|out|: warp maxima -> CTA max -> every CTA's slot
      const uint32_t m = __reduce_max_sync(0xffffffffu, max(am2 & 0xFFFFu, am2 >> 16) << 16);
      if (lane == 0) warp_max[cwarp] = m;
      named_bar_sync(1, kStreamConsumerThreads);
      if (cwarp == 0) {
        uint32_t c = lane < kStreamWarps * kStreamSets ? warp_max[lane] : 0u;
        c = __reduce_max_sync(0xffffffffu, c);
        bool ok = true;
        if (lane == 0) {
          ok = grid_max_publish_wait(ws, abort_flag ? kQuantAbortMark : c);
          if (!ok && status) atomicExch(status, QIK_DEV_TIMEOUT);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        __syncwarp();  // lane 0's acquire of the barrier before every lane's slot reads
        const uint32_t g = grid_max_collect(ws);
        if (lane == 0) amax_all = ok ? g : kQuantAbortMark;
      }
      named_bar_sync(1, kStreamConsumerThreads);
      skip = amax_all == kQuantAbortMark;
      const float s = skip ? __int_as_float(0x7fc00000) : scale_from_amax_bits(amax_all);
      inv = act_inverse(s);
      if (blockIdx.x == 0 && cwarp == 0 && lane == 0) scale_out[0] = s;
    }
    for (int64_t j = pass * mine + set; j < (pass + 1) * mine; j += kStreamSets) {
      const int st = static_cast<int>(j % stages);
      if (!__all_sync(0xffffffffu, mbar_wait(&full[st], static_cast<uint32_t>((j / stages) & 1), &abort_flag, status)))
        break;
      const int64_t row = (blockIdx.x + (j % mine) * gridDim.x) * kStreamWarps + cw;
      if (row < nrows) {
        const int64_t b = row / S, s = row % S;
        const int64_t mrow = (tmask == nullptr || tmask[s] != 0) ? b : B + b;
        const uint4* xr = ring + (static_cast<int64_t>(st) * kStreamWarps + cw) * nv;
        uint4* rs = stats + (j % mine) * kStreamWarps + cw;  // the row's (-mean, rstd) pairs
        if (pass == 0) {
          uint64_t nm2, r2;
          ln_row_stats(xr, nv, D, eps, lane, nm2, r2);
          if (lane == 0) *rs = make_uint4(static_cast<uint32_t>(nm2), static_cast<uint32_t>(nm2 >> 32),
                                          static_cast<uint32_t>(r2), static_cast<uint32_t>(r2 >> 32));
          ln_row_out(xr, table + mrow * nv, nv, nm2, r2, lane, [&](int, const uint32_t(&o)[4]) {
            am2 = absmax_bf16x2(absmax_bf16x2(am2, o[0]), o[1]);
            am2 = absmax_bf16x2(absmax_bf16x2(am2, o[2]), o[3]);
          });
        } else if (!skip) {
          const uint4 sv = *rs;  // written by this warp's lane 0 in pass 0
          const uint64_t nm2 = (static_cast<uint64_t>(sv.y) << 32) | sv.x;
          const uint64_t r2 = (static_cast<uint64_t>(sv.w) << 32) | sv.z;
          uint2* qrow = reinterpret_cast<uint2*>(q + row * D);
          ln_row_out(xr, table + mrow * nv, nv, nm2, r2, lane, [&](int idx, const uint32_t(&o)[4]) {
            uint32_t hi;
            const uint32_t lo = pack8_e4m3(make_uint4(o[0], o[1], o[2], o[3]), inv, hi);
            qrow[idx] = make_uint2(lo, hi);
          });
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  }
}

// RMSNorm + RoPE over tokens whose heads are contiguous (x_sh == D, as in the strided
// q / k views of the fused QKV output): a stage holds 8 tokens' H x D elements (one
// bulk copy per token), a consumer warp walks its token's heads 32 / G at a time with
// the token's cos / sin rows loaded once.
template <int G>
__global__ void __launch_bounds__(kStreamThreads, 1)
    rms_rope_stream_kernel(const uint16_t* __restrict__ x, int64_t x_sb, int64_t x_ss, uint16_t* __restrict__ out,
                           int64_t o_sb, int64_t o_ss, int64_t o_sh, const float* __restrict__ w,
                           const float* __restrict__ cs, const float* __restrict__ sn, int64_t B, int64_t S, int H,
                           float eps, int stages) {
  constexpr int D = 8 * G, HALF = D / 2, RPW = 32 / G;
  extern __shared__ __align__(128) uint4 ring[];
  __shared__ __align__(8) uint64_t full[kStreamMaxStages], empty[kStreamMaxStages];
  __shared__ int abort_flag;
  stream_bars_init(full, empty, stages, &abort_flag);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok_vecs = H * G;  // 16-byte vectors per token
  const int64_t ntok = B * S;
  const int64_t ngroups = (ntok + kStreamWarps - 1) / kStreamWarps;
  if (warp == 0) {
    if (lane == 0) {
      int i = 0;
      for (int64_t g = blockIdx.x; g < ngroups; g += gridDim.x, ++i) {
        const int st = i % stages;
        if (!mbar_wait(&empty[st], ((i / stages) & 1) ^ 1u, &abort_flag, nullptr)) break;
        const int64_t t0 = g * kStreamWarps;
        const int toks = static_cast<int>(min(static_cast<int64_t>(kStreamWarps), ntok - t0));
        const uint32_t bytes = static_cast<uint32_t>(tok_vecs) * 16u;
        mbar_arrive_expect_tx(&full[st], bytes * static_cast<uint32_t>(toks));
        for (int k = 0; k < toks; ++k) {
          const int64_t t = t0 + k, b = t / S, s = t - b * S;
          bulk_load(ring + (static_cast<int64_t>(st) * kStreamWarps + k) * tok_vecs, x + b * x_sb + s * x_ss, bytes,
                    &full[st]);
        }
      }
    }
    return;
  }
  const int set = (warp - 1) / kStreamWarps, cw = (warp - 1) % kStreamWarps;
  const int sub = lane / G, gl = lane % G;
  const float4 w0 = ldg16f(w + gl * 8), w1 = ldg16f(w + gl * 8 + 4);
  const uint64_t w2[4] = {f2_pack(w0.x, w0.y), f2_pack(w0.z, w0.w), f2_pack(w1.x, w1.y), f2_pack(w1.z, w1.w)};
  int i = set;
  for (int64_t g = blockIdx.x + static_cast<int64_t>(set) * gridDim.x; g < ngroups;
       g += static_cast<int64_t>(kStreamSets) * gridDim.x, i += kStreamSets) {
    const int st = i % stages;
    if (!__all_sync(0xffffffffu, mbar_wait(&full[st], (i / stages) & 1, &abort_flag, nullptr))) break;
    const int64_t t = g * kStreamWarps + cw;
    if (t < ntok) {
      const int64_t b = t / S, s = t - b * S;
      const float4 c4 = ldg16f(cs + s * HALF + gl * 4), s4 = ldg16f(sn + s * HALF + gl * 4);
      // (e + i o)(c + i s): the pair (e c - o s, e s + o c) = e (c, s) + o (-s, c)
      const uint64_t cs2[4] = {f2_pack(c4.x, s4.x), f2_pack(c4.y, s4.y), f2_pack(c4.z, s4.z), f2_pack(c4.w, s4.w)};
      const uint64_t sc2[4] = {f2_pack(-s4.x, c4.x), f2_pack(-s4.y, c4.y), f2_pack(-s4.z, c4.z),
                               f2_pack(-s4.w, c4.w)};
      const uint4* xt = ring + (static_cast<int64_t>(st) * kStreamWarps + cw) * tok_vecs;
      uint16_t* ot = out + b * o_sb + s * o_ss;
#pragma unroll 2
      for (int h0 = 0; h0 < H; h0 += RPW) {
        const int h = h0 + sub;
        const bool live = h < H;
        const uint4 v = live ? xt[h * G + gl] : make_uint4(0u, 0u, 0u, 0u);
        float ss = rms_ss8(v.x, v.y, v.z, v.w);
#pragma unroll
        for (int o = G / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rrms = rms_rstd(ss, D, eps);
        const uint64_t rr2 = f2_pack(rrms, rrms);
        // fp32 norm and weight, one rounding to bf16, the rotation in fp32
        const uint32_t o4[4] = {rms_rope_pair(v.x, rr2, w2[0], cs2[0], sc2[0]),
                                rms_rope_pair(v.y, rr2, w2[1], cs2[1], sc2[1]),
                                rms_rope_pair(v.z, rr2, w2[2], cs2[2], sc2[2]),
                                rms_rope_pair(v.w, rr2, w2[3], cs2[3], sc2[3])};
        if (live) *reinterpret_cast<uint4*>(ot + h * o_sh + gl * 8) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
}

// Shared memory ring of a streaming kernel: stages of `stage_bytes`, at least 2 and at
// most kStreamMaxStages within kStreamRingBytes less `reserved` bytes; 0 when a stage
// does not fit twice.  The count is even: the two consumer sets take alternate ring
// items, so a stage's previous item then belongs to the same set, which has consumed
// it before it waits on the stage's next phase (with an odd count the other set's
// previous item could still be in flight, and a parity wait would see a stale phase).
int stream_stages(int64_t stage_bytes, int64_t reserved = 0) {
  int64_t n = (kStreamRingBytes - reserved) / stage_bytes;
  n = n < kStreamMaxStages ? n : kStreamMaxStages;
  return n < 2 ? 0 : static_cast<int>(n & ~int64_t{1});
}

template <typename Kernel>
int stream_smem_attr(Kernel kernel, std::once_flag* once, const char* what, int bytes = kStreamRingBytes) {
  int dev = 0;
  QIK_TRY_CUDA(cudaGetDevice(&dev));
  QIK_REQUIRE(dev >= 0 && dev < 64, "%s: device ordinal %d out of range", what, dev);
  cudaError_t rc = cudaSuccess;
  std::call_once(once[dev], [&] {
    rc = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  });
  return cuda_status(rc, what);
}
// Dynamic shared memory of ln_modulate_e4m3_kernel: the ring and table as the other
// streaming kernels, plus 16 bytes of row statistics for each row of its CTA.
constexpr int kLnE4m3SmemBytes = 224 * 1024;

// ---------------------------------------------------------------- gate + residual
// Thread = one 8-column vector of the width, walking kGateRows consecutive rows
// (4 at a time, loads first).  bf16(tanh(gate)) depends only on the modulation row
// (b for target positions, B + b otherwise), so each thread computes it once per
// distinct row it meets and keeps the two rows of the current sample in registers.
constexpr int kGateRows = 32;
constexpr int kGateThreads = 128;

struct GateCache {
  int64_t row;
  float t[8];
};

__device__ __forceinline__ void gate_fill(GateCache& c, int64_t mrow, const uint16_t* __restrict__ mod,
                                          int64_t mod_stride, int64_t col) {
  const uint4 g4 = ldg16(mod + mrow * mod_stride + col);
  const uint32_t gu[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    c.t[2 * j] = round_bf16(tanhf(bf_lo(gu[j])));
    c.t[2 * j + 1] = round_bf16(tanhf(bf_hi(gu[j])));
  }
  c.row = mrow;
}

__global__ void __launch_bounds__(kGateThreads, 7) gate_residual_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ f, const uint16_t* __restrict__ mod,
    int64_t mod_stride, int64_t gate_off, const uint8_t* __restrict__ tmask, uint16_t* __restrict__ out, int64_t B,
    int64_t S, int64_t D) {
  const int64_t nvr = D >> 3;
  const int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (v >= nvr) return;
  const int64_t rows = B * S;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kGateRows;
  const int64_t r1 = min(rows, r0 + kGateRows);
  const int64_t col = gate_off + v * 8;
  GateCache ct, cz;  // row b (target positions) and row B + b (t = 0 positions)
  ct.row = cz.row = -1;
  for (int64_t rb = r0; rb < r1; rb += 4) {
    uint4 x4[4], f4[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t r = rb + k;
      x4[k] = r < r1 ? ldg16(x + r * D + v * 8) : make_uint4(0u, 0u, 0u, 0u);
      f4[k] = r < r1 ? ldg16(f + r * D + v * 8) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t r = rb + k;
      if (r >= r1) break;
      const int64_t b = static_cast<uint32_t>(r) / static_cast<uint32_t>(S);  // rows < 2^31 (host check)
      const int64_t s = r - b * S;
      const uint32_t xu[4] = {x4[k].x, x4[k].y, x4[k].z, x4[k].w}, fu[4] = {f4[k].x, f4[k].y, f4[k].z, f4[k].w};
      uint32_t o[4];
      auto apply = [&](const GateCache& c) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float t0 = round_bf16(c.t[2 * j] * bf_lo(fu[j]));
          const float t1 = round_bf16(c.t[2 * j + 1] * bf_hi(fu[j]));
          o[j] = pack_bf16x2(bf_lo(xu[j]) + t0, bf_hi(xu[j]) + t1);
        }
      };
      if (tmask == nullptr || tmask[s] != 0) {
        if (ct.row != b) gate_fill(ct, b, mod, mod_stride, col);
        apply(ct);
      } else {
        if (cz.row != B + b) gate_fill(cz, B + b, mod, mod_stride, col);
        apply(cz);
      }
      *reinterpret_cast<uint4*>(out + r * D + v * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// ---------------------------------------------------------------- SwiGLU
// silu_bf16 (qik_device.cuh): bf16(g / (1 + e^-g)), shared with the GEMM's SwiGLU epilogue.

__global__ void __launch_bounds__(kThreads) swiglu_kernel(const uint16_t* __restrict__ g, int64_t ld_g,
                                                          const uint16_t* __restrict__ p, int64_t ld_p,
                                                          uint16_t* __restrict__ out, int64_t ld_o, int64_t M,
                                                          int64_t N, uint32_t* __restrict__ amax_out) {
  const int64_t nvr = N >> 3;
  const int64_t total = M * nvr;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  uint32_t am2 = 0;
  // two vectors per iteration, both loads issued first
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += 2 * nthreads) {
    uint4 g4[2], p4[2];
    int64_t off[2][3];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int64_t e = i + k * nthreads;
      // total < 2^31 (host check): 32-bit division
      const int64_t m = e < total ? static_cast<uint32_t>(e) / static_cast<uint32_t>(nvr) : 0;
      const int64_t c = e < total ? (e - m * nvr) * 8 : 0;
      off[k][0] = m * ld_g + c;
      off[k][1] = m * ld_p + c;
      off[k][2] = m * ld_o + c;
      g4[k] = e < total ? ldg16(g + off[k][0]) : make_uint4(0u, 0u, 0u, 0u);
      p4[k] = e < total ? ldg16(p + off[k][1]) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (i + k * nthreads >= total) break;
      const uint32_t gu[4] = {g4[k].x, g4[k].y, g4[k].z, g4[k].w}, pu[4] = {p4[k].x, p4[k].y, p4[k].z, p4[k].w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[j] = pack_bf16x2(silu_bf16(bf_lo(gu[j])) * bf_lo(pu[j]), silu_bf16(bf_hi(gu[j])) * bf_hi(pu[j]));
        am2 = absmax_bf16x2(am2, o[j]);
      }
      *reinterpret_cast<uint4*>(out + off[k][2]) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  if (amax_out) block_atomic_max(max(am2 & 0xFFFFu, am2 >> 16) << 16, amax_out);
}

int grid_cap(int64_t want, int per_sm) {
  const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
  const int64_t g = want < cap ? want : cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

bool aligned_elems(int64_t v) { return (v & 7) == 0; }  // multiple of 8 bf16 = 16 bytes

}  // namespace
}  // namespace qik

using namespace qik;

extern "C" {

int qik_rms_norm_rope(const void* x, int64_t B, int64_t S, int64_t H, int64_t D, int64_t x_sb, int64_t x_ss,
                      int64_t x_sh, const float* weight, const float* cos_tab, const float* sin_tab, float eps,
                      void* out, int64_t o_sb, int64_t o_ss, int64_t o_sh, void* stream) {
  QIK_REQUIRE(B >= 0 && S >= 0 && H >= 0, "qik_rms_norm_rope: negative size");
  const int64_t nrows = B * S * H;
  if (nrows == 0) return QIK_OK;
  QIK_REQUIRE(x && out && weight && cos_tab && sin_tab, "qik_rms_norm_rope: NULL pointer");
  if (D != 64 && D != 128 && D != 256)
    return set_error(QIK_ERR_UNSUPPORTED, "qik_rms_norm_rope: head dim %lld (64, 128 or 256 supported)",
                     static_cast<long long>(D));
  QIK_REQUIRE(aligned16(x) && aligned16(out) && aligned16(weight) && aligned16(cos_tab) && aligned16(sin_tab),
              "qik_rms_norm_rope: pointers must be 16-byte aligned");
  QIK_REQUIRE(nrows < (int64_t{1} << 31), "qik_rms_norm_rope: more than 2^31 rows");
  QIK_REQUIRE(aligned_elems(x_sb) && aligned_elems(x_ss) && aligned_elems(x_sh) && aligned_elems(o_sb) &&
                  aligned_elems(o_ss) && aligned_elems(o_sh),
              "qik_rms_norm_rope: strides must be multiples of 8 elements");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t ntok = B * S;
  const int stages = x_sh == D ? stream_stages(static_cast<int64_t>(kStreamWarps) * H * D * 2) : 0;
  if (stages > 0 && H <= 65535) {
    // heads of a token contiguous: stream 8-token groups through shared memory
    static std::once_flag once8[64], once16[64], once32[64];
    const int grid = grid_cap((ntok + kStreamWarps - 1) / kStreamWarps, 1);
    const size_t smem = static_cast<size_t>(stages) * kStreamWarps * H * D * 2;
    const uint16_t* xs = static_cast<const uint16_t*>(x);
    uint16_t* os = static_cast<uint16_t*>(out);
    int rc;
    if (D == 64) {
      if ((rc = stream_smem_attr(rms_rope_stream_kernel<8>, once8, "rms_rope_stream_kernel"))) return rc;
      rms_rope_stream_kernel<8><<<grid, kStreamThreads, smem, st>>>(xs, x_sb, x_ss, os, o_sb, o_ss, o_sh, weight,
                                                                    cos_tab, sin_tab, B, S, static_cast<int>(H), eps,
                                                                    stages);
    } else if (D == 128) {
      if ((rc = stream_smem_attr(rms_rope_stream_kernel<16>, once16, "rms_rope_stream_kernel"))) return rc;
      rms_rope_stream_kernel<16><<<grid, kStreamThreads, smem, st>>>(xs, x_sb, x_ss, os, o_sb, o_ss, o_sh, weight,
                                                                     cos_tab, sin_tab, B, S, static_cast<int>(H), eps,
                                                                     stages);
    } else {
      if ((rc = stream_smem_attr(rms_rope_stream_kernel<32>, once32, "rms_rope_stream_kernel"))) return rc;
      rms_rope_stream_kernel<32><<<grid, kStreamThreads, smem, st>>>(xs, x_sb, x_ss, os, o_sb, o_ss, o_sh, weight,
                                                                     cos_tab, sin_tab, B, S, static_cast<int>(H), eps,
                                                                     stages);
    }
    return check_launch("rms_rope_stream_kernel");
  }
  const int rows_per_cta = (kThreads / 32) * (32 / static_cast<int>(D / 8)) * kRopeUnroll;
  const int grid = grid_cap((nrows + rows_per_cta - 1) / rows_per_cta, 8);
  const uint16_t* xs = static_cast<const uint16_t*>(x);
  uint16_t* os = static_cast<uint16_t*>(out);
  if (D == 64)
    rms_rope_kernel<8><<<grid, kThreads, 0, st>>>(xs, x_sb, x_ss, x_sh, os, o_sb, o_ss, o_sh, weight, cos_tab,
                                                  sin_tab, S, H, nrows, eps);
  else if (D == 128)
    rms_rope_kernel<16><<<grid, kThreads, 0, st>>>(xs, x_sb, x_ss, x_sh, os, o_sb, o_ss, o_sh, weight, cos_tab,
                                                   sin_tab, S, H, nrows, eps);
  else
    rms_rope_kernel<32><<<grid, kThreads, 0, st>>>(xs, x_sb, x_ss, x_sh, os, o_sb, o_ss, o_sh, weight, cos_tab,
                                                   sin_tab, S, H, nrows, eps);
  return check_launch("rms_rope_kernel");
}

static int check_ln_args(const char* what, const void* x, int64_t B, int64_t S, int64_t D, const void* modulation,
                         int64_t mod_rows, int64_t mod_stride, int64_t scale_off, const uint8_t* target_mask,
                         const void* out) {
  QIK_REQUIRE(x && modulation && out, "%s: NULL pointer", what);
  QIK_REQUIRE(D % 8 == 0 && D <= 4096, "%s: D must be a multiple of 8 and at most 4096", what);
  QIK_REQUIRE(B * S < (int64_t{1} << 31), "%s: more than 2^31 rows", what);
  QIK_REQUIRE(aligned16(x) && aligned16(out) && aligned16(modulation), "%s: pointers must be 16-byte aligned", what);
  QIK_REQUIRE(aligned_elems(mod_stride) && aligned_elems(scale_off) && scale_off >= 0 && scale_off + D <= mod_stride,
              "%s: modulation stride/offset must be multiples of 8 with offset + D <= stride", what);
  QIK_REQUIRE(mod_rows >= (target_mask ? 2 * B : B), "%s: %lld modulation rows; B = %lld needs %s", what,
              static_cast<long long>(mod_rows), static_cast<long long>(B),
              target_mask ? "2B (rows B..2B-1 are the t = 0 rows)" : "B");
  return QIK_OK;
}

// Ring geometry of the layer-norm kernels: 8-row stages beside the table of bf16(1 +
// scale) for every modulation row in use.  Returns the stage count (0: does not fit).
static int ln_ring(int64_t B, int64_t D, const uint8_t* target_mask, int* mod_used, size_t* smem) {
  *mod_used = static_cast<int>(target_mask ? 2 * B : B);
  const int64_t table_bytes = static_cast<int64_t>(*mod_used) * D * 2;
  const int64_t stage_bytes = static_cast<int64_t>(kStreamWarps) * D * 2;
  const int stages = table_bytes < kStreamRingBytes ? stream_stages(stage_bytes, table_bytes) : 0;
  *smem = static_cast<size_t>(stages) * stage_bytes + static_cast<size_t>(table_bytes);
  return stages;
}

int qik_layer_norm_modulate(const void* x, int64_t B, int64_t S, int64_t D, const void* modulation,
                            int64_t mod_rows, int64_t mod_stride, int64_t scale_off, const uint8_t* target_mask,
                            float eps, void* out, uint32_t* amax_out, void* stream) {
  QIK_REQUIRE(B >= 0 && S >= 0 && D > 0, "qik_layer_norm_modulate: bad sizes");
  if (B * S == 0) return QIK_OK;
  int rc = check_ln_args("qik_layer_norm_modulate", x, B, S, D, modulation, mod_rows, mod_stride, scale_off,
                         target_mask, out);
  if (rc) return rc;
  int mod_used = 0;
  size_t smem = 0;
  const int stages = ln_ring(B, D, target_mask, &mod_used, &smem);
  if (stages == 0)
    return set_error(QIK_ERR_UNSUPPORTED,
                     "qik_layer_norm_modulate: width %lld with %d modulation rows does not fit the row ring",
                     static_cast<long long>(D), mod_used);
  // rows streamed through shared memory, 8 per stage
  static std::once_flag once[64];
  if ((rc = stream_smem_attr(ln_modulate_stream_kernel, once, "ln_modulate_stream_kernel"))) return rc;
  const int grid = grid_cap((B * S + kStreamWarps - 1) / kStreamWarps, 1);
  ln_modulate_stream_kernel<<<grid, kStreamThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(modulation), mod_stride, scale_off, target_mask,
      static_cast<uint16_t*>(out), B, S, static_cast<int>(D), eps, amax_out, stages, mod_used);
  return check_launch("ln_modulate_stream_kernel");
}

int qik_layer_norm_modulate_e4m3(const void* x, int64_t B, int64_t S, int64_t D, const void* modulation,
                                 int64_t mod_rows, int64_t mod_stride, int64_t scale_off, const uint8_t* target_mask,
                                 float eps, uint8_t* q, float* scale_out, void* ws, int* status, void* stream) {
  QIK_REQUIRE(B >= 0 && S >= 0 && D > 0, "qik_layer_norm_modulate_e4m3: bad sizes");
  QIK_REQUIRE(scale_out && ws, "qik_layer_norm_modulate_e4m3: scale_out/ws is NULL");
  QIK_REQUIRE(aligned16(ws), "qik_layer_norm_modulate_e4m3: ws must be 16-byte aligned");
  if (B * S == 0) return QIK_OK;
  int rc = check_ln_args("qik_layer_norm_modulate_e4m3", x, B, S, D, modulation, mod_rows, mod_stride, scale_off,
                         target_mask, q);
  if (rc) return rc;
  int mod_used = 0;
  size_t smem = 0;
  int stages = ln_ring(B, D, target_mask, &mod_used, &smem);
  // cooperative: every CTA resident (one per SM) for the grid-wide amax exchange
  const int64_t ngroups = (B * S + kStreamWarps - 1) / kStreamWarps;
  const int64_t cap = sm_count() < kQuantMaxCtas ? sm_count() : kQuantMaxCtas;
  const int64_t grid = ngroups < cap ? ngroups : cap;
  const size_t stats_bytes = static_cast<size_t>((ngroups + grid - 1) / grid) * kStreamWarps * 16;
  const size_t stage_bytes = static_cast<size_t>(kStreamWarps) * D * 2;
  while (stages > 2 && smem + stats_bytes > static_cast<size_t>(kLnE4m3SmemBytes)) {
    stages -= 2;  // even, as stream_stages keeps it
    smem -= 2 * stage_bytes;
  }
  if (stages == 0 || smem + stats_bytes > static_cast<size_t>(kLnE4m3SmemBytes))
    return set_error(QIK_ERR_UNSUPPORTED,
                     "qik_layer_norm_modulate_e4m3: width %lld with %d modulation rows and %lld rows does not fit "
                     "shared memory",
                     static_cast<long long>(D), mod_used, static_cast<long long>(B * S));
  smem += stats_bytes;
  static std::once_flag once[64];
  if ((rc = stream_smem_attr(ln_modulate_e4m3_kernel, once, "ln_modulate_e4m3_kernel", kLnE4m3SmemBytes))) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kStreamThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QIK_TRY_CUDA(cudaLaunchKernelEx(&cfg, ln_modulate_e4m3_kernel, static_cast<const uint16_t*>(x),
                                  static_cast<const uint16_t*>(modulation), mod_stride, scale_off, target_mask, q,
                                  scale_out, B, S, static_cast<int>(D), eps, stages, mod_used,
                                  static_cast<QuantWs*>(ws), status));
  return check_launch("ln_modulate_e4m3_kernel");
}

// bf16(tanh(gate)) of every modulation row, as gate_fill computes it: the table the
// FP8 GEMM's gated-residual epilogue reads.
__global__ void __launch_bounds__(kThreads) gate_table_kernel(const uint16_t* __restrict__ mod, int64_t mod_stride,
                                                              int64_t gate_off, int64_t rows, int64_t D,
                                                              uint16_t* __restrict__ table) {
  pdl_wait();  // the modulation rows come from the previous kernel
  const int64_t nv = D >> 3, total = rows * nv;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nv, v = i - r * nv;
    GateCache c;
    gate_fill(c, r, mod, mod_stride, gate_off + v * 8);
    *reinterpret_cast<uint4*>(table + r * D + v * 8) =
        make_uint4(pack_bf16x2(c.t[0], c.t[1]), pack_bf16x2(c.t[2], c.t[3]), pack_bf16x2(c.t[4], c.t[5]),
                   pack_bf16x2(c.t[6], c.t[7]));
  }
}

int qik_gate_table(const void* modulation, int64_t mod_rows, int64_t mod_stride, int64_t gate_off, int64_t D,
                   void* table, void* stream) {
  QIK_REQUIRE(mod_rows >= 0 && D > 0, "qik_gate_table: bad sizes");
  if (mod_rows == 0) return QIK_OK;
  QIK_REQUIRE(modulation && table, "qik_gate_table: NULL pointer");
  QIK_REQUIRE(D % 8 == 0 && aligned16(modulation) && aligned16(table),
              "qik_gate_table: D must be a multiple of 8 and the pointers 16-byte aligned");
  QIK_REQUIRE(aligned_elems(mod_stride) && aligned_elems(gate_off) && gate_off >= 0 && gate_off + D <= mod_stride,
              "qik_gate_table: modulation stride/offset must be multiples of 8 with offset + D <= stride");
  const int grid = grid_cap((mod_rows * (D / 8) + kThreads - 1) / kThreads, 1);
  // a programmatic dependent of the previous kernel (the modulation linear)
  QIK_TRY_CUDA(launch_kernel(gate_table_kernel, dim3(grid), dim3(kThreads), 0, static_cast<cudaStream_t>(stream), true,
                             static_cast<const uint16_t*>(modulation), mod_stride, gate_off, mod_rows, D,
                             static_cast<uint16_t*>(table)));
  return check_launch("gate_table_kernel");
}

int qik_gate_residual(const void* x, const void* f, int64_t B, int64_t S, int64_t D, const void* modulation,
                      int64_t mod_rows, int64_t mod_stride, int64_t gate_off, const uint8_t* target_mask, void* out,
                      void* stream) {
  QIK_REQUIRE(B >= 0 && S >= 0 && D > 0, "qik_gate_residual: bad sizes");
  if (B * S == 0) return QIK_OK;
  QIK_REQUIRE(x && f && modulation && out, "qik_gate_residual: NULL pointer");
  QIK_REQUIRE(D % 8 == 0, "qik_gate_residual: D must be a multiple of 8");
  QIK_REQUIRE(aligned16(x) && aligned16(f) && aligned16(out) && aligned16(modulation),
              "qik_gate_residual: pointers must be 16-byte aligned");
  QIK_REQUIRE(B * S < (int64_t{1} << 31), "qik_gate_residual: more than 2^31 rows");
  QIK_REQUIRE(aligned_elems(mod_stride) && aligned_elems(gate_off) && gate_off >= 0 && gate_off + D <= mod_stride,
              "qik_gate_residual: modulation stride/offset must be multiples of 8 with offset + D <= stride");
  QIK_REQUIRE(mod_rows >= (target_mask ? 2 * B : B), "qik_gate_residual: %lld modulation rows; B = %lld needs %s",
              static_cast<long long>(mod_rows), static_cast<long long>(B),
              target_mask ? "2B (rows B..2B-1 are the t = 0 rows)" : "B");
  const dim3 grid(static_cast<unsigned>((D / 8 + kGateThreads - 1) / kGateThreads),
                  static_cast<unsigned>((B * S + kGateRows - 1) / kGateRows));
  QIK_REQUIRE((B * S + kGateRows - 1) / kGateRows < 65536, "qik_gate_residual: too many rows (%lld)",
              static_cast<long long>(B * S));
  gate_residual_kernel<<<grid, kGateThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(f), static_cast<const uint16_t*>(modulation),
      mod_stride, gate_off, target_mask, static_cast<uint16_t*>(out), B, S, D);
  return check_launch("gate_residual_kernel");
}

int qik_swiglu(const void* gate, int64_t ld_gate, const void* up, int64_t ld_up, int64_t M, int64_t N, void* out,
               int64_t ld_out, uint32_t* amax_out, void* stream) {
  QIK_REQUIRE(M >= 0 && N >= 0, "qik_swiglu: negative size");
  if (M * N == 0) return QIK_OK;
  QIK_REQUIRE(gate && up && out, "qik_swiglu: NULL pointer");
  QIK_REQUIRE(N % 8 == 0 && aligned_elems(ld_gate) && aligned_elems(ld_up) && aligned_elems(ld_out),
              "qik_swiglu: N and the row pitches must be multiples of 8 elements");
  QIK_REQUIRE(ld_gate >= N && ld_up >= N && ld_out >= N, "qik_swiglu: row pitch smaller than N");
  QIK_REQUIRE(aligned16(gate) && aligned16(up) && aligned16(out), "qik_swiglu: pointers must be 16-byte aligned");
  const int64_t total = M * (N / 8);
  QIK_REQUIRE(total < (int64_t{1} << 31), "qik_swiglu: more than 2^34 elements");
  const int grid = grid_cap((total + 2 * kThreads - 1) / (2 * kThreads), 8);
  swiglu_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(gate), ld_gate, static_cast<const uint16_t*>(up), ld_up,
      static_cast<uint16_t*>(out), ld_out, M, N, amax_out);
  return check_launch("swiglu_kernel");
}

}  // extern "C"
