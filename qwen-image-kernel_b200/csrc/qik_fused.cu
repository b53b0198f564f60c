// qik_fused.cu -- the elementwise / normalization kernels of the DiT block.
//
// Restatements of the reference's fused Triton kernels
// (qwen_image_kernel/triton_fused.py) with the same rounding points:
//   rms_norm_rope    per-head RMSNorm (fp32 weight multiply, one bf16 rounding) +
//                    complex RoPE on (even, odd) pairs             (:27-67)
//   layer_norm_mod   LayerNorm without affine, bf16, times bf16(1 + scale) with the
//                    per-position modulation row map              (:75-108)
//   gate_residual    x + bf16(tanh(gate)) * f                      (:168-196)
//   swiglu           bf16(silu(g)) * up                            (:227-240)
// All four are HBM-bound: 16-byte vector loads and stores, grids a multiple of the
// SM count with grid-stride loops.  Layer norm and SwiGLU can also accumulate the
// amax of their bf16 output (fp32 bit patterns, atomicMax), which is the reduction
// the next FP8 linear's dynamic quantizer needs, so that linear can skip its own
// amax pass (qik_quantize_act_from_amax).
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
  __shared__ uint32_t red[kThreads / 32];
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
// lane; 32 / G rows per warp.  Sum of squares reduced over the lane group.
template <int G>
__global__ void __launch_bounds__(kThreads) rms_rope_kernel(const uint16_t* __restrict__ x, int64_t x_sb,
                                                            int64_t x_ss, int64_t x_sh, uint16_t* __restrict__ out,
                                                            int64_t o_sb, int64_t o_ss, int64_t o_sh,
                                                            const float* __restrict__ w, const float* __restrict__ cs,
                                                            const float* __restrict__ sn, int64_t S, int64_t H,
                                                            int64_t nrows, float eps) {
  constexpr int D = 8 * G, HALF = D / 2, RPW = 32 / G;
  const int lane = threadIdx.x & 31;
  const int sub = lane / G, gl = lane % G;
  // weights of this lane's 8 columns: loop invariant
  const float4 w0 = ldg16f(w + gl * 8), w1 = ldg16f(w + gl * 8 + 4);
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t groups = (nrows + RPW - 1) / RPW;
  for (int64_t wg = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); wg < groups;
       wg += warps_total) {
    const int64_t row = wg * RPW + sub;
    const bool live = row < nrows;
    const int64_t r = live ? row : 0;
    const int64_t h = r % H, bs = r / H;
    const int64_t s = bs % S, b = bs / S;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (live) v = ldg16(x + b * x_sb + s * x_ss + h * x_sh + gl * 8);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    float xe[4], xo[4];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xe[i] = bf_lo(u[i]);
      xo[i] = bf_hi(u[i]);
      ss = fmaf(xe[i], xe[i], ss);
      ss = fmaf(xo[i], xo[i], ss);
    }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rrms = rsqrtf(ss / static_cast<float>(D) + eps);
    const float4 c4 = ldg16f(cs + s * HALF + gl * 4), s4 = ldg16f(sn + s * HALF + gl * 4);
    const float cv[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
    uint32_t o4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // fp32 norm, one rounding to bf16, back to fp32 for the rotation
      const float ne = round_bf16((xe[i] * rrms) * wv[2 * i]);
      const float no = round_bf16((xo[i] * rrms) * wv[2 * i + 1]);
      // (e + i o)(c + i s) = (e c - o s) + i (e s + o c)
      o4[i] = pack_bf16x2(ne * cv[i] - no * sv[i], ne * sv[i] + no * cv[i]);
    }
    if (live)
      *reinterpret_cast<uint4*>(out + b * o_sb + s * o_ss + h * o_sh + gl * 8) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
}

// ---------------------------------------------------------------- LayerNorm + modulate
// One warp per row of D (D % 8 == 0, D <= 8 * 32 * MAXV): the row stays in
// registers between the mean, the centred variance and the output pass.
template <int MAXV>
__global__ void __launch_bounds__(kThreads) ln_modulate_kernel(const uint16_t* __restrict__ x,
                                                               const uint16_t* __restrict__ mod, int64_t mod_stride,
                                                               int64_t scale_off, const uint8_t* __restrict__ tmask,
                                                               uint16_t* __restrict__ out, int64_t B, int64_t S, int D,
                                                               float eps, uint32_t* __restrict__ amax_out) {
  const int lane = threadIdx.x & 31;
  const int nv = D >> 3;
  const int64_t nrows = B * S;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  uint32_t am2 = 0;  // two running bf16 |y| maxima
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); row < nrows;
       row += warps_total) {
    const int64_t b = row / S, s = row % S;
    const uint16_t* xr = x + row * D;
    uint4 xv[MAXV];
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int idx = lane + 32 * i;
      xv[i] = idx < nv ? ldg16(xr + idx * 8) : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t u[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) sum += bf_lo(u[j]) + bf_hi(u[j]);
    }
    sum = warp_sum(sum);
    const float mean = sum / static_cast<float>(D);
    float var = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (lane + 32 * i < nv) {
        const uint32_t u[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = bf_lo(u[j]) - mean, c = bf_hi(u[j]) - mean;
          var = fmaf(a, a, var);
          var = fmaf(c, c, var);
        }
      }
    }
    var = warp_sum(var) / static_cast<float>(D);
    const float rstd = rsqrtf(var + eps);
    // target positions use their own sample's row b, the others row B + b
    const int64_t mrow = (tmask == nullptr || tmask[s] != 0) ? b : B + b;
    const uint16_t* sc = mod + mrow * mod_stride + scale_off;
    uint16_t* orow = out + row * D;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int idx = lane + 32 * i;
      if (idx < nv) {
        const uint4 sv = ldg16(sc + idx * 8);
        const uint32_t u[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
        const uint32_t m[4] = {sv.x, sv.y, sv.z, sv.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float y0 = round_bf16((bf_lo(u[j]) - mean) * rstd), y1 = round_bf16((bf_hi(u[j]) - mean) * rstd);
          o[j] = pack_bf16x2(y0 * round_bf16(1.0f + bf_lo(m[j])), y1 * round_bf16(1.0f + bf_hi(m[j])));
          am2 = absmax_bf16x2(am2, o[j]);
        }
        *reinterpret_cast<uint4*>(orow + idx * 8) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  if (amax_out) block_atomic_max(max(am2 & 0xFFFFu, am2 >> 16) << 16, amax_out);
}

// ---------------------------------------------------------------- gate + residual
// 8 elements per thread iteration; rows of D contiguous elements.
__global__ void __launch_bounds__(kThreads) gate_residual_kernel(const uint16_t* __restrict__ x,
                                                                 const uint16_t* __restrict__ f,
                                                                 const uint16_t* __restrict__ mod, int64_t mod_stride,
                                                                 int64_t gate_off, const uint8_t* __restrict__ tmask,
                                                                 uint16_t* __restrict__ out, int64_t B, int64_t S,
                                                                 int64_t D) {
  const int64_t nvr = D >> 3;
  const int64_t total = B * S * nvr;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += nthreads) {
    const int64_t row = i / nvr, v = i - row * nvr;
    const int64_t b = row / S, s = row % S;
    const int64_t mrow = (tmask == nullptr || tmask[s] != 0) ? b : B + b;
    const uint4 g4 = ldg16(mod + mrow * mod_stride + gate_off + v * 8);
    const uint4 x4 = ldg16(x + i * 8), f4 = ldg16(f + i * 8);
    const uint32_t gu[4] = {g4.x, g4.y, g4.z, g4.w}, xu[4] = {x4.x, x4.y, x4.z, x4.w},
                   fu[4] = {f4.x, f4.y, f4.z, f4.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float t0 = round_bf16(round_bf16(tanhf(bf_lo(gu[j]))) * bf_lo(fu[j]));
      const float t1 = round_bf16(round_bf16(tanhf(bf_hi(gu[j]))) * bf_hi(fu[j]));
      o[j] = pack_bf16x2(bf_lo(xu[j]) + t0, bf_hi(xu[j]) + t1);
    }
    *reinterpret_cast<uint4*>(out + i * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------- SwiGLU
__device__ __forceinline__ float silu_bf16(float g) { return round_bf16(g / (1.0f + __expf(-g))); }

__global__ void __launch_bounds__(kThreads) swiglu_kernel(const uint16_t* __restrict__ g, int64_t ld_g,
                                                          const uint16_t* __restrict__ p, int64_t ld_p,
                                                          uint16_t* __restrict__ out, int64_t ld_o, int64_t M,
                                                          int64_t N, uint32_t* __restrict__ amax_out) {
  const int64_t nvr = N >> 3;
  const int64_t total = M * nvr;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  uint32_t am2 = 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += nthreads) {
    const int64_t m = i / nvr, c = (i - m * nvr) * 8;
    const uint4 g4 = ldg16(g + m * ld_g + c), p4 = ldg16(p + m * ld_p + c);
    const uint32_t gu[4] = {g4.x, g4.y, g4.z, g4.w}, pu[4] = {p4.x, p4.y, p4.z, p4.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[j] = pack_bf16x2(silu_bf16(bf_lo(gu[j])) * bf_lo(pu[j]), silu_bf16(bf_hi(gu[j])) * bf_hi(pu[j]));
      am2 = absmax_bf16x2(am2, o[j]);
    }
    *reinterpret_cast<uint4*>(out + m * ld_o + c) = make_uint4(o[0], o[1], o[2], o[3]);
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
  QIK_REQUIRE(aligned_elems(x_sb) && aligned_elems(x_ss) && aligned_elems(x_sh) && aligned_elems(o_sb) &&
                  aligned_elems(o_ss) && aligned_elems(o_sh),
              "qik_rms_norm_rope: strides must be multiples of 8 elements");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int rows_per_cta = (kThreads / 32) * (32 / static_cast<int>(D / 8));
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

int qik_layer_norm_modulate(const void* x, int64_t B, int64_t S, int64_t D, const void* modulation,
                            int64_t mod_rows, int64_t mod_stride, int64_t scale_off, const uint8_t* target_mask,
                            float eps, void* out, uint32_t* amax_out, void* stream) {
  QIK_REQUIRE(B >= 0 && S >= 0 && D > 0, "qik_layer_norm_modulate: bad sizes");
  if (B * S == 0) return QIK_OK;
  QIK_REQUIRE(x && modulation && out, "qik_layer_norm_modulate: NULL pointer");
  QIK_REQUIRE(D % 8 == 0 && D <= 4096, "qik_layer_norm_modulate: D must be a multiple of 8 and at most 4096");
  QIK_REQUIRE(aligned16(x) && aligned16(out) && aligned16(modulation),
              "qik_layer_norm_modulate: pointers must be 16-byte aligned");
  QIK_REQUIRE(aligned_elems(mod_stride) && aligned_elems(scale_off) && scale_off >= 0 && scale_off + D <= mod_stride,
              "qik_layer_norm_modulate: modulation stride/offset must be multiples of 8 with offset + D <= stride");
  QIK_REQUIRE(mod_rows >= (target_mask ? 2 * B : B),
              "qik_layer_norm_modulate: %lld modulation rows; B = %lld needs %s", static_cast<long long>(mod_rows),
              static_cast<long long>(B), target_mask ? "2B (rows B..2B-1 are the t = 0 rows)" : "B");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t rows = B * S;
  const int grid = grid_cap((rows + 7) / 8, 8);
  const int nv = static_cast<int>(D / 8);
  const uint16_t* xs = static_cast<const uint16_t*>(x);
  const uint16_t* ms = static_cast<const uint16_t*>(modulation);
  uint16_t* os = static_cast<uint16_t*>(out);
  if (nv <= 32 * 4)
    ln_modulate_kernel<4><<<grid, kThreads, 0, st>>>(xs, ms, mod_stride, scale_off, target_mask, os, B, S,
                                                     static_cast<int>(D), eps, amax_out);
  else if (nv <= 32 * 12)
    ln_modulate_kernel<12><<<grid, kThreads, 0, st>>>(xs, ms, mod_stride, scale_off, target_mask, os, B, S,
                                                      static_cast<int>(D), eps, amax_out);
  else
    ln_modulate_kernel<16><<<grid, kThreads, 0, st>>>(xs, ms, mod_stride, scale_off, target_mask, os, B, S,
                                                      static_cast<int>(D), eps, amax_out);
  return check_launch("ln_modulate_kernel");
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
  QIK_REQUIRE(aligned_elems(mod_stride) && aligned_elems(gate_off) && gate_off >= 0 && gate_off + D <= mod_stride,
              "qik_gate_residual: modulation stride/offset must be multiples of 8 with offset + D <= stride");
  QIK_REQUIRE(mod_rows >= (target_mask ? 2 * B : B), "qik_gate_residual: %lld modulation rows; B = %lld needs %s",
              static_cast<long long>(mod_rows), static_cast<long long>(B),
              target_mask ? "2B (rows B..2B-1 are the t = 0 rows)" : "B");
  const int64_t total = B * S * (D / 8);
  const int grid = grid_cap((total + kThreads - 1) / kThreads, 8);
  gate_residual_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
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
  const int grid = grid_cap((total + kThreads - 1) / kThreads, 8);
  swiglu_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(gate), ld_gate, static_cast<const uint16_t*>(up), ld_up,
      static_cast<uint16_t*>(out), ld_out, M, N, amax_out);
  return check_launch("swiglu_kernel");
}

}  // extern "C"
