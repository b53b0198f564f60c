/*
 * qik_oracle.c -- CPU restatement of the reference's byte-level quantizer math.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels under qwen-image-kernel_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may load it; the product path never does.
 *
 * What it restates (reference = gomezcojj-coder/qwen-image-kernel):
 *   - compute_scale           qwen_image_kernel/fp8.py:24-26
 *   - _scale_cast_fp8_kernel  qwen_image_kernel/fp8.py:29-41  (q = e4m3(x * (1/s)))
 *   - quantize_weight_tensorwise  qwen_image_kernel/fp8.py:56-60
 *   - _LayerView.store (fp8-V)    qwen_image_kernel/kv_cache.py:30-45
 *
 * Scale forms.  `x.abs().amax().float() / 448.0` is evaluated by PyTorch as a
 * true division on CPU but as a multiplication by the fp32 reciprocal
 * fl32(1/448) on CUDA (division by a CPU scalar).  The reference runs on CUDA,
 * so QIK_SCALE_CUDA is the product semantics; QIK_SCALE_CPU reproduces what the
 * reference's functions return when they are run on CPU tensors (used to check
 * this restatement against golden vectors produced by the reference itself).
 *
 * e4m3 (float8_e4m3fn): 1 sign, 4 exponent bits (bias 7), 3 mantissa bits, no
 * infinities, S.1111.111 is NaN, largest finite 448, smallest subnormal 2^-9.
 * Two conversions appear in the reference:
 *   - satfinite: the device cvt used by the activation cast (Triton's fp32->e4m3
 *     conversion on sm_89+): round-to-nearest-even, |x| > 448 -> 448, NaN -> NaN.
 *   - torch:     c10's software conversion used by `.to(torch.float8_e4m3fn)`
 *     (weights, slab V): round-to-nearest-even, results that round past 448
 *     become NaN.  The reference clamps to +-448 first, so only NaN inputs differ.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define QIK_SCALE_CUDA 0
#define QIK_SCALE_CPU 1
#define E4M3_MAX 448.0f
#define SCALE_FLOOR 1e-12f

static inline float bits_to_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bf16_to_f32(uint16_t h) { return bits_to_f32(((uint32_t)h) << 16); }

/* Round |a| (finite, >= 0) to the e4m3 grid with ties to even.  The grid
 * spacing for 2^E <= a < 2^(E+1) is 2^(E-3), and 2^-9 below 2^-6; dividing by a
 * power of two is exact in fp32 and rintf() rounds half to even. */
static float e4m3_round_abs(float a) {
    if (a == 0.0f) return 0.0f;
    int e;
    frexpf(a, &e);            /* a = f * 2^e, f in [0.5, 1) -> 2^(e-1) <= a < 2^e */
    int E = e - 1;
    if (E < -6) E = -6;
    float ulp = ldexpf(1.0f, E - 3);
    return rintf(a / ulp) * ulp;
}

/* Encode a value that is already on the e4m3 grid and <= 448. */
static uint8_t e4m3_encode_grid(float r, uint8_t sign) {
    if (r == 0.0f) return sign;
    int e;
    float f = frexpf(r, &e);  /* r = f * 2^e */
    int E = e - 1;            /* r = 2^E * (2f) with 2f in [1, 2) */
    if (E >= -6) {
        int m = (int)((2.0f * f - 1.0f) * 8.0f);
        return (uint8_t)(sign | ((E + 7) << 3) | m);
    }
    int m = (int)(r * 512.0f); /* subnormal: r = m * 2^-9 */
    return (uint8_t)(sign | m);
}

uint8_t qik_oracle_e4m3_satfinite(float x) {
    uint32_t u = f32_to_bits(x);
    uint8_t sign = (uint8_t)((u >> 24) & 0x80);
    float a = fabsf(x);
    if (isnan(a)) return 0x7F;
    if (a > E4M3_MAX) return (uint8_t)(sign | 0x7E);
    float r = e4m3_round_abs(a);
    if (r > E4M3_MAX) r = E4M3_MAX;
    return e4m3_encode_grid(r, sign);
}

uint8_t qik_oracle_e4m3_torch(float x) {
    uint32_t u = f32_to_bits(x);
    uint8_t sign = (uint8_t)((u >> 24) & 0x80);
    float a = fabsf(x);
    if (isnan(a) || a >= 480.0f) return (uint8_t)(sign | 0x7F);
    float r = e4m3_round_abs(a);
    if (r > E4M3_MAX) return (uint8_t)(sign | 0x7F);
    return e4m3_encode_grid(r, sign);
}

float qik_oracle_e4m3_to_f32(uint8_t b) {
    int sign = b & 0x80;
    int E = (b >> 3) & 0xF;
    int m = b & 7;
    float v;
    if (E == 15 && m == 7) v = NAN;
    else if (E == 0) v = ldexpf((float)m, -9);
    else v = ldexpf(1.0f + (float)m / 8.0f, E - 7);
    return sign ? -v : v;
}

/* max |x| over bf16 values; NaN propagates (torch.amax semantics). */
float qik_oracle_amax_bf16(const uint16_t* x, int64_t n) {
    uint16_t best = 0;
    for (int64_t i = 0; i < n; ++i) {
        uint16_t a = x[i] & 0x7FFF;
        if (a > 0x7F80) return NAN;       /* NaN */
        if (a > best) best = a;
    }
    return bf16_to_f32(best);
}

float qik_oracle_amax_f32(const float* x, int64_t n) {
    float best = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        float a = fabsf(x[i]);
        if (isnan(a)) return NAN;
        if (a > best) best = a;
    }
    return best;
}

/* s = clamp_min(amax / 448, 1e-12) in the requested evaluation form. */
float qik_oracle_scale_from_amax(float amax, int mode) {
    float s;
    if (mode == QIK_SCALE_CPU) {
        s = amax / E4M3_MAX;
    } else {
        const float recip = 1.0f / E4M3_MAX;   /* fl32(1/448) */
        s = amax * recip;
    }
    if (s < SCALE_FLOOR) s = SCALE_FLOOR;      /* NaN stays NaN, as torch.clamp_min */
    return s;
}

/* Activation cast of fp8.py:39-41: q = e4m3_satfinite(fl32(x) * inv), where inv
 * is the device's fp32 value of 1/s (passed in: the caller decides how the
 * reciprocal is formed). */
void qik_oracle_pack_act_bf16(const uint16_t* x, int64_t n, float inv, uint8_t* q) {
    for (int64_t i = 0; i < n; ++i) q[i] = qik_oracle_e4m3_satfinite(bf16_to_f32(x[i]) * inv);
}

/* Weight / slab-V cast of fp8.py:59 and kv_cache.py:40:
 * q = e4m3_torch(clamp(fl32(w) / s, -448, 448)) with IEEE division. */
static inline float clamp448(float v) {
    if (v < -E4M3_MAX) return -E4M3_MAX;
    if (v > E4M3_MAX) return E4M3_MAX;
    return v;                                  /* NaN passes through */
}

void qik_oracle_pack_div_bf16(const uint16_t* w, int64_t n, float s, uint8_t* q) {
    for (int64_t i = 0; i < n; ++i) q[i] = qik_oracle_e4m3_torch(clamp448(bf16_to_f32(w[i]) / s));
}

void qik_oracle_pack_div_f32(const float* w, int64_t n, float s, uint8_t* q) {
    for (int64_t i = 0; i < n; ++i) q[i] = qik_oracle_e4m3_torch(clamp448(w[i] / s));
}

/* Slab V store (kv_cache.py:36-42): v is [B, P, H, D] bf16 with arbitrary
 * strides (elements); v8 is written as [B, H, P, D] dense into a buffer whose
 * per-(b,h) row pitch is pmax*D; scale is [B, H]. */
void qik_oracle_slab_v_store(const uint16_t* v, int64_t B, int64_t P, int64_t H, int64_t D,
                             int64_t sb, int64_t sp, int64_t sh, int64_t pmax,
                             uint8_t* v8, float* scale, int mode) {
    for (int64_t b = 0; b < B; ++b) {
        for (int64_t h = 0; h < H; ++h) {
            uint16_t best = 0;
            int has_nan = 0;
            for (int64_t p = 0; p < P; ++p)
                for (int64_t d = 0; d < D; ++d) {
                    uint16_t a = v[b * sb + p * sp + h * sh + d] & 0x7FFF;
                    if (a > 0x7F80) has_nan = 1;
                    if (a > best) best = a;
                }
            float amax = has_nan ? NAN : bf16_to_f32(best);
            float s = qik_oracle_scale_from_amax(amax, mode);
            scale[b * H + h] = s;
            uint8_t* dst = v8 + (b * H + h) * pmax * D;
            for (int64_t p = 0; p < P; ++p)
                for (int64_t d = 0; d < D; ++d)
                    dst[p * D + d] = qik_oracle_e4m3_torch(clamp448(bf16_to_f32(v[b * sb + p * sp + h * sh + d]) / s));
        }
    }
}
