/*
 * qik.h -- C ABI of the B200-native (sm_100a) Qwen-Image FP8 DiT hot path.
 *
 * One shared library (libqik.so) exports these entry points.  They take plain
 * device pointers, sizes and a CUDA stream (as void*, a cudaStream_t; NULL = the
 * legacy default stream); no framework types cross the boundary.  Every entry
 * point is asynchronous on the given stream, allocates nothing, and returns a
 * status code (QIK_OK = 0); qik_last_error() gives the message of the last
 * failure on the calling thread.  Kernels never trap: a device-side failure (a
 * bounded wait that ran out) is written to the optional `status` word, which the
 * caller reads when it synchronizes.
 *
 * Each entry point names the reference interface it replaces
 * (gomezcojj-coder/qwen-image-kernel, file:line).
 */
#ifndef QIK_H_
#define QIK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QIK_OK 0
#define QIK_ERR_INVALID 1     /* bad pointer, shape, stride or alignment */
#define QIK_ERR_CUDA 2        /* a CUDA runtime/driver call failed */
#define QIK_ERR_UNSUPPORTED 3 /* valid request this build does not implement */

/* Element types used in `dtype` arguments. */
#define QIK_DTYPE_BF16 0
#define QIK_DTYPE_F32 1
#define QIK_DTYPE_E4M3 2

/* Device-side status word values (written to `status` when non-NULL). */
#define QIK_STATUS_OK 0
#define QIK_STATUS_TIMEOUT 1

/* Library version (major*10000 + minor*100 + patch). */
int qik_version(void);
/* Message for the last non-zero status returned on this thread. */
const char* qik_last_error(void);

/* Bytes of scratch `ws` the quantizer entry points need (16-byte aligned; 1024). */
size_t qik_quant_workspace_bytes(void);

/*
 * Dynamic per-tensor scale: *scale_out = clamp_min(amax|x| * fl32(1/448), 1e-12),
 * fp32, on the device.  Replaces compute_scale (qwen_image_kernel/fp8.py:24-26),
 * evaluated as the reference evaluates it on CUDA.
 *   x: n elements of `dtype` (BF16 or F32), contiguous.
 */
int qik_compute_scale(const void* x, int dtype, int64_t n, float* scale_out, void* ws, void* stream);

/*
 * max|x| accumulated into *amax_bits as the fp32 bit pattern (atomicMax; the caller
 * zeroes it first): the `x.abs().amax()` of compute_scale
 * (qwen_image_kernel/fp8.py:26).  Non-negative floats order like their bit
 * patterns, so an integer MAX reduction of amax_bits across shards (e.g. a 4-byte
 * all-reduce) yields the amax of the whole tensor; qik_quantize_act_from_amax then
 * quantizes each shard with the global scale.
 */
int qik_amax(const void* x, int dtype, int64_t n, uint32_t* amax_bits, void* stream);

/*
 * Dynamic per-tensor e4m3 activation quantization: scale as qik_compute_scale,
 * q[i] = e4m3_rn_satfinite(fl32(x[i]) * (1/scale)).  Replaces quantize_tensorwise
 * + _scale_cast_fp8_kernel (qwen_image_kernel/fp8.py:29-53).
 *   x: n bf16, contiguous; q: n bytes; scale_out: 1 fp32 (device).
 *   ws: qik_quant_workspace_bytes() bytes that carry a grid-barrier state from one
 *       call to the next: zero them once before the first call, then keep passing
 *       the same workspace (every completed call leaves it ready for the next, so
 *       the call is a single kernel launch with no clearing).  Calls sharing one
 *       workspace must be ordered (one stream); give each stream its own.  When a
 *       call fails (non-zero return, or a NaN *scale_out: a bounded wait inside the
 *       kernel gave up), zero the workspace again before reusing it.  With x, q or
 *       ws not 16-byte aligned the call takes a two-pass form that keeps no state.
 */
int qik_quantize_act(const void* x, int64_t n, uint8_t* q, float* scale_out, void* ws, void* stream);

/*
 * qik_quantize_act without a workspace argument, for callers that cannot
 * allocate device memory: plugin hosts and serving runtimes that hand a kernel
 * only its inputs and outputs from a pre-planned pool, and code that must not
 * call cudaMalloc (or torch's allocator) on its launch path.  Same result as
 * qik_quantize_act (bytes and scale).  No counterpart in the reference: it is an
 * addition of this library.
 *
 * The scratch lives in one file-scope __device__ array of
 * QIK_NOALLOC_SCRATCH_BYTES bytes that every GPU loading the library holds until
 * the process exits; this entry point needs qik_quant_workspace_bytes() of it for
 * any n and returns QIK_ERR_INVALID if that ever exceeds the array.  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress);
 * make that first call before any stream capture.  The address is cached per
 * device ordinal for the life of the process, which assumes the device's primary
 * context is never reset (cudaDeviceReset) while the library is loaded.  All calls
 * share the array; each call clears the array's barrier word on the stream before
 * its kernel runs (the rest of the array needs no clearing), so calls that overlap
 * on the GPU (different streams, or different host threads on one device) race;
 * serialize them.
 */
#define QIK_NOALLOC_SCRATCH_BYTES 1024
int qik_quantize_act_noalloc(const void* x, int64_t n, uint8_t* q, float* scale_out, void* stream);

/*
 * e4m3 activation pack with a scale already on the device (the second half of
 * qik_quantize_act, used after a producer kernel accumulated the amax):
 *   amax_bits: fp32 bit pattern of max|x| (as written by qik_fp8_gemm's amax_out).
 * Writes *scale_out and q as qik_quantize_act does.
 */
int qik_quantize_act_from_amax(const void* x, int64_t n, const uint32_t* amax_bits, uint8_t* q, float* scale_out,
                               void* stream);

/*
 * Static per-tensor e4m3 weight quantization: scale as qik_compute_scale,
 * q[i] = e4m3(clamp(fl32(w[i]) / scale, -448, 448)) with IEEE division.
 * Replaces quantize_weight_tensorwise (qwen_image_kernel/fp8.py:56-60) and the
 * per-linear step of _staged_quantize (qwen_image_kernel/quantize_offline.py:19-26).
 *   w: n elements of `dtype` (BF16 or F32), contiguous.
 */
int qik_quantize_weight(const void* w, int dtype, int64_t n, uint8_t* q, float* scale_out, void* ws, void* stream);

/* Epilogue selectors for qik_fp8_gemm. */
#define QIK_EPI_SCALE 0      /* y = acc * sa * sb (+ bias) */
#define QIK_EPI_GELU_TANH 1  /* y = gelu_tanh(bf16(acc * sa * sb (+ bias))) */
#define QIK_EPI_SCATTER 2    /* fp32 acc * sa * sb rows to their owner rank (qik_fp8_gemm_scatter) */
#define QIK_EPI_SWIGLU 3     /* SwiGLU of the fused gate / up linear (B rows [0, N/2) gate, [N/2, N)
                                up, as fused_swiglu's chunk(2) splits them): C[:, j] =
                                bf16(bf16(silu(g_j)) * u_j), g_j, u_j the bf16 outputs of B rows j
                                and N/2 + j (+ bias); C has N / 2 columns; N % 256 == 0, BF16 */
#define QIK_EPI_RMS_ROPE 4   /* the fused QKV linear with per-head RMSNorm + RoPE of q and k
                                (qik_fp8_gemm_qkv_rms_rope only) */
#define QIK_EPI_GATE_RES 5   /* gated residual x + bf16(bf16(tanh(gate)) * y) of the bf16 output y
                                (qik_fp8_gemm_gate_residual only) */

/*
 * FP8 GEMM on tcgen05: C[M,N] = epilogue(A[M,K] . B[N,K]^T), e4m3 x e4m3 with
 * fp32 accumulation in tensor memory.  Replaces the torch._scaled_mm call of
 * FP8Linear.forward (qwen_image_kernel/fp8.py:87-88).
 *   A: row-major [M, K] e4m3, row pitch lda bytes (lda % 16 == 0, K % 16 == 0)
 *   B: row-major [N, K] e4m3 (the FP8Linear weight buffer), row pitch ldb bytes
 *   scale_a, scale_b: 1 fp32 each (device)
 *   bias: N bf16 or NULL
 *   C: row-major [M, N] of out_dtype (BF16 or F32), row pitch ldc elements
 *      (N % 16 == 0, ldc % 8 == 0, C 16-byte aligned); [M, N / 2] for QIK_EPI_SWIGLU
 *   epilogue: QIK_EPI_*; QIK_EPI_SWIGLU always runs on CTA-pair 256 x 256 tiles
 *      (a tile holds 128 gate and the matching 128 up columns)
 *   amax_out: NULL, or a u32 that receives atomicMax of the fp32 bit patterns of
 *      |C| (BF16 output only): the amax of the next dynamic quantization.
 *   status: NULL or a device int set to QIK_STATUS_TIMEOUT on a failed wait.
 */
int qik_fp8_gemm(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                 const float* scale_a, const float* scale_b, const void* bias, void* C, int64_t ldc, int out_dtype,
                 int epilogue, uint32_t* amax_out, int* status, void* stream);

/* Tile configurations of the FP8 GEMM (qik_fp8_gemm_tiled). */
#define QIK_GEMM_TILE_AUTO 0        /* the configuration qik_fp8_gemm picks for (M, N) */
#define QIK_GEMM_TILE_PAIR_256 1    /* CTA pairs (cta_group::2), 256 x 256 tiles */
#define QIK_GEMM_TILE_SINGLE_256 2  /* single CTAs, 128 x 256 tiles */
#define QIK_GEMM_TILE_SINGLE_128 3  /* single CTAs, 128 x 128 tiles */
#define QIK_GEMM_TILE_SINGLE_64 4   /* single CTAs, 128 x 64 tiles */
#define QIK_GEMM_TILE_SWAP_16 5     /* M <= 16 only: operands swapped, 128 weight rows x 16 activation rows */
/* Tile raster, or-ed into tile_cfg: output tiles walked in groups of g (1..255) row
 * tiles, each group column tile by column tile (g = 1: row-major); 0 = what
 * qik_fp8_gemm picks. */
#define QIK_GEMM_RASTER(g) ((g) << 8)

/*
 * qik_fp8_gemm with the tile configuration forced (QIK_GEMM_TILE_*, optionally or-ed
 * with QIK_GEMM_RASTER(g); AUTO = what qik_fp8_gemm picks).  Every configuration
 * computes the same result; this entry point exists for measurement and for tests that
 * cover each configuration.  No counterpart in the reference (its GEMM is cuBLASLt's
 * choice).
 */
int qik_fp8_gemm_tiled(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K, int64_t lda,
                       int64_t ldb, const float* scale_a, const float* scale_b, const void* bias, void* C,
                       int64_t ldc, int out_dtype, int epilogue, uint32_t* amax_out, int tile_cfg, int* status,
                       void* stream);

/*
 * The fused QKV linear followed by the per-head RMSNorm + RoPE of its q and k heads, in
 * one GEMM: replaces fused_qkv(hidden_states) and the two fused_rms_norm_rope calls of
 * QwenImage21AttnProcessor.__call__ (qwen_image_kernel/processors.py:64-79).  B is the
 * fused weight [3 heads head_dim, K] (q rows, then k, then v), C bf16 [M, 3 heads
 * head_dim] with row pitch ldc: the q and k columns hold rms_norm_rope(bf16 GEMM output)
 * exactly as qik_rms_norm_rope computes it on that output (w_q / w_k fp32 [head_dim],
 * rope_cos / rope_sin fp32 [seq, head_dim / 2] at position row % seq, eps), the v
 * columns the bf16 GEMM output.  head_dim == 128, M % seq == 0; runs on CTA-pair tiles.
 */
int qik_fp8_gemm_qkv_rms_rope(const uint8_t* A, const uint8_t* B, int64_t M, int64_t K, int64_t lda, int64_t ldb,
                              const float* scale_a, const float* scale_b, const void* bias, void* C, int64_t ldc,
                              int heads, int head_dim, const float* w_q, const float* w_k, const float* rope_cos,
                              const float* rope_sin, int64_t seq, float eps, int* status, void* stream);

/*
 * bf16(tanh(modulation[r, gate_off + c])) for r < mod_rows, c < D, as the gated residual
 * computes it (qik_gate_residual): the table qik_fp8_gemm_gate_residual reads, [mod_rows,
 * D] bf16 contiguous.  Part of the reference's fused_gate_residual
 * (qwen_image_kernel/triton_fused.py:183-231).
 */
int qik_gate_table(const void* modulation, int64_t mod_rows, int64_t mod_stride, int64_t gate_off, int64_t D,
                   void* table, void* stream);

/*
 * An FP8 linear followed by the DiT block's gated residual, in one GEMM: replaces
 * attn.to_out[0](...) / img_mlp.out(...) and the fused_gate_residual call after it
 * (qwen_image_kernel/processors.py:172-187, triton_fused.py:183-231).  C [M, N] bf16 =
 * x + bf16(T[t] * y), y the bf16 linear output (qik_fp8_gemm with QIK_EPI_SCALE), x
 * bf16 [M, N] (row pitch ldx), T the qik_gate_table output (row pitch ldt) and, for row
 * b * seq + s, t = b when target_mask is NULL or target_mask[s] != 0, else batch + b (the
 * table then has 2 batch rows).  The bytes equal qik_gate_residual on y, except where a
 * product T * y lies below 2^-126 in magnitude (rounded once here, twice there).
 * M == batch * seq; C must not alias x.
 */
int qik_fp8_gemm_gate_residual(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K, int64_t lda,
                               int64_t ldb, const float* scale_a, const float* scale_b, const void* bias,
                               const void* x, int64_t ldx, const void* gate_table, int64_t ldt,
                               const uint8_t* target_mask, int64_t batch, int64_t seq, void* C, int64_t ldc,
                               int* status, void* stream);

/*
 * Bytes of workspace qik_fp8_ffn needs for an [M, K] input and a hidden width.
 */
size_t qik_fp8_ffn_workspace_bytes(int64_t M, int64_t K, int64_t hidden);

/*
 * DiT FFN pair y = down(gelu_tanh(up(x))), both linears FP8 per-tensor with the
 * hidden activation re-quantized dynamically: two FP8Linear.forward calls
 * (qwen_image_kernel/fp8.py:78-90) with GELU-tanh between them, run as one chain
 * of four kernels (single-pass quantizer of x, GEMM+GELU+amax, pack, GEMM; amax and
 * pack of x instead of the single pass when x is not 16-byte aligned) with
 * programmatic dependent launches.
 *   x: [M, K] bf16 row-major; w_up: [hidden, K] e4m3, s_up: 1 fp32, b_up: hidden bf16
 *   or NULL; w_down: [K, hidden] e4m3, s_down, b_down likewise; y: [M, K] bf16.
 *   ws: qik_fp8_ffn_workspace_bytes(M, K, hidden) bytes, 256-byte aligned (holds the
 *   quantized input, the bf16 and e4m3 hidden activations and the scales).
 */
int qik_fp8_ffn(const void* x, int64_t M, int64_t K, int64_t hidden, const uint8_t* w_up, const float* s_up,
                const void* b_up, const uint8_t* w_down, const float* s_down, const void* b_down, void* y, void* ws,
                size_t ws_bytes, int* status, void* stream);

/*
 * qik_fp8_ffn with max|x| supplied: x_amax_bits holds the fp32 bits of max|x| (as the
 * amax outputs of qik_layer_norm_modulate / qik_swiglu accumulate it), so the chain
 * starts at the pack of x.  Same result as qik_fp8_ffn on the same x.
 */
int qik_fp8_ffn_from_amax(const void* x, const uint32_t* x_amax_bits, int64_t M, int64_t K, int64_t hidden,
                          const uint8_t* w_up, const float* s_up, const void* b_up, const uint8_t* w_down,
                          const float* s_down, const void* b_down, void* y, void* ws, size_t ws_bytes, int* status,
                          void* stream);

/*
 * qik_fp8_ffn with x already quantized by its producer: xq holds the [M, K] e4m3 codes
 * of x (16-byte aligned) and x_scale their dynamic scale (as
 * qik_layer_norm_modulate_e4m3 emits them), so the chain starts at the up-projection
 * GEMM.  Same result as qik_fp8_ffn on the x those codes quantize.
 */
int qik_fp8_ffn_e4m3(const uint8_t* xq, const float* x_scale, int64_t M, int64_t K, int64_t hidden,
                     const uint8_t* w_up, const float* s_up, const void* b_up, const uint8_t* w_down,
                     const float* s_down, const void* b_down, void* y, void* ws, size_t ws_bytes, int* status,
                     void* stream);

/* Attention flags. */
#define QIK_ATTN_HAS_CACHE 1     /* keys/values = virtual concat [cache ; fresh] */
#define QIK_ATTN_HAS_KEY_VALID 2 /* per-(batch, key) validity bytes */
#define QIK_ATTN_UNIFORM 4       /* every row attends to [0, P+SN): L unused */
#define QIK_ATTN_V_FP8 8         /* cache V is e4m3 with per-(batch, head) scales */
#define QIK_ATTN_F16 16          /* q / k / v / cache K (and a 16-bit cache V) / out are fp16, not bf16 */

/* Strides are in elements of the tensor they describe. */
typedef struct qik_attn_args {
  const void* q;       /* [B, SQ, H, D] bf16 (fp16 with QIK_ATTN_F16) */
  const void* k;       /* [B, SN, H, D] fresh keys, q's type */
  const void* v;       /* [B, SN, H, D] fresh values, q's type */
  const void* cache_k; /* [B, P, H, D] q's type, or NULL */
  const void* cache_v; /* [B, P, H, D] q's type or e4m3, or NULL */
  const float* cache_v_scale; /* [B, H] fp32 (V_FP8 only) */
  const int32_t* L;    /* [SQ]: row attends kv iff 0 <= kv <= L[row]; -1 -> no key */
  const uint8_t* key_valid; /* [B, P + SN] bytes, non-zero = valid (HAS_KEY_VALID) */
  void* out;           /* [B, SQ, H, D] q's type */
  int64_t B, SQ, SN, P, H, D;
  int64_t q_sb, q_ss, q_sh;
  int64_t k_sb, k_ss, k_sh;
  int64_t v_sb, v_ss, v_sh;
  int64_t ck_sb, ck_ss, ck_sh;
  int64_t cv_sb, cv_ss, cv_sh;
  int64_t o_sb, o_ss, o_sh;
  int64_t kv_sb;       /* key_valid batch stride */
  float sm_scale;      /* softmax scale, D^-0.5 in the reference */
  int flags;           /* QIK_ATTN_* */
  uint32_t* amax_out;  /* NULL, or one device word that receives (atomic max) the fp32 bits of
                          max|out| over the rows written: the dynamic scale of the FP8
                          out-projection that consumes out, without a pass over out */
} qik_attn_args;

/*
 * Block-causal flash attention over [prefix slab ; fresh K/V] with per-row
 * prefix lengths, optional key validity and an e4m3 slab V dequantized in the
 * loop as bf16(fl32(v8) * scale[b, h]).  Replaces block_causal_flash_attention
 * + _qwen21_attn_fwd (qwen_image_kernel/triton_attention.py:35-260), for bf16 or
 * (QIK_ATTN_F16) fp16 tensors as the reference accepts both
 * (triton_attention.py:190): P is rounded to the tensors' type before P.V
 * (triton_attention.py:162-163), fp32 accumulation.
 * Requires D == 128 and unit stride along D; rows with no allowed key give 0.  SN may be
 * 0 (the rows attend to the cache alone; k and v are then not read and may be NULL).
 */
int qik_block_causal_attention(const qik_attn_args* args, int* status, void* stream);

/*
 * Prefix-KV slab store for one layer: K copied to [B, H, Pmax, D] bf16; V either
 * copied (bf16) or quantized per (b, h): s = clamp_min(amax * fl32(1/448), 1e-12),
 * v8 = e4m3(clamp(fl32(v) / s, -448, 448)).  Replaces _LayerView.store
 * (qwen_image_kernel/kv_cache.py:30-45).
 *   k, v: [B, P, H, D] bf16 with element strides (sb, sp, sh) and unit D stride
 *   k_layer: K slab of the layer, [B, H, pmax, D] bf16 dense
 *   v_layer: V slab of the layer, [B, H, pmax, D] (bf16, or e4m3 when v_fp8)
 *   v_scale_layer: [B, H] fp32 (v_fp8 only); ws: qik_quant_workspace_bytes() * B*H
 */
int qik_kv_store(const void* k, const void* v, int64_t B, int64_t P, int64_t H, int64_t D, int64_t k_sb,
                 int64_t k_sp, int64_t k_sh, int64_t v_sb, int64_t v_sp, int64_t v_sh, void* k_layer, void* v_layer,
                 int64_t pmax, int v_fp8, float* v_scale_layer, void* ws, void* stream);

/*
 * Per-head RMSNorm + rotary embedding of one of q / k: for every (b, s, h) row of D,
 * rrms = rsqrt(sum(x^2) / D + eps), n = bf16(x * rrms * weight), then each pair
 * (n[2i], n[2i+1]) is rotated by (cos[s, i], sin[s, i]); bf16 out.  Replaces
 * fused_rms_norm_rope + rms_rope_kernel (qwen_image_kernel/triton_fused.py:28-105);
 * unlike the reference it reads strided q / k views of the fused QKV output directly.
 *   x: [B, S, H, D] bf16, element strides (x_sb, x_ss, x_sh), unit D stride
 *   weight: D fp32; cos_tab, sin_tab: [S, D/2] fp32 (rows contiguous)
 *   out: [B, S, H, D] bf16 with strides (o_sb, o_ss, o_sh)
 *   D in {64, 128, 256}; pointers 16-byte aligned, strides multiples of 8.
 */
int qik_rms_norm_rope(const void* x, int64_t B, int64_t S, int64_t H, int64_t D, int64_t x_sb, int64_t x_ss,
                      int64_t x_sh, const float* weight, const float* cos_tab, const float* sin_tab, float eps,
                      void* out, int64_t o_sb, int64_t o_ss, int64_t o_sh, void* stream);

/*
 * LayerNorm (no affine, fp32 mean and centred variance, bf16 result) times
 * bf16(1 + scale), the scale row chosen per position: row b where target_mask[s]
 * is non-zero (or target_mask is NULL), row B + b elsewhere (the t = 0 rows).
 * Replaces fused_layer_norm_modulate + ln_modulate_kernel and _modulation_row_map
 * (qwen_image_kernel/triton_fused.py:111-177).
 *   x, out: [B, S, D] bf16 contiguous; modulation: mod_rows rows of mod_stride bf16
 *   (at least B rows, 2B with a target_mask), scale at column scale_off;
 *   target_mask: S bytes or NULL; D % 8 == 0, D <= 4096.
 *   amax_out: NULL, or a u32 receiving atomicMax of the fp32 bit patterns of |out|
 *   (the amax of the next linear's dynamic quantization; the caller zeroes it).
 */
int qik_layer_norm_modulate(const void* x, int64_t B, int64_t S, int64_t D, const void* modulation,
                            int64_t mod_rows, int64_t mod_stride, int64_t scale_off, const uint8_t* target_mask,
                            float eps, void* out, uint32_t* amax_out, void* stream);

/*
 * qik_layer_norm_modulate feeding an FP8 linear: the same bf16 outputs, quantized
 * with their own dynamic per-tensor scale exactly as qik_quantize_act would quantize
 * them (same codes, same scale), without the bf16 tensor ever being written.
 * Replaces fused_layer_norm_modulate (qwen_image_kernel/triton_fused.py:111-177)
 * followed by the quantize_tensorwise of the next FP8Linear.forward
 * (qwen_image_kernel/fp8.py:44-53, 85-86).  One cooperative kernel: the rows are
 * normalized twice, once for max|out| and, after a grid-wide exchange, once for the
 * codes (the second read of x comes from L2 while x fits there).
 *   q: [B, S, D] e4m3 (16-byte aligned); scale_out: 1 fp32 (device).
 *   ws: qik_quant_workspace_bytes() bytes with the qik_quantize_act contract (zero
 *       once, then reuse in stream order; zero again after a failed call).
 *   status: NULL or a device int set to QIK_STATUS_TIMEOUT on a failed wait (the
 *       scale is then NaN).
 * Other arguments and limits as qik_layer_norm_modulate.
 */
int qik_layer_norm_modulate_e4m3(const void* x, int64_t B, int64_t S, int64_t D, const void* modulation,
                                 int64_t mod_rows, int64_t mod_stride, int64_t scale_off, const uint8_t* target_mask,
                                 float eps, uint8_t* q, float* scale_out, void* ws, int* status, void* stream);

/*
 * Gated residual out = x + bf16(tanh(gate)) * f in bf16 arithmetic, the gate row
 * chosen per position as in qik_layer_norm_modulate.  Replaces fused_gate_residual
 * + gate_residual_kernel (qwen_image_kernel/triton_fused.py:183-231).
 *   x, f, out: [B, S, D] bf16 contiguous, out distinct from x and f; gate at column gate_off.
 */
int qik_gate_residual(const void* x, const void* f, int64_t B, int64_t S, int64_t D, const void* modulation,
                      int64_t mod_rows, int64_t mod_stride, int64_t gate_off, const uint8_t* target_mask, void* out,
                      void* stream);

/*
 * SwiGLU out = bf16(bf16(silu(gate)) * up).  Replaces fused_swiglu + swiglu_kernel
 * (qwen_image_kernel/triton_fused.py:237-263); gate and up may be the two halves of
 * the fused up-projection output (row pitches ld_*, in elements), read in place.
 *   [M, N] bf16 each; N and the pitches multiples of 8; amax_out as in
 *   qik_layer_norm_modulate (for the down projection's quantizer).
 */
int qik_swiglu(const void* gate, int64_t ld_gate, const void* up, int64_t ld_up, int64_t M, int64_t N, void* out,
               int64_t ld_out, uint32_t* amax_out, void* stream);

/* ---------------------------------------------------------------- tensor parallel
 * Row-parallel FP8 linear with the reduction over peer memory, replacing the
 * fp32 partial product + NCCL all-reduce of the tensor-parallel block stack
 * (4 DiT blocks tensor parallel over the GPUs; the reference itself is single-GPU: its
 * FP8Linear.forward is qwen_image_kernel/fp8.py:78-90).  One process per GPU; every
 * rank maps its peers' workspaces (CUDA IPC) and calls, in the same order:
 *   qik_fp8_gemm_scatter   (its GEMM's fp32 rows stored straight into the owner
 *                           rank's receive slot over NVLink, tile by tile, each tile
 *                           counted at the owner with a system-scope atomic),
 *   qik_tp_reduce_gather   (the owner sums its rows over the ranks in rank order,
 *                           adds the bias, stores bf16 rows into every rank's output
 *                           and counts them there),
 *   qik_tp_wait            (this rank waits until every owner's rows arrived).
 * Rank o owns rows [o R, min((o + 1) R, M)), R a multiple of 256.  Counters only grow:
 * call number e waits for e x the per-call count (uint32 arithmetic modulo 2^32), and
 * the receive slots alternate with the parity of e.  Every wait is bounded (status
 * QIK_STATUS_TIMEOUT); no multicast is used.
 */
#define QIK_TP_MAX_WORLD 8

/* Bytes of a CUDA IPC memory handle (cudaIpcMemHandle_t). */
size_t qik_ipc_handle_bytes(void);

/*
 * Export the allocation holding `ptr`: writes its IPC handle (qik_ipc_handle_bytes()
 * bytes) and the offset of `ptr` from the allocation's base.
 */
int qik_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out);

/*
 * Map a peer's exported allocation into this process: *base_out is the mapped base
 * (to pass to qik_ipc_close), the exported pointer is *base_out + offset.
 */
int qik_ipc_open(const void* handle, void** base_out);
int qik_ipc_close(void* base);

/*
 * Arrivals qik_fp8_gemm_scatter produces per call at owner `owner` from one rank
 * (tiles whose first row the owner holds x tiles across N x CTAs per tile).
 */
int64_t qik_fp8_gemm_scatter_signals(int64_t M, int64_t N, int64_t rows_per_owner, int owner);

/*
 * Partial product of a row-parallel linear: P = A . B^T * sa * sb (fp32, no bias),
 * row r stored at dst[r / R] + (r mod R) * N and, after each tile, one
 * atomicAdd (system scope) of 1 at cnt[owner].
 *   A [M, K] e4m3 (this rank's K slice), B [N, K] e4m3; dst / cnt: host arrays of
 *   `world` device pointers (peer memory for other owners); status as qik_fp8_gemm.
 */
int qik_fp8_gemm_scatter(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K, int64_t lda,
                         int64_t ldb, const float* scale_a, const float* scale_b, int world, int64_t rows_per_owner,
                         float* const* dst, uint32_t* const* cnt, int* status, void* stream);

/*
 * Owner step: waits until cnt_in[s] reached cnt_target (as signed 32-bit distance) for
 * every rank s, then out_p[row, :] = bf16(sum_{s = 0..world-1} recv[s][row - o R, :]
 * (+ bias)) for its rows, into every rank p's output out[p] ([M, N] bf16), and one
 * atomicAdd (system scope) of 1 per CTA at gcnt[p]; `ctas` CTAs (the per-call count).
 *   recv: world slots of R x N fp32, slot s at recv + s R N.
 */
int qik_tp_reduce_gather(const float* recv, const uint32_t* cnt_in, uint32_t cnt_target, int world, int owner,
                         int64_t M, int64_t N, int64_t rows_per_owner, const void* bias, void* const* out,
                         uint32_t* const* gcnt, int ctas, int* status, void* stream);

/* Waits until gcnt[o] reached target for every owner o (this rank's counters). */
int qik_tp_wait(const uint32_t* gcnt, uint32_t target, int world, int* status, void* stream);

/*
 * Sequence-parallel form of the TP stack: after the reduce-scatter of a row-parallel
 * linear's fp32 partial products, this rank's rows x [rows, N] become
 * out = bf16(x + bias) (bias bf16 [N] or NULL; fp32 add, one rounding) with max|out|
 * accumulated into *amax_out (fp32 bits, atomic max; NULL to skip) for the next FP8
 * linear's dynamic scale.  The bias add and bf16 output of FP8Linear.forward
 * (qwen_image_kernel/fp8.py:86-90), applied once after the sum over the ranks.
 * N a multiple of 8; x, out, bias 16-byte aligned.
 */
int qik_rows_bias_bf16(const float* x, int64_t rows, int64_t N, const void* bias, void* out, uint32_t* amax_out,
                       void* stream);

/*
 * Self-test of the bounded-wait machinery: launches one CTA that waits on an
 * mbarrier nothing will ever complete, with a limit of `wait_ns` nanoseconds, and
 * writes QIK_STATUS_TIMEOUT to *status when the wait gives up.  The GPU context
 * stays usable afterwards.
 */
int qik_selftest_wait_timeout(int* status, uint64_t wait_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QIK_H_ */
