// qik_ffn.cu -- the DiT FFN pair as one chain of launches.
//
// y = down(gelu_tanh(up(x))) with both linears FP8 per-tensor: two applications of
// FP8Linear.forward (qwen_image_kernel/fp8.py:78-90) with GELU-tanh between them
// (the DiT FFN pair 3072 -> 12288 -> 3072; the reference block uses SwiGLU through a fused up
// projection, processors.py:180-187), the hidden activation re-quantized
// dynamically.  Four kernels in one stream (five without the single pass):
//   quantize(x) -> GEMM1 (+GELU, amax(h)) -> pack(h) -> GEMM2
// where quantize(x) is the single-pass cooperative quantizer (x 16-byte aligned) or
// amax(x) -> pack(x) (qik_fp8_ffn_from_amax: pack(x) alone, with max|x| from x's
// producer; qik_fp8_ffn_e4m3: nothing, x arrives quantized from its producer).
// Every kernel after the quantizer is launched as a programmatic dependent of its
// predecessor, so its launch and set-up (TMEM allocation, barrier init, descriptor
// prefetch) overlap the predecessor's tail; each waits for the predecessor's
// results before reading them.  The intermediates live in the caller's workspace.
#include "qik_device.cuh"
#include "qik_host.h"

namespace qik {
namespace {
struct FfnHeader {
  uint32_t amax_x;
  uint32_t amax_h;
  float sx;
  float sh;
};
constexpr size_t kAlign = 256;
// workspace head: the single-pass quantizer's workspace (1 KB), then the chain's
// header words; one memset per call clears both (the quantizer's barrier state and
// amax_h, which GEMM1's epilogue accumulates into)
constexpr size_t kQuantWsBytes = 1024;
constexpr size_t kHeaderOffset = kQuantWsBytes;
constexpr size_t kHeadBytes = 1280;
size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }
}  // namespace
}  // namespace qik

using namespace qik;

extern "C" size_t qik_fp8_ffn_workspace_bytes(int64_t M, int64_t K, int64_t hidden) {
  if (M <= 0 || K <= 0 || hidden <= 0) return kHeadBytes;
  return kHeadBytes + align_up(static_cast<size_t>(M) * K) + align_up(static_cast<size_t>(M) * hidden * 2) +
         align_up(static_cast<size_t>(M) * hidden);
}

// x_amax: NULL (the chain computes max|x| itself) or the fp32 bits of max|x| already
// accumulated by x's producer (a layer norm's or SwiGLU's amax output).  x_scale: NULL,
// or x is already the e4m3 input ([M, K] codes) quantized with the scale *x_scale.
static int fp8_ffn_chain(const void* x, const uint32_t* x_amax, const float* x_scale, int64_t M, int64_t K,
                         int64_t hidden, const uint8_t* w_up, const float* s_up, const void* b_up,
                         const uint8_t* w_down, const float* s_down, const void* b_down, void* y, void* ws,
                         size_t ws_bytes, int* status, void* stream) {
  QIK_REQUIRE(M >= 0 && K > 0 && hidden > 0, "qik_fp8_ffn: bad sizes");
  if (M == 0) return QIK_OK;
  QIK_REQUIRE(x && w_up && s_up && w_down && s_down && y && ws, "qik_fp8_ffn: NULL pointer");
  QIK_REQUIRE(ws_bytes >= qik_fp8_ffn_workspace_bytes(M, K, hidden), "qik_fp8_ffn: workspace of %zu bytes too small",
              ws_bytes);
  QIK_REQUIRE((reinterpret_cast<uintptr_t>(ws) & (kAlign - 1)) == 0, "qik_fp8_ffn: workspace must be 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* base = static_cast<uint8_t*>(ws);
  QuantWs* qws = reinterpret_cast<QuantWs*>(base);
  FfnHeader* hdr = reinterpret_cast<FfnHeader*>(base + kHeaderOffset);
  uint8_t* xq_ws = base + kHeadBytes;  // the quantized input, unless the caller passed it
  void* h = xq_ws + align_up(static_cast<size_t>(M) * K);
  uint8_t* hq = static_cast<uint8_t*>(h) + align_up(static_cast<size_t>(M) * hidden * 2);
  const uint8_t* xq = x_scale ? static_cast<const uint8_t*>(x) : xq_ws;
  const float* sx = x_scale ? x_scale : &hdr->sx;

  QIK_TRY_CUDA(cudaMemsetAsync(base, 0, kHeaderOffset + sizeof(FfnHeader), st));
  int rc = QIK_OK;
  if (x_scale) {
    // quantized by its producer
  } else if (x_amax) {
    rc = launch_pack_act(x, M * K, x_amax, xq_ws, &hdr->sx, st, false);
  } else if (aligned16(x)) {
    // one kernel: x read from HBM once (it fits the SMs' shared memory up to ~28 MB)
    rc = launch_quant_single_pass(x, M * K, xq_ws, &hdr->sx, qws, st, false);
  } else {
    rc = launch_amax(x, QIK_DTYPE_BF16, M * K, &hdr->amax_x, st, false);
    if (!rc) rc = launch_pack_act(x, M * K, &hdr->amax_x, xq_ws, &hdr->sx, st, true);
  }
  // h larger than a few MB: stored with an L2 evict-last policy, so more of it is still
  // in L2 when the pack below reads it
  const bool keep_h = static_cast<int64_t>(M) * hidden * 2 > (int64_t{32} << 20);
  if (!rc)
    rc = launch_fp8_gemm(xq, w_up, M, hidden, K, K, K, sx, s_up, b_up, h, hidden, QIK_DTYPE_BF16,
                         QIK_EPI_GELU_TANH, &hdr->amax_h, status, st, x_scale == nullptr, keep_h);
  // backward: h was just written by GEMM1 in row order and exceeds what L2 keeps of it
  if (!rc) rc = launch_pack_act(h, M * hidden, &hdr->amax_h, hq, &hdr->sh, st, true, true);
  if (!rc)
    rc = launch_fp8_gemm(hq, w_down, M, K, hidden, hidden, hidden, &hdr->sh, s_down, b_down, y, K, QIK_DTYPE_BF16,
                         QIK_EPI_SCALE, nullptr, status, st, true);
  return rc;
}

extern "C" int qik_fp8_ffn(const void* x, int64_t M, int64_t K, int64_t hidden, const uint8_t* w_up,
                           const float* s_up, const void* b_up, const uint8_t* w_down, const float* s_down,
                           const void* b_down, void* y, void* ws, size_t ws_bytes, int* status, void* stream) {
  return fp8_ffn_chain(x, nullptr, nullptr, M, K, hidden, w_up, s_up, b_up, w_down, s_down, b_down, y, ws, ws_bytes,
                       status, stream);
}

extern "C" int qik_fp8_ffn_from_amax(const void* x, const uint32_t* x_amax_bits, int64_t M, int64_t K, int64_t hidden,
                                     const uint8_t* w_up, const float* s_up, const void* b_up, const uint8_t* w_down,
                                     const float* s_down, const void* b_down, void* y, void* ws, size_t ws_bytes,
                                     int* status, void* stream) {
  QIK_REQUIRE(x_amax_bits, "qik_fp8_ffn_from_amax: NULL amax");
  return fp8_ffn_chain(x, x_amax_bits, nullptr, M, K, hidden, w_up, s_up, b_up, w_down, s_down, b_down, y, ws,
                       ws_bytes, status, stream);
}

extern "C" int qik_fp8_ffn_e4m3(const uint8_t* xq, const float* x_scale, int64_t M, int64_t K, int64_t hidden,
                                const uint8_t* w_up, const float* s_up, const void* b_up, const uint8_t* w_down,
                                const float* s_down, const void* b_down, void* y, void* ws, size_t ws_bytes,
                                int* status, void* stream) {
  QIK_REQUIRE(x_scale, "qik_fp8_ffn_e4m3: NULL scale");
  QIK_REQUIRE(aligned16(xq), "qik_fp8_ffn_e4m3: xq must be 16-byte aligned");
  return fp8_ffn_chain(xq, nullptr, x_scale, M, K, hidden, w_up, s_up, b_up, w_down, s_down, b_down, y, ws, ws_bytes,
                       status, stream);
}
