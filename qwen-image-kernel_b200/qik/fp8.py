"""FP8 (W8A8, per-tensor e4m3) linear layers on the sm_100a tensor core.

Drop-in for ``qwen_image_kernel/fp8.py`` of gomezcojj-coder/qwen-image-kernel: the
same names, module buffers and return conventions, with the arithmetic done by the
hand-written CUDA kernels of libqik.so instead of Triton + torch._scaled_mm:

  compute_scale               fp8.py:24-26   -> qik_compute_scale
  quantize_tensorwise         fp8.py:44-53   -> qik_quantize_act (amax + e4m3 pack)
  quantize_weight_tensorwise  fp8.py:56-60   -> qik_quantize_weight
  FP8Linear.forward           fp8.py:78-90   -> qik_quantize_act + qik_fp8_gemm
  FP8Linear.from_linear       fp8.py:92-101
  convert_linears_fp8         fp8.py:104-120
  fp8_state_dict              fp8.py:123-127

Scales stay on the device (no host synchronization), as in the reference.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib as L

FP8_E4M3_MAX = 448.0


def _ws(device: torch.device) -> torch.Tensor:
    """Scratch for the calls that clear what they use on every call (compute_scale,
    quantize_weight_tensorwise)."""
    return torch.empty(L.load().qik_quant_workspace_bytes(), dtype=torch.uint8, device=device)


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return L.DTYPE_BF16
    if t.dtype == torch.float32:
        return L.DTYPE_F32
    raise TypeError(f"qik: unsupported dtype {t.dtype} (bf16 or fp32)")


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"qik: {name} must be a CUDA tensor (the kernels have no CPU path)")


def compute_scale(x: torch.Tensor) -> torch.Tensor:
    """Dynamic per-tensor fp8 activation scale (fp32 0-dim tensor, on the device):
    clamp_min(amax|x| / 448, 1e-12), evaluated as the reference does on CUDA."""
    _require_cuda(x, "x")
    lib = L.load()
    xc = x.contiguous()
    s = torch.empty((), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        L.check(lib.qik_compute_scale(xc.data_ptr(), _dtype_code(xc), xc.numel(), s.data_ptr(),
                                      _ws(x.device).data_ptr(), L.stream_ptr()), "qik_compute_scale")
    return s


def quantize_tensorwise(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[..., K] bf16 -> (e4m3 of the same shape, scale fp32 [1]).  One amax reduction
    and one scale+cast pass: q = e4m3_rn_satfinite(x * (1/s))."""
    _require_cuda(x, "x")
    if x.dtype != torch.bfloat16:
        raise TypeError("qik.quantize_tensorwise: bf16 activations only")
    lib = L.load()
    xc = x.contiguous()
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(1, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        stream = L.stream_ptr()
        L.check(lib.qik_quantize_act(xc.data_ptr(), xc.numel(), q.data_ptr(), s.data_ptr(),
                                     L.quant_state(x.device, stream).data_ptr(), stream), "qik_quantize_act")
    return q, s


def amax_bits(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """max|x| as the fp32 bit pattern in an int32 [1] tensor (accumulated into ``out``
    with atomicMax when given, so several tensors can share one amax).  Integer MAX of
    these bits across shards equals the bits of the global amax."""
    _require_cuda(x, "x")
    lib = L.load()
    xc = x.contiguous()
    if out is None:
        out = torch.zeros(1, dtype=torch.int32, device=x.device)
    with torch.cuda.device(x.device):
        L.check(lib.qik_amax(xc.data_ptr(), _dtype_code(xc), xc.numel(), out.data_ptr(), L.stream_ptr()), "qik_amax")
    return out


def quantize_from_amax(x: torch.Tensor, amax_bits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The pack half of quantize_tensorwise when a producer kernel already accumulated
    max|x| (fp32 bit pattern in ``amax_bits``, int32 [1])."""
    lib = L.load()
    xc = x.contiguous()
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(1, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        L.check(lib.qik_quantize_act_from_amax(xc.data_ptr(), xc.numel(), amax_bits.data_ptr(), q.data_ptr(),
                                               s.data_ptr(), L.stream_ptr()), "qik_quantize_act_from_amax")
    return q, s


def quantize_weight_tensorwise(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[N, K] -> (fp8 [N, K], scale fp32 [1]); q = e4m3(clamp(w / s, +-448)).

    Runs on the GPU.  A CPU weight is staged to the current CUDA device and the
    results are returned on the weight's device, as the reference's offline
    quantizer does (quantize_offline.py:19-26)."""
    src_dev = w.device
    wd = w if w.is_cuda else w.to(torch.device("cuda", torch.cuda.current_device()), non_blocking=True)
    lib = L.load()
    wc = wd.contiguous()
    q = torch.empty(w.shape, dtype=torch.float8_e4m3fn, device=wd.device)
    s = torch.empty(1, dtype=torch.float32, device=wd.device)
    with torch.cuda.device(wd.device):
        L.check(lib.qik_quantize_weight(wc.data_ptr(), _dtype_code(wc), wc.numel(), q.data_ptr(), s.data_ptr(),
                                        _ws(wd.device).data_ptr(), L.stream_ptr()), "qik_quantize_weight")
    if src_dev.type != "cuda":
        return q.to(src_dev), s.to(src_dev)
    return q, s


def fp8_gemm(xq: torch.Tensor, sx: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
             bias: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
             epilogue: int = L.EPI_SCALE, amax_out: torch.Tensor | None = None,
             out: torch.Tensor | None = None, tile_cfg: int = L.GEMM_TILE_AUTO) -> torch.Tensor:
    """y[M, N] = epilogue((xq . wq^T) * sx * sw (+ bias)) on the tensor core.

    xq [M, K] e4m3 (row pitch a multiple of 16 bytes), wq [N, K] e4m3, sx/sw fp32 [1]
    on the device, bias bf16 [N] or None.  out_dtype bf16, or fp32 for the pre-cast
    parity output.  ``amax_out`` (int32 [1], zeroed by the caller) receives the
    amax of the bf16 output for the next dynamic quantization.  ``tile_cfg`` forces a
    tile configuration (``qik._lib.GEMM_TILE_*``, for measurements and tests; the
    result is the same).  ``epilogue=EPI_SWIGLU`` takes wq as the fused gate / up
    weight (rows [0, N/2) gate, [N/2, N) up) and returns silu(gate) * up, [M, N/2]
    bf16, the bytes fused_swiglu gives on the two halves of the plain GEMM's output."""
    lib = L.load()
    if xq.dtype != torch.float8_e4m3fn or wq.dtype != torch.float8_e4m3fn:
        raise TypeError("qik.fp8_gemm: operands must be float8_e4m3fn")
    if xq.stride(-1) != 1:
        xq = xq.contiguous()
    if wq.stride(-1) != 1:
        wq = wq.contiguous()
    M, K = xq.shape
    N, K2 = wq.shape
    if K2 != K:
        raise ValueError(f"qik.fp8_gemm: K mismatch {K} vs {K2}")
    if out is None:
        out = torch.empty(M, N // 2 if epilogue == L.EPI_SWIGLU else N, dtype=out_dtype, device=xq.device)
    if bias is not None:
        bias = bias.to(torch.bfloat16).contiguous()
    status = L.status_word(xq.device)
    out_code = L.DTYPE_F32 if out.dtype == torch.float32 else L.DTYPE_BF16
    with torch.cuda.device(xq.device):
        if tile_cfg == L.GEMM_TILE_AUTO:
            L.check(lib.qik_fp8_gemm(xq.data_ptr(), wq.data_ptr(), M, N, K, xq.stride(0), wq.stride(0), sx.data_ptr(),
                                     sw.data_ptr(), L.ptr(bias), out.data_ptr(), out.stride(0), out_code, epilogue,
                                     L.ptr(amax_out), status.data_ptr(), L.stream_ptr()), "qik_fp8_gemm")
        else:
            L.check(lib.qik_fp8_gemm_tiled(xq.data_ptr(), wq.data_ptr(), M, N, K, xq.stride(0), wq.stride(0),
                                           sx.data_ptr(), sw.data_ptr(), L.ptr(bias), out.data_ptr(), out.stride(0),
                                           out_code, epilogue, L.ptr(amax_out), tile_cfg, status.data_ptr(),
                                           L.stream_ptr()), "qik_fp8_gemm_tiled")
    return out


class FP8Linear(nn.Module):
    """Drop-in replacement for nn.Linear with e4m3 weights (static per-tensor scale)
    and dynamic per-tensor activation quantization, computed by the qik tcgen05 GEMM.

    Buffers (state-dict compatible with the reference's e4m3 cache):
      weight        float8_e4m3fn [out_features, in_features]
      weight_scale  float32 [1]
      bias          bfloat16 [out_features] or None
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.register_buffer("weight", torch.zeros(out_features, in_features, dtype=torch.float8_e4m3fn))
        self.register_buffer("weight_scale", torch.ones(1, dtype=torch.float32))
        if bias:
            self.register_buffer("bias", torch.zeros(out_features, dtype=torch.bfloat16))
        else:
            self.bias = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.in_features < 256:
            # Same rule as the reference (fp8.py:79-84): skinny-K linears (img_in,
            # K=64) dequantize the weight and run a bf16 linear.
            w = self.weight.to(torch.bfloat16).float() * self.weight_scale
            out = torch.nn.functional.linear(x, w.to(x.dtype), self.bias)
            return out.to(x.dtype)
        x2 = x.reshape(-1, x.shape[-1])
        xq, s_a = quantize_tensorwise(x2)
        out = fp8_gemm(xq, s_a, self.weight, self.weight_scale, self.bias)
        out = out.reshape(*x.shape[:-1], self.out_features)
        return out.to(x.dtype) if out.dtype != x.dtype else out

    def forward_from_amax(self, x: torch.Tensor, amax: torch.Tensor | None) -> torch.Tensor:
        """forward(x) when the producer of x already reduced max|x| into ``amax``
        (int32 [1], fp32 bit pattern; e.g. the amax_out of the fused layer-norm /
        SwiGLU kernels): the quantizer skips its own amax pass.  Same bytes and
        scale as forward(x), since the amax is the same number."""
        if amax is None or self.in_features < 256:
            return self.forward(x)
        x2 = x.reshape(-1, x.shape[-1])
        xq, s_a = quantize_from_amax(x2, amax)
        out = fp8_gemm(xq, s_a, self.weight, self.weight_scale, self.bias)
        out = out.reshape(*x.shape[:-1], self.out_features)
        return out.to(x.dtype) if out.dtype != x.dtype else out

    def forward_e4m3(self, xq: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
        """forward(x) for an input already quantized as forward(x) would quantize it:
        ``xq`` e4m3 [..., in_features] with its dynamic scale ``scale`` (fp32 [1] on the
        device), e.g. from ``fused_layer_norm_modulate_e4m3``.  Returns bf16."""
        if xq.dtype != torch.float8_e4m3fn or xq.shape[-1] != self.in_features:
            raise ValueError(f"FP8Linear.forward_e4m3: expected float8_e4m3fn [..., {self.in_features}], "
                             f"got {xq.dtype} {tuple(xq.shape)}")
        if self.in_features < 256:
            raise ValueError("FP8Linear.forward_e4m3: linears with in_features < 256 take bf16 input (forward)")
        out = fp8_gemm(xq.reshape(-1, self.in_features), scale, self.weight, self.weight_scale, self.bias)
        return out.reshape(*xq.shape[:-1], self.out_features)

    def forward_swiglu_e4m3(self, xq: torch.Tensor, scale: torch.Tensor,
                            amax_out: torch.Tensor | None = None) -> torch.Tensor:
        """fused_swiglu(*forward_e4m3(xq, scale).chunk(2, -1)) for the fused gate / up
        linear of the MLP, in one GEMM whose epilogue applies the SwiGLU: returns bf16
        [..., out_features / 2].  ``amax_out`` (int32 [1], zeroed) receives the amax of
        the result, as fused_swiglu's does.  Needs out_features % 256 == 0."""
        if xq.dtype != torch.float8_e4m3fn or xq.shape[-1] != self.in_features:
            raise ValueError(f"FP8Linear.forward_swiglu_e4m3: expected float8_e4m3fn [..., {self.in_features}], "
                             f"got {xq.dtype} {tuple(xq.shape)}")
        if self.in_features < 256 or self.out_features % 256:
            raise ValueError("FP8Linear.forward_swiglu_e4m3: needs in_features >= 256 and out_features % 256 == 0")
        out = fp8_gemm(xq.reshape(-1, self.in_features), scale, self.weight, self.weight_scale, self.bias,
                       epilogue=L.EPI_SWIGLU, amax_out=amax_out)
        return out.reshape(*xq.shape[:-1], self.out_features // 2)

    def forward_qkv_rms_rope_e4m3(self, xq: torch.Tensor, scale: torch.Tensor, heads: int, w_q: torch.Tensor,
                                  w_k: torch.Tensor, freqs_cis: torch.Tensor | None, eps: float) -> torch.Tensor:
        """The fused QKV linear (weight rows q, k, v of ``heads`` x 128 each) on its e4m3
        input [B, S, in_features], with the per-head RMSNorm (fp32 weights ``w_q`` /
        ``w_k``) + RoPE of the q and k heads applied in the GEMM epilogue: returns bf16
        [B, S, 3 heads, 128] whose q / k heads equal fused_rms_norm_rope of
        forward_e4m3's output bit for bit and whose v heads equal that output."""
        from .triton_fused import _fp32_weight, rope_tables
        if xq.dtype != torch.float8_e4m3fn or xq.dim() != 3 or xq.shape[-1] != self.in_features:
            raise ValueError(f"FP8Linear.forward_qkv_rms_rope_e4m3: expected float8_e4m3fn [B, S, {self.in_features}]"
                             f", got {xq.dtype} {tuple(xq.shape)}")
        D = 128
        if self.out_features != 3 * heads * D or self.in_features < 256:
            raise ValueError(f"FP8Linear.forward_qkv_rms_rope_e4m3: out_features {self.out_features} is not "
                             f"3 x {heads} heads x {D}")
        B, S, K = xq.shape
        x2 = xq.reshape(B * S, K)
        if x2.stride(-1) != 1 or x2.stride(0) % 16:
            x2 = x2.contiguous()
        cos, sin = rope_tables(freqs_cis, S, D, xq.device)
        wq, wk = _fp32_weight(w_q, xq.device), _fp32_weight(w_k, xq.device)
        out = torch.empty(B * S, self.out_features, dtype=torch.bfloat16, device=xq.device)
        lib = L.load()
        bias = None if self.bias is None else self.bias.to(torch.bfloat16).contiguous()
        with torch.cuda.device(xq.device):
            L.check(lib.qik_fp8_gemm_qkv_rms_rope(x2.data_ptr(), self.weight.data_ptr(), B * S, K, x2.stride(0),
                                                  self.weight.stride(0), scale.data_ptr(), self.weight_scale.data_ptr(),
                                                  L.ptr(bias), out.data_ptr(), out.stride(0), heads, D, wq.data_ptr(),
                                                  wk.data_ptr(), cos.data_ptr(), sin.data_ptr(), S, float(eps),
                                                  L.status_word(xq.device).data_ptr(), L.stream_ptr()),
                    "qik_fp8_gemm_qkv_rms_rope")
        return out.view(B, S, 3 * heads, D)

    def forward_gate_residual(self, x: torch.Tensor, amax: torch.Tensor | None, residual: torch.Tensor,
                              table: torch.Tensor, target_token_mask: torch.Tensor | None) -> torch.Tensor:
        """fused_gate_residual(residual, forward_from_amax(x, amax), ...) in one GEMM whose
        epilogue applies the gated residual: x [B, S, in_features] bf16 (``amax`` its
        max|x| from the producer, or None), residual [B, S, out_features] bf16, ``table``
        the gate_table rows (B, or 2B with a target mask).  Same bytes as the two steps
        (up to products below 2^-126, rounded once here)."""
        from .triton_fused import _u8_mask
        B, S, K = x.shape
        if K != self.in_features or self.in_features < 256 or residual.shape != (B, S, self.out_features):
            raise ValueError(f"FP8Linear.forward_gate_residual: x {tuple(x.shape)} / residual "
                             f"{tuple(residual.shape)} do not fit [{self.in_features} -> {self.out_features}]")
        x2 = x.reshape(B * S, K)
        xq, s_a = quantize_tensorwise(x2) if amax is None else quantize_from_amax(x2, amax)
        res = residual.contiguous()
        # the table may be a column slice of a wider table (row pitch a multiple of 8)
        tab = table if (table.dim() == 2 and table.stride(-1) == 1 and table.stride(0) % 8 == 0
                        and table.stride(0) >= table.shape[1] and table.data_ptr() % 16 == 0) else table.contiguous()
        if tab.shape[0] < (2 * B if target_token_mask is not None else B) or tab.shape[1] != self.out_features:
            raise ValueError(f"FP8Linear.forward_gate_residual: gate table {tuple(tab.shape)} too small")
        mask = _u8_mask(target_token_mask, S, x.device)
        out = torch.empty(B, S, self.out_features, dtype=torch.bfloat16, device=x.device)
        bias = None if self.bias is None else self.bias.to(torch.bfloat16).contiguous()
        lib = L.load()
        with torch.cuda.device(x.device):
            L.check(lib.qik_fp8_gemm_gate_residual(xq.data_ptr(), self.weight.data_ptr(), B * S, self.out_features, K,
                                                   xq.stride(0), self.weight.stride(0), s_a.data_ptr(),
                                                   self.weight_scale.data_ptr(), L.ptr(bias), res.data_ptr(),
                                                   self.out_features, tab.data_ptr(), tab.stride(0), L.ptr(mask),
                                                   B, S, out.data_ptr(), self.out_features,
                                                   L.status_word(x.device).data_ptr(), L.stream_ptr()),
                    "qik_fp8_gemm_gate_residual")
        return out

    def forward_fp32(self, x: torch.Tensor) -> torch.Tensor:
        """Same computation with the fp32 GEMM output before the bf16 cast (parity mode)."""
        x2 = x.reshape(-1, x.shape[-1])
        xq, s_a = quantize_tensorwise(x2)
        out = fp8_gemm(xq, s_a, self.weight, self.weight_scale, self.bias, out_dtype=torch.float32)
        return out.reshape(*x.shape[:-1], self.out_features)

    @staticmethod
    def from_linear(linear: nn.Linear) -> "FP8Linear":
        """An FP8Linear holding ``linear``'s weight quantized per tensor (on the GPU, from
        its fp32 values, as fp8.py:92-101 does) and its bias in bf16, on the linear's
        device.  The shell is made on the meta device, so no zero buffers are allocated
        before the quantized tensors are assigned."""
        dev = linear.weight.device
        wq, scale = quantize_weight_tensorwise(linear.weight.detach().float())
        with torch.device("meta"):
            mod = FP8Linear(linear.in_features, linear.out_features, bias=linear.bias is not None)
        mod.weight = wq.to(dev)
        mod.weight_scale = scale.to(dev)
        if linear.bias is not None:
            mod.bias = linear.bias.detach().to(device=dev, dtype=torch.bfloat16).clone()
        return mod

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"


def convert_linears_fp8(module: nn.Module, skip_patterns: tuple[str, ...] = (), prefix: str = "") -> list[str]:
    """Swap every nn.Linear under ``module`` for ``FP8Linear.from_linear`` of it, in
    place (fp8.py:104-120).  A submodule whose qualified name (``prefix`` + the path)
    contains one of ``skip_patterns`` is left alone with everything below it.  Returns
    the qualified names converted, parents before children and siblings in
    registration order."""
    converted: list[str] = []
    pending = [(prefix, module)]
    while pending:
        path, mod = pending.pop()
        below = []
        for name, child in mod.named_children():
            full = f"{path}.{name}" if path else name
            if any(p in full for p in skip_patterns):
                continue
            if isinstance(child, nn.Linear):
                setattr(mod, name, FP8Linear.from_linear(child))
                converted.append(full)
            else:
                below.append((full, child))
        pending.extend(reversed(below))
    return converted


def fp8_state_dict(model: nn.Module) -> dict[str, torch.Tensor]:
    """State dict where converted linears expose fp8 ``weight`` + ``weight_scale``."""
    return {k: v for k, v in model.state_dict().items()}


def fp8_ffn_gelu(x: torch.Tensor, up: FP8Linear, down: FP8Linear, workspace: torch.Tensor | None = None,
                 out: torch.Tensor | None = None, x_amax: torch.Tensor | None = None,
                 x_scale: torch.Tensor | None = None) -> torch.Tensor:
    """DiT FFN pair: down(gelu_tanh(up(x))) with both linears FP8 per-tensor and the
    hidden activation re-quantized dynamically between them (qik_fp8_ffn: one chain
    of four kernels with programmatic dependent launches).

    The up-projection epilogue applies GELU-tanh to the bf16 linear output and
    accumulates max|h| on the fly, so the hidden tensor is quantized with one pack
    pass.  ``workspace`` (uint8, >= qik_fp8_ffn_workspace_bytes) may be passed to
    avoid an allocation per call, ``out`` (contiguous bf16, x's shape) to write the
    result into a buffer the caller owns, ``x_amax`` (int32 [1] on x's device: the
    fp32 bits of max|x|, as fused_layer_norm_modulate's ``amax_out`` accumulates them)
    to skip the chain's own max pass.  With ``x_scale`` (fp32 [1] on x's device), x is
    already the e4m3 input of the up projection quantized with that scale (as
    fused_layer_norm_modulate_e4m3 returns them) and the chain starts at its GEMM."""
    _require_cuda(x, "x")
    if x.dtype != (torch.float8_e4m3fn if x_scale is not None else torch.bfloat16):
        raise TypeError("qik.fp8_ffn_gelu: bf16 activations, or float8_e4m3fn ones with x_scale")
    lib = L.load()
    K = x.shape[-1]
    hidden = up.out_features
    if up.in_features != K or down.in_features != hidden or down.out_features != K:
        raise ValueError("qik.fp8_ffn_gelu: up must be K -> hidden and down hidden -> K")
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    nbytes = lib.qik_fp8_ffn_workspace_bytes(M, K, hidden)
    if workspace is None or workspace.numel() < nbytes or workspace.data_ptr() % 256:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    if out is None:
        y = torch.empty(M, K, dtype=torch.bfloat16, device=x.device)
    else:
        if (out.dtype != torch.bfloat16 or out.device != x.device or not out.is_contiguous()
                or out.numel() != M * K):
            raise ValueError("qik.fp8_ffn_gelu: out must be a contiguous bf16 tensor of x's shape on x's device")
        y = out.view(M, K)
    b_up = None if up.bias is None else up.bias.to(torch.bfloat16).contiguous()
    b_down = None if down.bias is None else down.bias.to(torch.bfloat16).contiguous()
    status = L.status_word(x.device)
    with torch.cuda.device(x.device):
        if x_scale is not None:
            if x_scale.dtype != torch.float32 or x_scale.device != x.device:
                raise ValueError("qik.fp8_ffn_gelu: x_scale must be an fp32 tensor on x's device")
            L.check(lib.qik_fp8_ffn_e4m3(x2.data_ptr(), x_scale.data_ptr(), M, K, hidden, up.weight.data_ptr(),
                                         up.weight_scale.data_ptr(), L.ptr(b_up), down.weight.data_ptr(),
                                         down.weight_scale.data_ptr(), L.ptr(b_down), y.data_ptr(),
                                         workspace.data_ptr(), workspace.numel(), status.data_ptr(),
                                         L.stream_ptr()), "qik_fp8_ffn_e4m3")
        elif x_amax is None:
            L.check(lib.qik_fp8_ffn(x2.data_ptr(), M, K, hidden, up.weight.data_ptr(), up.weight_scale.data_ptr(),
                                    L.ptr(b_up), down.weight.data_ptr(), down.weight_scale.data_ptr(), L.ptr(b_down),
                                    y.data_ptr(), workspace.data_ptr(), workspace.numel(), status.data_ptr(),
                                    L.stream_ptr()), "qik_fp8_ffn")
        else:
            if x_amax.dtype != torch.int32 or x_amax.device != x.device or x_amax.numel() < 1:
                raise ValueError("qik.fp8_ffn_gelu: x_amax must be an int32 tensor on x's device")
            L.check(lib.qik_fp8_ffn_from_amax(x2.data_ptr(), x_amax.data_ptr(), M, K, hidden, up.weight.data_ptr(),
                                              up.weight_scale.data_ptr(), L.ptr(b_up), down.weight.data_ptr(),
                                              down.weight_scale.data_ptr(), L.ptr(b_down), y.data_ptr(),
                                              workspace.data_ptr(), workspace.numel(), status.data_ptr(),
                                              L.stream_ptr()), "qik_fp8_ffn_from_amax")
    return y.reshape(*x.shape[:-1], K)
