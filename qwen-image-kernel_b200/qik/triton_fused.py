"""Fused elementwise / normalization ops of the DiT block, same names and signatures
as ``qwen_image_kernel/triton_fused.py`` (gomezcojj-coder/qwen-image-kernel).

Each function launches one qik CUDA kernel (``csrc/qik_fused.cu``) with the
reference kernel's rounding points:

* ``fused_rms_norm_rope`` -- per-head RMSNorm (fp32 weight multiply, one bf16
  rounding) + complex RoPE (triton_fused.py:28-105).  Strided q / k views of the
  fused QKV output are read in place; the reference copies them to contiguous.
* ``fused_layer_norm_modulate`` -- LayerNorm (no affine) then ``* (1 + scale)`` with
  the per-position modulation row map (triton_fused.py:111-177).
* ``fused_gate_residual`` -- ``x + tanh(gate) * f`` (triton_fused.py:183-231).
* ``fused_swiglu`` -- ``silu(gate) * up`` (triton_fused.py:237-263); the two halves of
  the fused up-projection output are read in place.

``fused_layer_norm_modulate`` and ``fused_swiglu`` take an optional ``amax_out``
(int32 [1] on the device, zeroed by the caller): the kernel accumulates the fp32
bit pattern of max|out| into it, which is what the next FP8 linear's dynamic
quantizer reduces (``qik.fp8.quantize_from_amax``).  ``fused_layer_norm_modulate_e4m3``
goes one step further for a layer norm whose only consumers are FP8 linears: it
returns that linear's e4m3 input and scale directly (``FP8Linear.forward_e4m3``).
"""
from __future__ import annotations

import torch

from . import _lib as L
from .fp8 import _require_cuda

# Derived tables keyed on the source tensor's address and version; each entry keeps
# the source alive so that its address cannot be reused by another tensor while cached.
_cos_sin_cache: dict = {}
_weight_cache: dict = {}


def _require_bf16(**tensors: torch.Tensor) -> None:
    for name, t in tensors.items():
        _require_cuda(t, name)
        if t.dtype != torch.bfloat16:
            raise TypeError(f"qik: {name} must be bf16, got {t.dtype}")


def _u8_mask(target_token_mask: torch.Tensor | None, S: int, device: torch.device) -> torch.Tensor | None:
    if target_token_mask is None:
        return None
    m = target_token_mask.reshape(-1)
    if m.numel() != S:
        raise ValueError(f"target_token_mask has {m.numel()} entries for {S} positions")
    m = m.to(device=device, dtype=torch.uint8) if m.dtype != torch.bool or m.device != device else m.view(torch.uint8)
    return m.contiguous()


def _modulation_row_map(target_token_mask: torch.Tensor | None, B: int, S: int,
                        device: torch.device) -> torch.Tensor:
    """Per-position modulation row offset: 0 = own sample's timestep row, B = the
    t = 0 rows (triton_fused.py:141-151).  The kernels add the sample index."""
    if target_token_mask is not None:
        return torch.where(target_token_mask.to(torch.bool),
                           torch.zeros(S, dtype=torch.int32, device=device),
                           torch.full((S,), B, dtype=torch.int32, device=device))
    return torch.zeros(S, dtype=torch.int32, device=device)


def _fp32_weight(weight: torch.Tensor, device: torch.device) -> torch.Tensor:
    if weight.dtype == torch.float32 and weight.device == device and weight.is_contiguous():
        return weight
    key = (weight.data_ptr(), weight.dtype, weight._version, device)
    hit = _weight_cache.get(key)
    if hit is None:
        hit = (weight, weight.detach().to(device=device, dtype=torch.float32).contiguous())
        if len(_weight_cache) > 256:
            _weight_cache.clear()
        _weight_cache[key] = hit
    return hit[1]


def rope_tables(freqs_cis: torch.Tensor | None, S: int, D: int, device: torch.device) -> tuple:
    """fp32 cos / sin tables [S, D/2] of the complex rotary frequencies (the identity
    rotation for None), cached per frequency tensor."""
    key = (S, D, device, None if freqs_cis is None else (freqs_cis.data_ptr(), freqs_cis._version, freqs_cis.device))
    cached = _cos_sin_cache.get(key)
    if cached is not None:
        return cached[1], cached[2]
    if freqs_cis is None:  # no rotary embedding: the identity rotation
        cos = torch.ones(S, D // 2, dtype=torch.float32, device=device)
        sin = torch.zeros(S, D // 2, dtype=torch.float32, device=device)
    else:
        if tuple(freqs_cis.shape) != (S, D // 2):
            raise ValueError(f"freqs_cis has shape {tuple(freqs_cis.shape)}, expected ({S}, {D // 2})")
        cos = freqs_cis.real.float().to(device).contiguous()
        sin = freqs_cis.imag.float().to(device).contiguous()
    if len(_cos_sin_cache) > 8:
        _cos_sin_cache.clear()
    _cos_sin_cache[key] = (freqs_cis, cos, sin)
    return cos, sin


def fused_rms_norm_rope(x: torch.Tensor, weight: torch.Tensor, freqs_cis: torch.Tensor, eps: float) -> torch.Tensor:
    """x: [B, S, H, D] bf16 (any strides with a unit D stride); weight: [D];
    freqs_cis: complex [S, D/2] (None: no rotation).  Returns a contiguous
    [B, S, H, D] bf16 tensor."""
    _require_bf16(x=x)
    B, S, H, D = x.shape
    if x.stride(-1) != 1 or any(s % 8 for s in x.stride()[:3]) or x.data_ptr() % 16:
        x = x.contiguous()
    cos, sin = rope_tables(freqs_cis, S, D, x.device)
    w = _fp32_weight(weight, x.device)
    out = torch.empty((B, S, H, D), dtype=torch.bfloat16, device=x.device)
    lib = L.load()
    L.check(lib.qik_rms_norm_rope(x.data_ptr(), B, S, H, D, x.stride(0), x.stride(1), x.stride(2), w.data_ptr(),
                                  cos.data_ptr(), sin.data_ptr(), float(eps), out.data_ptr(), out.stride(0),
                                  out.stride(1), out.stride(2), L.stream_ptr(x.device)),
            "qik_rms_norm_rope")
    return out


def fused_layer_norm_modulate(x: torch.Tensor, modulation: torch.Tensor, scale_offset: int, modulation_stride: int,
                              target_token_mask: torch.Tensor | None, eps: float,
                              amax_out: torch.Tensor | None = None) -> torch.Tensor:
    """LayerNorm then (1 + scale).  ``modulation`` holds rows [0, B) of the samples'
    timesteps and, when a target mask is given, rows [B, 2B) of t = 0."""
    _require_bf16(x=x, modulation=modulation)
    B, S, D = x.shape
    x = x.contiguous()
    if modulation.stride(-1) != 1:
        raise ValueError("modulation must have a unit column stride")
    out = torch.empty_like(x)
    mask = _u8_mask(target_token_mask, S, x.device)
    lib = L.load()
    L.check(lib.qik_layer_norm_modulate(x.data_ptr(), B, S, D, modulation.data_ptr(), modulation.shape[0],
                                        int(modulation_stride),
                                        int(scale_offset), L.ptr(mask), float(eps), out.data_ptr(), L.ptr(amax_out),
                                        L.stream_ptr(x.device)),
            "qik_layer_norm_modulate")
    return out


def fused_layer_norm_modulate_e4m3(x: torch.Tensor, modulation: torch.Tensor, scale_offset: int,
                                   modulation_stride: int, target_token_mask: torch.Tensor | None,
                                   eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """fused_layer_norm_modulate followed by the next FP8 linear's dynamic quantizer,
    in one kernel: returns (e4m3 [B, S, D], scale fp32 [1]) -- the same codes and scale
    as ``quantize_tensorwise(fused_layer_norm_modulate(...))`` -- without writing the
    bf16 output (qik_layer_norm_modulate_e4m3)."""
    _require_bf16(x=x, modulation=modulation)
    B, S, D = x.shape
    x = x.contiguous()
    if modulation.stride(-1) != 1:
        raise ValueError("modulation must have a unit column stride")
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(1, dtype=torch.float32, device=x.device)
    mask = _u8_mask(target_token_mask, S, x.device)
    lib = L.load()
    with torch.cuda.device(x.device):
        stream = L.stream_ptr()
        L.check(lib.qik_layer_norm_modulate_e4m3(x.data_ptr(), B, S, D, modulation.data_ptr(), modulation.shape[0],
                                                 int(modulation_stride), int(scale_offset), L.ptr(mask), float(eps),
                                                 q.data_ptr(), s.data_ptr(), L.quant_state(x.device, stream).data_ptr(),
                                                 L.status_word(x.device).data_ptr(), stream),
                "qik_layer_norm_modulate_e4m3")
    return q, s


def fused_gate_residual(x: torch.Tensor, f: torch.Tensor, modulation: torch.Tensor, gate_offset: int,
                        target_token_mask: torch.Tensor | None) -> torch.Tensor:
    """x + tanh(gate) * f with the gate row chosen per position."""
    _require_bf16(x=x, f=f, modulation=modulation)
    B, S, D = x.shape
    x = x.contiguous()
    f = f.reshape(B, S, D).contiguous()
    if modulation.stride(-1) != 1:
        raise ValueError("modulation must have a unit column stride")
    out = torch.empty_like(x)
    mask = _u8_mask(target_token_mask, S, x.device)
    lib = L.load()
    L.check(lib.qik_gate_residual(x.data_ptr(), f.data_ptr(), B, S, D, modulation.data_ptr(), modulation.shape[0],
                                  modulation.stride(0),
                                  int(gate_offset), L.ptr(mask), out.data_ptr(), L.stream_ptr(x.device)),
            "qik_gate_residual")
    return out


def gate_table(modulation: torch.Tensor, gate_offset: int, rows: int, D: int) -> torch.Tensor:
    """bf16(tanh(modulation[r, gate_offset:gate_offset + D])) for r < rows, as
    fused_gate_residual computes the gate: the table of the FP8 linears' gated-residual
    epilogue (qik.fp8.FP8Linear.forward_gate_residual)."""
    _require_bf16(modulation=modulation)
    if modulation.stride(-1) != 1:
        raise ValueError("modulation must have a unit column stride")
    if rows > modulation.shape[0]:
        raise ValueError(f"gate_table: {rows} rows requested, modulation has {modulation.shape[0]}")
    out = torch.empty(rows, D, dtype=torch.bfloat16, device=modulation.device)
    lib = L.load()
    L.check(lib.qik_gate_table(modulation.data_ptr(), rows, modulation.stride(0), int(gate_offset), D, out.data_ptr(),
                               L.stream_ptr(modulation.device)), "qik_gate_table")
    return out


def _rows(t: torch.Tensor, M: int, N: int) -> tuple[torch.Tensor, int]:
    """t ([..., N]) as an [M, N] view with one row pitch (elements), copying only when
    the leading dims do not flatten or the pitch / base is not 16-byte aligned."""
    if t.stride(-1) == 1:
        try:
            v = t.view(M, N)
        except RuntimeError:
            v = None
        if v is not None:
            pitch = v.stride(0) if M > 1 else N
            if pitch % 8 == 0 and pitch >= N and v.data_ptr() % 16 == 0:
                return v, pitch
    return t.contiguous().view(M, N), N


def fused_swiglu(gate: torch.Tensor, up: torch.Tensor, amax_out: torch.Tensor | None = None) -> torch.Tensor:
    """gate, up: [..., N] bf16 (e.g. the halves of the fused up-projection output)
    -> silu(gate) * up, contiguous."""
    _require_bf16(gate=gate, up=up)
    if gate.shape != up.shape:
        raise ValueError("gate and up must have the same shape")
    N = gate.shape[-1]
    out = torch.empty(gate.shape, dtype=torch.bfloat16, device=gate.device)
    if out.numel() == 0:
        return out
    M = out.numel() // N
    g, ldg = _rows(gate, M, N)
    p, ldp = _rows(up, M, N)
    lib = L.load()
    L.check(lib.qik_swiglu(g.data_ptr(), ldg, p.data_ptr(), ldp, M, N, out.data_ptr(), N, L.ptr(amax_out),
                           L.stream_ptr(gate.device)),
            "qik_swiglu")
    return out
