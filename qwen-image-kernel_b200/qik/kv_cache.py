"""Contiguous preallocated prefix KV slab with optional e4m3 V (per-head scales).

Drop-in for ``qwen_image_kernel/kv_cache.py`` of gomezcojj-coder/qwen-image-kernel:
the same single allocation and layouts (kv_cache.py:63-93) --
K ``[L, B, H, Pmax, D]`` bf16, V the same shape in bf16 or e4m3, ``v_scale``
``[L, B, H]`` fp32, ``lengths [L]`` -- and the same ``store`` / ``get`` / ``views``
contract (kv_cache.py:23-60).  ``store`` runs the qik_kv_store kernel: K is copied
into the per-head-contiguous layout and V is either copied or quantized per
(b, h) with s = clamp_min(amax / 448, 1e-12), v8 = e4m3(clamp(v / s, +-448)).
"""
from __future__ import annotations

import torch

from . import _lib as L

FP8_E4M3_MAX = 448.0


class _LayerView:
    """Per-layer store/get interface compatible with the stock cache."""

    def __init__(self, cache: "ContiguousKVCache", layer: int):
        self._c = cache
        self._layer = layer

    def store(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """k, v: [B, P, H, D] (post-RoPE).  Backing layout [B, H, P, D] so each head's
        token sequence is dense for the attention kernel's tile reads."""
        c = self._c
        B, P, H, D = k.shape
        assert v.shape == k.shape, "k and v must have the same shape"
        assert k.dtype == c.k_buf.dtype and (c.v_fp8 or v.dtype == c.v_buf.dtype)
        if c.v_fp8 and v.dtype != torch.bfloat16:
            raise NotImplementedError("qik fp8-V slab: bf16 values only")
        if P > c.capacity:
            raise ValueError(f"prefix of {P} tokens exceeds the slab capacity {c.capacity}")
        k = k if k.stride(-1) == 1 else k.contiguous()
        v = v if v.stride(-1) == 1 else v.contiguous()
        lib = L.load()
        ws = torch.empty(max(1, B * H), dtype=torch.int32, device=k.device) if c.v_fp8 else None
        kb = c.k_buf[self._layer]
        vb = c.v_buf[self._layer]
        with torch.cuda.device(k.device):
            L.check(lib.qik_kv_store(k.data_ptr(), v.data_ptr(), B, P, H, D, k.stride(0), k.stride(1), k.stride(2),
                                     v.stride(0), v.stride(1), v.stride(2), kb.data_ptr(), vb.data_ptr(),
                                     c.capacity, int(c.v_fp8), c.v_scale[self._layer].data_ptr() if c.v_fp8 else None,
                                     ws.data_ptr() if ws is not None else None, L.stream_ptr()), "qik_kv_store")
        c.lengths[self._layer] = P

    def get(self):
        """Returns (k, v) as [B, P, H, D] views (strided; the kernel is stride-agnostic)."""
        P = int(self._c.lengths[self._layer])
        k = self._c.k_buf[self._layer, :, :, :P, :].transpose(1, 2)
        v = self._c.v_buf[self._layer, :, :, :P, :].transpose(1, 2)
        return k, v

    def views(self):
        """(k, v, v_scale_or_None) for the kernel wrapper."""
        P = int(self._c.lengths[self._layer])
        k = self._c.k_buf[self._layer, :, :, :P, :].transpose(1, 2)
        v = self._c.v_buf[self._layer, :, :, :P, :].transpose(1, 2)
        scale = self._c.v_scale[self._layer] if self._c.v_fp8 else None
        return k, v, scale


class ContiguousKVCache:
    """Single-slab prefix KV cache: one allocation for all layers.

    K layout: [L, B, H, P_max, D] bf16.  V layout: same (bf16) or fp8e4m3 with
    per-head fp32 scales [L, B, H].  Per prefix token across 32 layers at H=32,
    D=128: K+V bf16 = 512 KB, K bf16 + V fp8 = 384 KB.
    """

    def __init__(self, num_layers: int, batch: int, prefix_max: int, num_heads: int, head_dim: int,
                 v_fp8: bool = False, device: torch.device | str = "cuda", dtype: torch.dtype = torch.bfloat16):
        self.v_fp8 = v_fp8
        self.num_layers = num_layers
        self.capacity = prefix_max
        self.batch_size = batch
        self.k_buf = torch.empty(num_layers, batch, num_heads, prefix_max, head_dim, dtype=dtype, device=device)
        v_dtype = torch.float8_e4m3fn if v_fp8 else dtype
        self.v_buf = torch.empty(num_layers, batch, num_heads, prefix_max, head_dim, dtype=v_dtype, device=device)
        self.v_scale = torch.empty(num_layers, batch, num_heads, dtype=torch.float32, device=device)
        self.lengths = torch.zeros(num_layers, dtype=torch.int64, device=device)
        self.layers = [_LayerView(self, i) for i in range(num_layers)]

    def get_layer(self, i: int) -> _LayerView:
        return self.layers[i]
