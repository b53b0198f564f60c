"""Offline e4m3 weight-cache builder, same format as the reference's.

Mirrors ``qwen_image_kernel/quantize_offline.py`` (gomezcojj-coder/qwen-image-kernel):
a mixed fp8/bf16 safetensors file whose converted linears expose
``<path>.weight`` (F8_E4M3 [N, K]), ``<path>.weight_scale`` (F32 [1]) and
``<path>.bias`` (BF16 [N]); Q/K/V and the MLP gate/proj are fused into
``attn.fused_qkv`` / ``img_mlp.fused_up`` with one scale over the concatenated weight
(quantize_offline.py:67-104); storages are de-aliased and ``.freqs`` buffers dropped
(quantize_offline.py:51-64, 130).  The quantization runs on the GPU kernels
(qik_quantize_weight); a cache written here loads into the reference's FP8Linear
shells and vice versa.
"""
from __future__ import annotations

import os
from typing import Callable

import torch

from .fp8 import FP8Linear, quantize_weight_tensorwise

Quantizer = Callable[[torch.Tensor], "tuple[torch.Tensor, torch.Tensor]"]


def _staged_quantize(w: torch.Tensor, quantize: Quantizer | None = None):
    """Quantize one weight; a CPU weight is staged through the GPU and the results come
    back to the CPU (quantize_offline.py:19-26)."""
    return (quantize or quantize_weight_tensorwise)(w)


def _convert_module_fp8(module: torch.nn.Module, skip: tuple[str, ...] = (),
                        quantize: Quantizer | None = None) -> list[str]:
    """Replace every nn.Linear in the tree by an FP8Linear (quantize_offline.py:29-48)."""
    converted = []
    for parent_name, parent_mod in list(module.named_modules()):
        for child_name, child in list(parent_mod.named_children()):
            full = f"{parent_name}.{child_name}" if parent_name else child_name
            if any(p in full for p in skip):
                continue
            if isinstance(child, torch.nn.Linear):
                in_f, out_f, has_b = child.in_features, child.out_features, child.bias is not None
                wq, s = _staged_quantize(child.weight.data, quantize)
                new = FP8Linear(in_f, out_f, bias=has_b)
                new.weight = wq
                new.weight_scale = s
                if has_b:
                    new.bias = child.bias.data.to(torch.bfloat16).clone()
                setattr(parent_mod, child_name, new)
                converted.append(full)
    return converted


def _sd_for_save(model: torch.nn.Module, drop_patterns: tuple[str, ...] = ()) -> dict[str, torch.Tensor]:
    """State dict safe for safetensors.save_file: shared storages split, views cloned,
    names matching ``drop_patterns`` dropped (quantize_offline.py:51-64)."""
    sd: dict[str, torch.Tensor] = {}
    seen: set[int] = set()
    for name, t in model.state_dict().items():
        if any(p in name for p in drop_patterns):
            continue
        ptr = t.untyped_storage().data_ptr()
        if t._base is not None or ptr in seen:
            t = t.clone()
            ptr = t.untyped_storage().data_ptr()
        seen.add(ptr)
        sd[name] = t.contiguous()
    return sd


def _fuse_block_linears(block, quantize: Quantizer | None = None) -> None:
    """Replace a block's attn.to_q/to_k/to_v and img_mlp.gate_layer/proj by single fused
    FP8 linears quantized once from the concatenated bf16 weights, and drop the
    originals (quantize_offline.py:67-104)."""
    attn, mlp = block.attn, block.img_mlp
    q, k, v = attn.to_q, attn.to_k, attn.to_v
    assert q.in_features == k.in_features == v.in_features
    assert q.out_features == k.out_features == v.out_features
    assert (q.bias is not None) == (k.bias is not None) == (v.bias is not None)
    inner = q.out_features
    fused_qkv = FP8Linear(q.in_features, 3 * inner, bias=q.bias is not None)
    w = torch.cat([q.weight.data, k.weight.data, v.weight.data], 0)
    wq, s = _staged_quantize(w, quantize)
    fused_qkv.weight = wq
    fused_qkv.weight_scale = s
    if q.bias is not None:
        fused_qkv.bias = torch.cat([q.bias.data, k.bias.data, v.bias.data], 0).to(torch.bfloat16)
    attn.fused_qkv = fused_qkv.to(w.device)
    attn.to_q = torch.nn.Identity()
    attn.to_k = torch.nn.Identity()
    attn.to_v = torch.nn.Identity()

    gate, proj = mlp.gate_layer, mlp.proj
    assert gate.in_features == proj.in_features and gate.out_features == proj.out_features
    assert (gate.bias is not None) == (proj.bias is not None)
    hidden = gate.out_features
    fused_up = FP8Linear(gate.in_features, 2 * hidden, bias=gate.bias is not None)
    w = torch.cat([gate.weight.data, proj.weight.data], 0)
    wq, s = _staged_quantize(w, quantize)
    fused_up.weight = wq
    fused_up.weight_scale = s
    if gate.bias is not None:
        fused_up.bias = torch.cat([gate.bias.data, proj.bias.data], 0).to(torch.bfloat16)
    mlp.fused_up = fused_up.to(w.device)
    mlp.gate_layer = torch.nn.Identity()
    mlp.proj = torch.nn.Identity()


def save_fp8_cache(model: torch.nn.Module, out_path: str, drop_patterns: tuple[str, ...] = (".freqs",)) -> int:
    """Write the model's (already converted) state dict in the cache format; returns the
    number of tensors written."""
    from safetensors.torch import save_file
    os.makedirs(os.path.dirname(out_path) or ".", exist_ok=True)
    sd = _sd_for_save(model, drop_patterns)
    save_file(sd, out_path)
    return len(sd)


def build_transformer_fp8_cache(model_id: str, out_path: str, fused_linears: bool = True) -> None:
    """Quantize the DiT's linears from the bf16 checkpoint into the cache file
    (quantize_offline.py:107-134).  Needs diffusers and the checkpoint.  The blocks are
    fused in place: the reference first wraps each block in a shell whose submodule
    names are the block's own, so the written keys are the same."""
    from diffusers.models.transformers.transformer_qwenimage21 import QwenImage21Transformer2DModel
    print(f"[fp8-cache] loading BF16 transformer from {model_id} ...", flush=True)
    model = QwenImage21Transformer2DModel.from_pretrained(model_id, subfolder="transformer",
                                                          torch_dtype=torch.bfloat16)
    if fused_linears:
        print("[fp8-cache] fusing qkv / mlp-up linears (single-rounding) ...", flush=True)
        for blk in model.transformer_blocks:
            _fuse_block_linears(blk)
    print("[fp8-cache] quantizing block linears to fp8 ...", flush=True)
    _convert_module_fp8(model)
    n = save_fp8_cache(model, out_path)
    print(f"[fp8-cache] wrote {out_path} ({n} tensors)", flush=True)


def build_text_encoder_fp8_cache(model_id: str, out_path: str) -> None:
    """Same for the Qwen3-VL text encoder (quantize_offline.py:137-150)."""
    from transformers import Qwen3VLForConditionalGeneration
    te = Qwen3VLForConditionalGeneration.from_pretrained(model_id, subfolder="text_encoder",
                                                         torch_dtype=torch.bfloat16)
    _convert_module_fp8(te)
    n = save_fp8_cache(te, out_path, drop_patterns=())
    print(f"[fp8-cache] wrote {out_path} ({n} tensors)", flush=True)
