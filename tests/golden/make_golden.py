"""Generate golden vectors by running the reference's own CPU-runnable functions.

Run once in a container where the reference checkout is present (it does not
travel to GPU boxes):

    python tests/golden/make_golden.py /path/to/qwen-image-kernel [section ...]

Sections: ``vectors`` (items 1-5 below, into the .npz files) and ``fp8_cache`` (item
6, into fp8_cache_ref.safetensors); the default is both.

The reference package cannot be imported as a whole (its ``__init__`` pulls in the
diffusers/accelerate runtime), so its leaf modules are loaded by file path under a
synthetic package.  Functions exercised (all run on CPU tensors):

  qwen_image_kernel/fp8.py:24-26          compute_scale
  qwen_image_kernel/fp8.py:56-60          quantize_weight_tensorwise
  qwen_image_kernel/kv_cache.py:23-95     ContiguousKVCache / _LayerView.store/get/views
  qwen_image_kernel/triton_attention.py:266-293  reference_block_causal_attention
  qwen_image_kernel/processors.py:22-36   _build_prefix_lengths
  qwen_image_kernel/quantize_offline.py:29-104  _fuse_block_linears, _convert_module_fp8,
                                          _sd_for_save (+ safetensors save_file): the e4m3
                                          cache of golden_inputs.standin_dit()

Inputs are drawn from numpy's PCG64 (stable across versions) so the tests can
regenerate them; only outputs (and input checksums) are stored.  CPU evaluation
means the per-tensor scales here use true division by 448 (the oracle's
SCALE_CPU form); the CUDA form is pinned on the GPU box by
tests/test_gpu_pins.py.
"""
from __future__ import annotations

import hashlib
import importlib.util
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import golden_inputs as GI  # noqa: E402


def load_reference(root: Path):
    pkg_dir = root / "qwen_image_kernel"
    pkg = types.ModuleType("qwen_image_kernel")
    pkg.__path__ = [str(pkg_dir)]
    sys.modules["qwen_image_kernel"] = pkg
    mods = {}
    for name in ("fp8", "triton_attention", "kv_cache", "triton_fused", "processors", "quantize_offline"):
        spec = importlib.util.spec_from_file_location(f"qwen_image_kernel.{name}", pkg_dir / f"{name}.py")
        m = importlib.util.module_from_spec(spec)
        sys.modules[f"qwen_image_kernel.{name}"] = m
        spec.loader.exec_module(m)
        mods[name] = m
    return mods


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()[:16]


def fp8_cache(R) -> None:
    """The reference's offline writer, exactly as build_transformer_fp8_cache drives it
    (quantize_offline.py:121-131), over the stand-in tree: fuse each block's groups,
    convert the remaining linears, drop ``.freqs``, save.  On a CPU-only machine the
    reference quantizes on the CPU (quantize_offline.py:16), i.e. with the true-division
    scale (the oracle's SCALE_CPU form)."""
    from safetensors.torch import save_file
    qo = R["quantize_offline"]
    model = GI.standin_dit()
    for blk in model.transformer_blocks:
        qo._fuse_block_linears(blk)
    qo._convert_module_fp8(model)
    save_file(qo._sd_for_save(model, drop_patterns=(".freqs",)), str(HERE / "fp8_cache_ref.safetensors"))


def main(ref_root: str, sections: list[str]) -> None:
    R = load_reference(Path(ref_root))
    torch.set_num_threads(8)
    if "fp8_cache" in sections:
        fp8_cache(R)
    if "vectors" in sections:
        vectors(R)
    print("golden files written to", HERE)


def vectors(R) -> None:
    fp8, attn, kvc, proc = R["fp8"], R["triton_attention"], R["kv_cache"], R["processors"]

    # ---- 1. compute_scale over every positive finite bf16 amax (CPU form) ----
    amax_bits = np.arange(1, 0x7F80, dtype=np.uint16)              # +min subnormal .. max finite
    amax_vals = torch.from_numpy(amax_bits.view(np.int16).copy()).view(torch.bfloat16)
    scales = np.empty(amax_bits.size, dtype=np.float32)
    for i in range(amax_bits.size):
        scales[i] = fp8.compute_scale(amax_vals[i:i + 1]).item()
    zero_scale = fp8.compute_scale(torch.zeros(4, dtype=torch.bfloat16)).item()
    np.savez_compressed(HERE / "compute_scale_cpu.npz", amax_bits=amax_bits, scale=scales,
                        zero_scale=np.float32(zero_scale))

    # ---- 2. quantize_weight_tensorwise ----
    wq_out = {}
    for name, w in GI.weight_cases().items():
        q, s = fp8.quantize_weight_tensorwise(w)
        wq_out[f"{name}__q"] = q.view(torch.uint8).numpy().copy()
        wq_out[f"{name}__s"] = s.numpy().astype(np.float32)
        wq_out[f"{name}__in"] = np.array(digest(w))
    np.savez_compressed(HERE / "weight_quant.npz", **wq_out)

    # ---- 3. ContiguousKVCache store / get / views ----
    kv_out = {}
    for name, (k, v, pmax, layers, layer) in GI.kv_cases().items():
        for v_fp8 in (False, True):
            c = kvc.ContiguousKVCache(layers, k.shape[0], pmax, k.shape[2], k.shape[3], v_fp8=v_fp8,
                                      device="cpu")
            c.k_buf.zero_()
            c.v_buf.view(torch.uint8).zero_() if v_fp8 else c.v_buf.zero_()
            c.v_scale.zero_()
            c.get_layer(layer).store(k, v)
            tag = f"{name}__fp8{int(v_fp8)}"
            kv_out[f"{tag}__k_buf"] = bits16(c.k_buf)
            kv_out[f"{tag}__v_buf"] = (c.v_buf.view(torch.uint8).numpy().copy() if v_fp8 else bits16(c.v_buf))
            kv_out[f"{tag}__v_scale"] = c.v_scale.numpy().copy()
            kv_out[f"{tag}__lengths"] = c.lengths.numpy().copy()
            gk, gv, sc = c.get_layer(layer).views()
            kv_out[f"{tag}__views_strides"] = np.array(list(gk.stride()) + list(gv.stride()), dtype=np.int64)
    np.savez_compressed(HERE / "kv_cache.npz", **kv_out)

    # ---- 4. _build_prefix_lengths ----
    pl_out = {}
    for name, (segments, S) in GI.prefix_cases().items():
        prefix_end = segments[-1][1] if segments else 0
        L = proc._build_prefix_lengths(segments, prefix_end, S, torch.device("cpu"))
        pl_out[name] = L.numpy().copy()
    np.savez_compressed(HERE / "prefix_lengths.npz", **pl_out)

    # ---- 5. reference_block_causal_attention ----
    at_out = {}
    for name, case in GI.attention_cases().items():
        q, k, v, L, kv_valid, ck, cv = (case[x] for x in ("q", "k", "v", "L", "key_valid", "cache_k", "cache_v"))
        if case.get("slab_fp8"):
            # fp8 slab: the reference stores V through ContiguousKVCache and the kernel
            # dequantizes bf16(fl32(v8) * vsc) (triton_attention.py:154-159); the fp32
            # reference then sees that dequantized V.
            B, P, H, D = ck.shape
            c = kvc.ContiguousKVCache(1, B, P, H, D, v_fp8=True, device="cpu")
            c.get_layer(0).store(ck, cv)
            ck8, cv8, vsc = c.get_layer(0).views()
            cv_deq = (cv8.float() * vsc[:, None, :, None]).to(torch.bfloat16)
            out = attn.reference_block_causal_attention(q, k, v, L, kv_valid, cache_k=ck8, cache_v=cv_deq)
            at_out[f"{name}__v8"] = cv8.contiguous().view(torch.uint8).numpy().copy()
            at_out[f"{name}__vsc"] = vsc.numpy().copy()
        else:
            out = attn.reference_block_causal_attention(q, k, v, L, kv_valid, cache_k=ck, cache_v=cv)
        at_out[f"{name}__out"] = bits16(out)
        at_out[f"{name}__in"] = np.array(digest(q) + digest(k) + digest(v))
    np.savez_compressed(HERE / "attention.npz", **at_out)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <reference checkout> [vectors] [fp8_cache]")
    main(sys.argv[1], sys.argv[2:] or ["vectors", "fp8_cache"])
