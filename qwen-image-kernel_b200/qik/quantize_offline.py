"""The e4m3 weight cache: writer and reader, driven by one table of fused groups.

Format (the reference's, gomezcojj-coder/qwen-image-kernel
``qwen_image_kernel/quantize_offline.py:29-134`` writes it and ``runtime.py:76-123,
176-201`` reads it), one safetensors file:

* every linear at module path ``p`` becomes ``p.weight`` (F8_E4M3 [N, K]),
  ``p.weight_scale`` (F32 [1], one per-tensor scale) and, when it has one, ``p.bias``
  (BF16 [N]);
* per transformer block, the linears of a fused group (``FUSED_GROUPS``) are stored as
  ONE linear under ``<block>.<owner>.<fused>``: the members' weights concatenated along
  the output dimension and quantized once (a single scale over the concatenation), the
  biases concatenated likewise; the members themselves have no keys;
* every other parameter and persistent buffer keeps its name and dtype, except names
  containing a dropped pattern (``.freqs``, rebuilt at model init);
* each stored tensor owns its storage (views and shared storages are copied out).

safetensors orders tensors by dtype and name, so the same set of (name, tensor) pairs
gives the same bytes whatever the traversal order: a cache written here is
byte-identical to the reference writer's for the same model and quantizer (tested
against a file the reference wrote).

The writer converts the model in place (``fuse_groups`` then ``quantize_linears``)
and saves its state dict, like the reference pipeline; the reader
(``install_fp8_shells`` / ``load_fp8_cache``) rebuilds the module tree a cache
describes from its key set, with shells created on the meta device and filled by
``load_state_dict(assign=True)``.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Callable, Iterable, Iterator, Mapping

import torch

from .fp8 import FP8Linear, quantize_weight_tensorwise

Quantizer = Callable[[torch.Tensor], "tuple[torch.Tensor, torch.Tensor]"]

DROPPED_PATTERNS: tuple[str, ...] = (".freqs",)


@dataclass(frozen=True)
class FusedGroup:
    """Linears ``<owner>.<member>`` of one block stored as ``<owner>.<fused>``, their
    outputs stacked in ``members`` order (quantize_offline.py:67-104; the processor
    splits the fused QKV output into q, k, v and the fused up output into gate, up)."""
    owner: str
    fused: str
    members: tuple[str, ...]


FUSED_GROUPS: tuple[FusedGroup, ...] = (
    FusedGroup("attn", "fused_qkv", ("to_q", "to_k", "to_v")),
    FusedGroup("img_mlp", "fused_up", ("gate_layer", "proj")),
)


def _qualified(prefix: str, name: str) -> str:
    return f"{prefix}.{name}" if prefix else name


def _linear_sites(model: torch.nn.Module, skip: Iterable[str] = ()) -> Iterator[tuple[torch.nn.Module, str, str]]:
    """(parent, attribute, qualified name) of every nn.Linear in the tree, in module
    order, skipping qualified names that contain a pattern of ``skip``.  The list is
    taken before any replacement, so the caller may swap modules while iterating."""
    skip = tuple(skip)
    sites = []
    for pname, parent in model.named_modules():
        for attr, child in parent.named_children():
            full = _qualified(pname, attr)
            if isinstance(child, torch.nn.Linear) and not any(p in full for p in skip):
                sites.append((parent, attr, full))
    return iter(sites)


def _quantized_linear(weight: torch.Tensor, bias: torch.Tensor | None, quantize: Quantizer | None) -> FP8Linear:
    """An FP8Linear holding quantize(weight) and the bias in bf16, on the weight's device."""
    n, k = weight.shape
    wq, scale = (quantize or quantize_weight_tensorwise)(weight)
    with torch.device("meta"):
        lin = FP8Linear(k, n, bias=bias is not None)
    lin.weight = wq.to(weight.device)
    lin.weight_scale = scale.reshape(1).to(weight.device)
    if bias is not None:
        lin.bias = bias.detach().to(torch.bfloat16).clone()
    return lin


def fuse_groups(block: torch.nn.Module, quantize: Quantizer | None = None,
                groups: tuple[FusedGroup, ...] = FUSED_GROUPS) -> list[str]:
    """Replace each group's member linears of ``block`` by one FP8Linear quantized from
    their concatenated bf16 weights (one scale), and the members by Identity.  Returns
    the fused attribute paths.  The members must agree on in_features, out_features
    and on having a bias (the same checks as quantize_offline.py:75-77,92-93)."""
    done = []
    for g in groups:
        owner = getattr(block, g.owner)
        members = [getattr(owner, m) for m in g.members]
        shapes = {(m.in_features, m.out_features, m.bias is not None) for m in members}
        assert len(shapes) == 1, f"{g.owner}: members {g.members} differ in shape or bias: {sorted(shapes)}"
        w = torch.cat([m.weight.detach() for m in members], dim=0)
        b = torch.cat([m.bias.detach() for m in members], dim=0) if members[0].bias is not None else None
        setattr(owner, g.fused, _quantized_linear(w, b, quantize))
        for m in g.members:
            setattr(owner, m, torch.nn.Identity())
        done.append(f"{g.owner}.{g.fused}")
    return done


def quantize_linears(model: torch.nn.Module, skip: Iterable[str] = (), quantize: Quantizer | None = None) -> list[str]:
    """Replace every nn.Linear of the tree by an FP8Linear of its quantized weight
    (quantize_offline.py:29-48); FP8Linear is not an nn.Linear, so fused linears are
    left as they are.  Returns the converted qualified names."""
    names = []
    for parent, attr, full in _linear_sites(model, skip):
        lin = getattr(parent, attr)
        setattr(parent, attr, _quantized_linear(lin.weight.detach(), lin.bias, quantize))
        names.append(full)
    return names


def cache_state_dict(model: torch.nn.Module, drop: Iterable[str] = DROPPED_PATTERNS) -> dict[str, torch.Tensor]:
    """The model's state dict as the cache stores it: names containing a ``drop``
    pattern removed, and every tensor that does not solely own a whole storage
    (a view, or one of several names on one storage) copied out, because
    safetensors refuses shared storage (quantize_offline.py:51-64)."""
    drop = tuple(drop)
    items = [(k, t) for k, t in model.state_dict().items() if not any(p in k for p in drop)]
    users: dict[int, int] = {}
    for _, t in items:
        key = t.untyped_storage().data_ptr()
        users[key] = users.get(key, 0) + 1
    out = {}
    for k, t in items:
        st = t.untyped_storage()
        whole = t.storage_offset() == 0 and t.nbytes == st.nbytes() and t.is_contiguous()
        out[k] = t if (whole and users[st.data_ptr()] == 1) else t.contiguous().clone()
    return out


def write_fp8_cache(model: torch.nn.Module, out_path: str, drop: Iterable[str] = DROPPED_PATTERNS) -> int:
    """Save an already converted model in the cache format; returns the tensor count."""
    from safetensors.torch import save_file
    os.makedirs(os.path.dirname(out_path) or ".", exist_ok=True)
    sd = cache_state_dict(model, drop)
    save_file(sd, out_path)
    return len(sd)


def convert_model_fp8(model: torch.nn.Module, blocks: Iterable[torch.nn.Module] | None = None,
                      quantize: Quantizer | None = None, skip: Iterable[str] = ()) -> list[str]:
    """Fuse the groups of every block in ``blocks`` (default: ``model.transformer_blocks``
    when the model has them), then quantize every remaining linear.  Returns the
    qualified names of the non-fused linears converted."""
    if blocks is None:
        blocks = getattr(model, "transformer_blocks", ())
    for blk in blocks:
        fuse_groups(blk, quantize)
    return quantize_linears(model, skip, quantize)


# ---------------------------------------------------------------------------
# reader
# ---------------------------------------------------------------------------
def install_fp8_shells(model: torch.nn.Module, keys: Iterable[str], skip: Iterable[str] = ()) -> list[str]:
    """Make the module tree match a cache's key set before loading it
    (runtime.py:76-123): wherever the keys hold ``<p>.<owner>.<fused>.weight`` for a
    module ``p`` whose ``<owner>`` has the group's member linears, an FP8Linear shell of
    the concatenated shape goes in as ``<owner>.<fused>`` and the members become
    Identity; then every remaining nn.Linear becomes an FP8Linear shell.  A shell has
    a bias exactly when the keys hold ``<its path>.bias``.  Shells live on the meta
    device and take their tensors from ``load_state_dict(assign=True)``.  Returns the
    qualified names of the shells."""
    keys = frozenset(keys)
    shells = []
    for pname, mod in list(model.named_modules()):
        for g in FUSED_GROUPS:
            owner = getattr(mod, g.owner, None)
            if owner is None:
                continue
            path = _qualified(pname, f"{g.owner}.{g.fused}")
            if f"{path}.weight" not in keys:
                continue
            members = [getattr(owner, m, None) for m in g.members]
            if not all(isinstance(m, torch.nn.Linear) for m in members):
                continue
            with torch.device("meta"):
                shell = FP8Linear(members[0].in_features, sum(m.out_features for m in members),
                                  bias=f"{path}.bias" in keys)
            setattr(owner, g.fused, shell)
            for m in g.members:
                setattr(owner, m, torch.nn.Identity())
            shells.append(path)
    for parent, attr, full in _linear_sites(model, skip):
        lin = getattr(parent, attr)
        with torch.device("meta"):
            shell = FP8Linear(lin.in_features, lin.out_features, bias=f"{full}.bias" in keys)
        setattr(parent, attr, shell)
        shells.append(full)
    return shells


def load_fp8_cache(model: torch.nn.Module, cache: str | Mapping[str, torch.Tensor],
                   dropped: Iterable[str] = DROPPED_PATTERNS) -> torch.nn.Module:
    """Load a cache (a path or an already loaded state dict) into ``model``, typically
    built with its parameters on the meta device: shells are installed from the key
    set, the tensors assigned, and the result checked as runtime.py:196-200 does: no
    unexpected key, no missing key (names with a dropped pattern excepted: the writer
    leaves them out and the model rebuilds them) and no parameter or persistent
    buffer left on the meta device.  Raises ValueError otherwise."""
    if isinstance(cache, (str, os.PathLike)):
        from safetensors.torch import load_file
        sd = load_file(str(cache))
    else:
        sd = dict(cache)
    install_fp8_shells(model, sd.keys())
    missing, unexpected = model.load_state_dict(sd, strict=False, assign=True)
    dropped = tuple(dropped)
    missing = [k for k in missing if not any(p in k for p in dropped)]
    if unexpected:
        raise ValueError(f"fp8 cache: unexpected keys {unexpected[:4]}")
    if missing:
        raise ValueError(f"fp8 cache: missing keys {missing[:8]}")
    meta_left = [k for k, t in model.state_dict().items() if t.is_meta and not any(p in k for p in dropped)]
    if meta_left:
        raise ValueError(f"fp8 cache: tensors left on the meta device {meta_left[:8]}")
    return model


# ---------------------------------------------------------------------------
# whole-model builders (need diffusers / transformers and the bf16 checkpoint)
# ---------------------------------------------------------------------------
def build_transformer_fp8_cache(model_id: str, out_path: str, fused_linears: bool = True) -> None:
    """Quantize the DiT's linears from the bf16 checkpoint into the cache file
    (quantize_offline.py:107-134).  The reference first wraps every block in its
    kernel-block shell, whose submodule names are the block's own, so fusing the
    blocks in place writes the same keys."""
    from diffusers.models.transformers.transformer_qwenimage21 import QwenImage21Transformer2DModel
    model = QwenImage21Transformer2DModel.from_pretrained(model_id, subfolder="transformer",
                                                          torch_dtype=torch.bfloat16)
    convert_model_fp8(model, model.transformer_blocks if fused_linears else ())
    n = write_fp8_cache(model, out_path)
    print(f"[fp8-cache] wrote {out_path} ({n} tensors)", flush=True)


def build_text_encoder_fp8_cache(model_id: str, out_path: str) -> None:
    """The Qwen3-VL text encoder's linears, no fused groups and nothing dropped
    (quantize_offline.py:137-150)."""
    from transformers import Qwen3VLForConditionalGeneration
    te = Qwen3VLForConditionalGeneration.from_pretrained(model_id, subfolder="text_encoder",
                                                         torch_dtype=torch.bfloat16)
    quantize_linears(te)
    n = write_fp8_cache(te, out_path, drop=())
    print(f"[fp8-cache] wrote {out_path} ({n} tensors)", flush=True)
