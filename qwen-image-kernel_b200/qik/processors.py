"""Attention processor and fused transformer block of Qwen-Image 2.1 on the qik kernels.

Same names and call signatures as ``qwen_image_kernel/processors.py``
(gomezcojj-coder/qwen-image-kernel):

* ``_build_prefix_lengths`` (processors.py:22-36): the block-causal mask of a joint
  [prefix ; target] sequence collapses to one inclusive key limit per query row --
  text rows are causal (L = q), image-block rows see the whole prefix up to the end
  of their block (L = end - 1), target rows see everything (L = S - 1).  The
  per-row "causal length" of the block-causal attention is the exclusive count L + 1.
* ``QwenImage21KernelProcessor`` (processors.py:39-126): fused QKV FP8 GEMM, per-head
  RMSNorm + RoPE, prefill (block-causal over the joint sequence) or decode (target
  rows over [cached prefix ; fresh target] without concatenation), output FP8 GEMM.
* ``QwenImage21KernelBlock`` (processors.py:129-187): LayerNorm + modulation, gated
  residuals and the SwiGLU MLP around the attention, same submodule names so state
  dicts load unchanged.
* ``convert_transformer_to_kernels`` (processors.py:190-211).

Where the data layout allows, tensors stay in place instead of being copied: q / k /
v are strided views of the fused QKV output, gate / up the two halves of the fused
up projection, and the slab store reads the key / value views directly.  A layer norm
whose only consumers are FP8 linears emits their e4m3 input and scale itself
(``fused_layer_norm_modulate_e4m3``: the bf16 output is never written); the fused QKV
linear then applies the q / k RMSNorm + RoPE in its GEMM epilogue (``_qkv_rms_rope``)
and the fused up projection the SwiGLU (``_swiglu_linear``: the gate / up output is
never written); the out-projection and the down projection add their gated output
to the residual in their GEMM epilogues (``_gate_linear``, with the bf16(tanh(gate))
rows from ``gate_table``).  SwiGLU and the attention reduce the amax
of their output, which the next FP8 linear uses instead of its own amax pass (same
bytes and scale).
"""
from __future__ import annotations

import torch

from .fp8 import FP8Linear
from .triton_attention import block_causal_flash_attention
from .triton_fused import (fused_gate_residual, fused_layer_norm_modulate, fused_layer_norm_modulate_e4m3,
                           fused_rms_norm_rope, fused_swiglu, gate_table)


def _build_prefix_lengths(segments: list[tuple[int, int, bool]], prefix_len: int, seq_len: int,
                          device: torch.device) -> torch.Tensor:
    """Per-row inclusive kv limit L: row q attends iff kv <= L[q]."""
    L = torch.arange(seq_len, dtype=torch.int32, device=device)
    for start, end, is_text in segments:
        if not is_text:
            L[start:end] = end - 1
    L[prefix_len:] = seq_len - 1
    return L


_prefix_cache: dict = {}


def _prefix_lengths_on(segments, prefix_len: int, seq_len: int, device: torch.device) -> torch.Tensor:
    """_build_prefix_lengths on ``device``, kept per (segments, lengths, device): every
    block of a forward pass reads the same read-only L, so it is built once (a few
    entries at most: one per distinct sequence layout, oldest dropped past 16)."""
    key = (tuple(tuple(x) for x in segments), prefix_len, seq_len, str(device))
    L = _prefix_cache.get(key)
    if L is None:
        if len(_prefix_cache) >= 16:
            _prefix_cache.pop(next(iter(_prefix_cache)))
        L = _build_prefix_lengths(segments, prefix_len, seq_len, device)
        _prefix_cache[key] = L
    return L


def _linear(mod, x: torch.Tensor, amax: torch.Tensor | None, scale: torch.Tensor | None = None) -> torch.Tensor:
    """mod(x), with the producer's amax of x when mod is an FP8 linear; with ``scale``,
    x is already the e4m3 input of the FP8 linear mod and ``scale`` its dynamic scale."""
    if scale is not None:
        return mod.forward_e4m3(x, scale)
    if amax is not None and isinstance(mod, FP8Linear):
        return mod.forward_from_amax(x, amax)
    return mod(x)


def _swiglu_linear(mod: FP8Linear, xq: torch.Tensor, scale: torch.Tensor, amax_out: torch.Tensor) -> torch.Tensor:
    """fused_swiglu(*mod(x).chunk(2, -1)) for the fused gate / up FP8 linear ``mod`` handed
    its e4m3 input ``xq`` with scale ``scale``: one GEMM with the SwiGLU in its epilogue
    (the gate / up output is never written); ``amax_out`` receives the result's amax."""
    return mod.forward_swiglu_e4m3(xq, scale, amax_out=amax_out)


def _qkv_fuses_rms_rope(mod, attn, D: int, rotary_emb, S: int) -> bool:
    """The fused QKV linear can apply the q / k RMSNorm + RoPE in its epilogue: an FP8
    linear on the tensor-core path, heads of 128, both norms with fp32-convertible weights
    and one eps, and a rotary table of the sequence's shape (or none)."""
    nq, nk = getattr(attn, "norm_q", None), getattr(attn, "norm_k", None)
    return (isinstance(mod, FP8Linear) and mod.in_features >= 256 and D == 128
            and getattr(nq, "weight", None) is not None and getattr(nk, "weight", None) is not None
            and nq.weight.numel() == D and nk.weight.numel() == D and nq.eps is not None and nq.eps == nk.eps
            and (rotary_emb is None or tuple(rotary_emb.shape) == (S, D // 2)))


def _qkv_rms_rope(mod: FP8Linear, xq: torch.Tensor, scale: torch.Tensor, heads: int, attn,
                  rotary_emb) -> torch.Tensor:
    """The fused QKV linear on its e4m3 input with the q / k RMSNorm + RoPE in the GEMM
    epilogue: [B, S, 3 heads, 128] bf16, q and k heads equal to fused_rms_norm_rope of
    the plain linear's output, v heads equal to that output."""
    return mod.forward_qkv_rms_rope_e4m3(xq, scale, heads, attn.norm_q.weight, attn.norm_k.weight, rotary_emb,
                                         attn.norm_q.eps)


def _gate_linear(mod: FP8Linear, x: torch.Tensor, amax: torch.Tensor | None, residual: torch.Tensor,
                 table: torch.Tensor, target_token_mask: torch.Tensor | None) -> torch.Tensor:
    """fused_gate_residual(residual, mod(x), ...) in one GEMM whose epilogue applies the
    gated residual with the bf16(tanh(gate)) rows of ``table`` (gate_table); same bytes."""
    return mod.forward_gate_residual(x, amax, residual, table, target_token_mask)


def _fuses_gate(lin, after=None) -> bool:
    """An FP8 linear on the tensor-core path (followed by nothing but an identity or an
    inactive dropout) can apply the gated residual in its GEMM epilogue."""
    if not (isinstance(lin, FP8Linear) and lin.in_features >= 256 and lin.out_features % 8 == 0):
        return False
    return (after is None or isinstance(after, torch.nn.Identity)
            or (isinstance(after, torch.nn.Dropout) and (after.p == 0 or not after.training)))


def _takes_e4m3(*mods) -> bool:
    """Every module is an FP8 linear on the tensor-core path (in_features >= 256), so a
    producer may hand them its output already quantized."""
    return all(isinstance(m, FP8Linear) and m.in_features >= 256 for m in mods)


def _new_amax(x: torch.Tensor) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=x.device)


class QwenImage21KernelProcessor:
    """Drop-in for ``QwenImage21AttnProcessor``: same call signature (plus the optional
    ``hidden_states_amax`` / ``hidden_states_scale`` the fused block passes), one
    attention kernel for both the prefill and the decode form."""

    _attention_backend = None
    _parallel_config = None

    def __call__(
        self,
        attn,
        hidden_states: torch.Tensor,
        attention_mask=None,
        rotary_emb=None,
        layer_cache=None,
        kv_cache_mode: str | None = None,
        cache_write_slice=None,
        segments=None,
        key_valid=None,
        hidden_states_amax: torch.Tensor | None = None,
        hidden_states_scale: torch.Tensor | None = None,
        gate_residual: tuple | None = None,
        out_amax: torch.Tensor | None = None,
    ) -> torch.Tensor:
        # hidden_states_scale: hidden_states is then the e4m3 input of the QKV linears
        # (fused_layer_norm_modulate_e4m3), quantized with this scale
        B, S, _ = hidden_states.shape
        H = attn.heads
        fused_qkv = getattr(attn, "fused_qkv", None)
        normed = False
        if fused_qkv is not None:
            # one quantization + one GEMM for Q, K and V; the splits are views
            D = fused_qkv.out_features // (3 * H)
            if hidden_states_scale is not None and _qkv_fuses_rms_rope(fused_qkv, attn, D, rotary_emb, S):
                # the GEMM epilogue normalises and rotates q and k (same bytes)
                qkv = _qkv_rms_rope(fused_qkv, hidden_states, hidden_states_scale, H, attn, rotary_emb)
                normed = True
            else:
                qkv = _linear(fused_qkv, hidden_states, hidden_states_amax, hidden_states_scale).unflatten(-1, (3 * H, D))
            query, key, value = qkv.chunk(3, dim=-2)
        else:
            D = attn.to_q.out_features // H
            query = _linear(attn.to_q, hidden_states, hidden_states_amax, hidden_states_scale).unflatten(-1, (H, D))
            key = _linear(attn.to_k, hidden_states, hidden_states_amax, hidden_states_scale).unflatten(-1, (H, D))
            value = _linear(attn.to_v, hidden_states, hidden_states_amax, hidden_states_scale).unflatten(-1, (H, D))

        if not normed:
            query = fused_rms_norm_rope(query, attn.norm_q.weight, rotary_emb, attn.norm_q.eps)
            key = fused_rms_norm_rope(key, attn.norm_k.weight, rotary_emb, attn.norm_k.eps)

        if kv_cache_mode == "extract" and layer_cache is not None and cache_write_slice is not None:
            # the slab store copies (and quantizes V) on the stream: the views suffice
            layer_cache.store(key[:, cache_write_slice], value[:, cache_write_slice])

        # max|attention output| for the FP8 out-projection, accumulated by the kernel
        # (out_amax: a zeroed int32 word from the caller, e.g. the fused block's, or a new one)
        if not isinstance(attn.to_out[0], FP8Linear):
            out_amax = None
        elif out_amax is None:
            out_amax = _new_amax(query)
        if segments is not None:
            # prefill over the full joint sequence
            assert key_valid is None or key_valid.dim() == 2
            prefix_end = segments[-1][1] if segments else 0
            L = _prefix_lengths_on(segments, prefix_end, S, query.device)
            out = block_causal_flash_attention(query, key, value, L, key_valid, cache_k=None, cache_v=None,
                                               amax_out=out_amax)
        else:
            kv_mask = attention_mask
            if kv_mask is not None:
                kv_mask = kv_mask.reshape(kv_mask.shape[0], -1)
            if layer_cache is not None:
                # decode: target rows over [prefix slab ; fresh target]
                if hasattr(layer_cache, "views"):
                    cache_k, cache_v, v_scale = layer_cache.views()
                else:
                    cache_k, cache_v = layer_cache.get()
                    v_scale = None
                kv_total = cache_k.shape[1] + key.shape[1]
                L = torch.full((key.shape[1],), kv_total - 1, dtype=torch.int32, device=query.device)
                out = block_causal_flash_attention(query, key, value, L, kv_mask, cache_k=cache_k, cache_v=cache_v,
                                                   cache_v_scale=v_scale, uniform_full=kv_mask is None,
                                                   amax_out=out_amax)
            else:
                L = torch.full((key.shape[1],), key.shape[1] - 1, dtype=torch.int32, device=query.device)
                out = block_causal_flash_attention(query, key, value, L, kv_mask, uniform_full=kv_mask is None,
                                                   amax_out=out_amax)

        out = out.flatten(2, 3).type_as(query)
        # the attention epilogue accumulated max|out|: the out-projection's quantizer
        # skips its own max pass
        if gate_residual is not None:
            # (residual, gate table, target mask) from the fused block: the out-projection
            # returns residual + bf16(tanh(gate)) * to_out(out) from its GEMM epilogue
            if not _fuses_gate(attn.to_out[0], attn.to_out[1]):
                raise ValueError("gate_residual needs an FP8 out-projection followed by an identity")
            residual, table, mask = gate_residual
            return _gate_linear(attn.to_out[0], out, out_amax, residual, table, mask)
        out = _linear(attn.to_out[0], out, out_amax)
        return attn.to_out[1](out)


class QwenImage21KernelBlock(torch.nn.Module):
    """Fused replacement for ``QwenImage21TransformerBlock`` (processors.py:129-187):
    reuses the original block's submodules, runs the fused norm / modulation / gate /
    SwiGLU kernels, and sends the attention through the (swapped) processor."""

    def __init__(self, original_block):
        super().__init__()
        self.img_norm1 = original_block.img_norm1  # LayerNorm without affine (params unused)
        self.attn = original_block.attn
        self.img_norm2 = original_block.img_norm2
        self.img_mlp = original_block.img_mlp
        self._eps = self.img_norm1.eps

    def forward(
        self,
        hidden_states: torch.Tensor,  # [B, S, D] bf16
        modulation: torch.Tensor,     # [B (+B), 4 inner]
        rotary_emb=None,
        attention_mask=None,
        target_token_mask=None,
        layer_cache=None,
        kv_cache_mode=None,
        cache_write_slice=None,
        segments=None,
        key_valid=None,
    ) -> torch.Tensor:
        mod_stride = modulation.stride(0)
        fused_qkv = getattr(self.attn, "fused_qkv", None)
        inner = fused_qkv.out_features // 3 if fused_qkv is not None else self.attn.to_q.out_features
        # mod1.scale @ 0, mod1.gate @ inner, mod2.scale @ 2 inner, mod2.gate @ 3 inner
        attn_kwargs = dict(attention_mask=attention_mask, rotary_emb=rotary_emb, layer_cache=layer_cache,
                           kv_cache_mode=kv_cache_mode, cache_write_slice=cache_write_slice, segments=segments,
                           key_valid=key_valid)
        qkv_mods = (fused_qkv,) if fused_qkv is not None else (self.attn.to_q, self.attn.to_k, self.attn.to_v)
        ours = isinstance(getattr(self.attn, "processor", None), QwenImage21KernelProcessor)
        # modulation rows the gates read: the samples' rows, and the t = 0 rows with a mask
        gate_rows = hidden_states.shape[0] * (2 if target_token_mask is not None else 1)
        fuse_gate1 = ours and _fuses_gate(self.attn.to_out[0], self.attn.to_out[1])
        fuse_gate2 = _fuses_gate(self.img_mlp.out)
        table1 = table2 = None
        if fuse_gate1 and fuse_gate2:
            # both gates' tables in one launch: columns [inner, 4 inner) of the modulation
            # (mod1.gate, mod2.scale, mod2.gate), the two gate slices used in place
            tables = gate_table(modulation, inner, gate_rows, 3 * inner)
            table1, table2 = tables[:, :inner], tables[:, 2 * inner:]
        # the max|.| words of the attention output and of the MLP's hidden activation:
        # one zeroed allocation
        amaxes = torch.zeros(2, dtype=torch.int32, device=hidden_states.device) if ours else None
        if ours:
            if _takes_e4m3(*qkv_mods):
                # the norm's only consumers are FP8 linears: it emits their e4m3 input
                img_mod, scale1 = fused_layer_norm_modulate_e4m3(hidden_states, modulation, 0, mod_stride,
                                                                 target_token_mask, self._eps)
                attn_kwargs["hidden_states_scale"] = scale1
            else:
                amax1 = _new_amax(hidden_states)
                img_mod = fused_layer_norm_modulate(hidden_states, modulation, 0, mod_stride, target_token_mask,
                                                    self._eps, amax_out=amax1)
                attn_kwargs["hidden_states_amax"] = amax1
        else:
            img_mod = fused_layer_norm_modulate(hidden_states, modulation, 0, mod_stride, target_token_mask,
                                                self._eps)
        if ours:
            attn_kwargs["out_amax"] = amaxes[0:1]
        if fuse_gate1:
            # the out-projection's GEMM epilogue adds the gated attention output to the residual
            if table1 is None:
                table1 = gate_table(modulation, inner, gate_rows, inner)
            attn_kwargs["gate_residual"] = (hidden_states, table1, target_token_mask)
            hidden_states = self.attn(hidden_states=img_mod, **attn_kwargs)
        else:
            attn_out = self.attn(hidden_states=img_mod, **attn_kwargs)
            hidden_states = fused_gate_residual(hidden_states, attn_out, modulation, inner, target_token_mask)

        fused_up = getattr(self.img_mlp, "fused_up", None)
        up_mods = (fused_up,) if fused_up is not None else (self.img_mlp.gate_layer, self.img_mlp.proj)
        amax2 = scale2 = None
        if _takes_e4m3(*up_mods):
            img_mod2, scale2 = fused_layer_norm_modulate_e4m3(hidden_states, modulation, 2 * inner, mod_stride,
                                                              target_token_mask, self._eps)
        else:
            amax2 = _new_amax(hidden_states)
            img_mod2 = fused_layer_norm_modulate(hidden_states, modulation, 2 * inner, mod_stride, target_token_mask,
                                                 self._eps, amax_out=amax2)
        amax3 = amaxes[1:2] if amaxes is not None else _new_amax(hidden_states)
        if fused_up is not None and scale2 is not None and fused_up.out_features % 256 == 0:
            mlp_mid = _swiglu_linear(fused_up, img_mod2, scale2, amax3)
        else:
            if fused_up is not None:
                gate, up = _linear(fused_up, img_mod2, amax2, scale2).chunk(2, dim=-1)
            else:
                gate = _linear(self.img_mlp.gate_layer, img_mod2, amax2, scale2)
                up = _linear(self.img_mlp.proj, img_mod2, amax2, scale2)
            mlp_mid = fused_swiglu(gate, up, amax_out=amax3)
        if fuse_gate2:
            if table2 is None:
                table2 = gate_table(modulation, 3 * inner, gate_rows, inner)
            return _gate_linear(self.img_mlp.out, mlp_mid, amax3, hidden_states, table2, target_token_mask)
        mlp_out = _linear(self.img_mlp.out, mlp_mid, amax3)
        return fused_gate_residual(hidden_states, mlp_out, modulation, 3 * inner, target_token_mask)


def convert_transformer_to_kernels(transformer, use_fp8: bool = False) -> int:
    """Swap the stock blocks for fused kernel blocks; optionally FP8-quantize the block
    linears (processors.py:190-211).  Returns the number of blocks converted."""
    new_blocks = []
    for blk in transformer.transformer_blocks:
        kb = QwenImage21KernelBlock(blk)
        if use_fp8:
            for lin_name in ("to_q", "to_k", "to_v"):
                lin = getattr(kb.attn, lin_name)
                if isinstance(lin, torch.nn.Linear):
                    setattr(kb.attn, lin_name, FP8Linear.from_linear(lin))
            if isinstance(kb.attn.to_out[0], torch.nn.Linear):
                kb.attn.to_out[0] = FP8Linear.from_linear(kb.attn.to_out[0])
            for mlp_name in ("gate_layer", "proj", "out"):
                lin = getattr(kb.img_mlp, mlp_name, None)
                if isinstance(lin, torch.nn.Linear):
                    setattr(kb.img_mlp, mlp_name, FP8Linear.from_linear(lin))
        kb.attn.set_processor(QwenImage21KernelProcessor())
        new_blocks.append(kb)
    transformer.transformer_blocks = torch.nn.ModuleList(new_blocks)
    return len(new_blocks)
