"""Deterministic inputs for the golden vectors (shared by make_golden.py and the tests).

numpy's PCG64 streams are stable across numpy versions, and fp32 -> bf16 rounding
is deterministic, so these regenerate bit-identically on any machine.  Shapes are
scaled-down versions of the reference's own test cases
(tests/test_attention.py:112-117, tests/test_kv_cache.py:15, tests/test_fp8.py:16)
so the CPU oracle finishes in seconds.
"""
from __future__ import annotations

import numpy as np
import torch


def randn_bf16(seed: int, shape, scale: float = 1.0) -> torch.Tensor:
    g = np.random.default_rng(seed)
    a = (g.standard_normal(size=shape, dtype=np.float32) * np.float32(scale)).astype(np.float32)
    return torch.from_numpy(a).to(torch.bfloat16)


def outlier_activations(seed: int, M: int, K: int, n_outlier: int = 8, factor: float = 20.0) -> torch.Tensor:
    """N(0,1) activations with channels [0, n_outlier) scaled by `factor`."""
    g = np.random.default_rng(seed)
    a = g.standard_normal(size=(M, K), dtype=np.float32)
    a[:, :n_outlier] *= np.float32(factor)
    return torch.from_numpy(a).to(torch.bfloat16)


def weight_cases() -> dict[str, torch.Tensor]:
    cases = {
        "w_bf16_64x96": randn_bf16(11, (64, 96), 0.02),
        "w_bf16_outlier": randn_bf16(12, (48, 128), 0.02),
        "w_f32_from_linear": randn_bf16(13, (32, 256), 0.02).float(),
        "w_zero": torch.zeros(16, 32, dtype=torch.bfloat16),
        "w_tiny": randn_bf16(14, (8, 64), 1e-30),
        "w_big": randn_bf16(15, (24, 40), 300.0),
    }
    cases["w_bf16_outlier"][3, 7] = 5.0
    return cases


def kv_cases():
    """name -> (k, v, pmax, num_layers, layer) with k, v [B, P, H, D] bf16."""
    return {
        "kv_b1": (randn_bf16(21, (1, 40, 4, 32)), randn_bf16(22, (1, 40, 4, 32)), 48, 2, 1),
        "kv_b2_ragged": (randn_bf16(23, (2, 33, 3, 16), 0.3), randn_bf16(24, (2, 33, 3, 16), 0.3), 40, 3, 0),
        "kv_outlier_head": (randn_bf16(25, (1, 24, 2, 128)), randn_bf16(26, (1, 24, 2, 128)) * torch.tensor(
            [1.0, 50.0], dtype=torch.bfloat16)[None, None, :, None], 24, 1, 0),
    }


def prefix_cases():
    """name -> (segments [(start, end, is_text)] over the prefix, total seq len)."""
    def segs(layout):
        out, pos = [], 0
        for kind, n in layout:
            out.append((pos, pos + n, kind == "text"))
            pos += n
        return out, pos
    cases = {}
    s, p = segs([("text", 256), ("img", 1024)])
    cases["t2i"] = (s[:1], p)          # target = image rows after the text prefix
    s, p = segs([("text", 64), ("img", 4096), ("text", 32), ("img", 256)])
    cases["edit"] = (s[:-1], p)
    s, p = segs([("text", 256), ("img", 2304), ("img", 4096)])
    cases["cfg4_edit_768"] = (s[:-1], p)
    s, p = segs([("text", 5)])
    cases["text_only"] = (s, p + 7)
    return cases


def _L_from_layout(layout, target_full=True):
    """Per-row L for a run layout where the last run is the target (full attention)."""
    pos = 0
    segs = []
    for kind, n in layout:
        segs.append((pos, pos + n, kind == "text"))
        pos += n
    S = pos
    Lt = torch.arange(S, dtype=torch.int32)
    for a, b, is_text in segs:
        if not is_text:
            Lt[a:b] = b - 1
    if target_full:
        Lt[segs[-1][0]:] = S - 1
    return Lt, S


def attention_cases():
    """name -> dict(q, k, v, L, key_valid, cache_k, cache_v[, slab_fp8])."""
    H, D = 2, 128
    cases = {}

    def prefill(name, layout, seed, batch=1, pad=False):
        L, S = _L_from_layout(layout)
        q = randn_bf16(seed, (batch, S, H, D), 0.3)
        k = randn_bf16(seed + 1, (batch, S, H, D), 0.3)
        v = randn_bf16(seed + 2, (batch, S, H, D), 0.3)
        kv = None
        if pad:
            first_text_end = layout[0][1]
            kv = torch.ones(batch, S, dtype=torch.bool)
            kv[:, first_text_end - 5:first_text_end] = False
        cases[name] = dict(q=q, k=k, v=v, L=L, key_valid=kv, cache_k=None, cache_v=None)

    prefill("t2i_prefill", [("text", 40), ("img", 150)], 100)
    prefill("edit_prefill", [("text", 16), ("img", 130), ("text", 9), ("img", 70)], 110)
    prefill("padded_prompt", [("text", 24), ("img", 100)], 120, pad=True)
    prefill("batch2", [("text", 12), ("img", 61)], 130, batch=2)

    def decode(name, P, T, seed, fp8=False):
        q = randn_bf16(seed, (1, T, H, D), 0.3)
        k = randn_bf16(seed + 1, (1, T, H, D), 0.3)
        v = randn_bf16(seed + 2, (1, T, H, D), 0.3)
        ck = randn_bf16(seed + 3, (1, P, H, D), 0.3)
        cv = randn_bf16(seed + 4, (1, P, H, D), 0.3)
        L = torch.full((T,), P + T - 1, dtype=torch.int32)
        cases[name] = dict(q=q, k=k, v=v, L=L, key_valid=None, cache_k=ck, cache_v=cv, slab_fp8=fp8)

    decode("decode_bf16_slab", 70, 130, 140)
    decode("decode_fp8_slab", 200, 96, 150, fp8=True)
    return cases


def standin_dit(d: int = 64, hidden: int = 96, n_blocks: int = 2, fill: bool = True) -> torch.nn.Module:
    """A small module tree with the attribute names of the Qwen-Image DiT that the e4m3
    cache format depends on: ``transformer_blocks.{i}`` with ``attn.to_q/to_k/to_v``
    (biased), ``attn.norm_q/norm_k`` (RMSNorm weights), ``attn.to_out.0`` and
    ``img_mlp.gate_layer/proj/out``; outside the blocks ``img_in`` (K < 256),
    ``norm_out.linear``, ``proj_out``, a persistent ``time_embed.freqs`` buffer (which
    the writer drops) and a buffer that is a view of another (which it must copy
    out).  ``fill=False`` leaves the tensors as allocated (use under a meta device
    context to get the skeleton a cache loads into); otherwise every tensor is drawn
    from ``randn_bf16`` with a fixed seed, so the tree rebuilds bit-identically."""
    nn = torch.nn
    seed = iter(range(1000, 2000))

    def linear(k, n, bias):
        lin = nn.Linear(k, n, bias=bias, dtype=torch.bfloat16)
        if fill:
            with torch.no_grad():
                lin.weight.copy_(randn_bf16(next(seed), (n, k), 0.02))
                if bias:
                    lin.bias.copy_(randn_bf16(next(seed), (n,), 0.1))
        return lin

    def block():
        b = nn.Module()
        b.img_norm1 = nn.LayerNorm(d, elementwise_affine=False, eps=1e-6)
        b.attn = nn.Module()
        for name in ("to_q", "to_k", "to_v"):
            setattr(b.attn, name, linear(d, d, True))
        b.attn.norm_q = nn.RMSNorm(32, eps=1e-6, dtype=torch.bfloat16)
        b.attn.norm_k = nn.RMSNorm(32, eps=1e-6, dtype=torch.bfloat16)
        b.attn.to_out = nn.ModuleList([linear(d, d, True), nn.Dropout(0.0)])
        b.img_norm2 = nn.LayerNorm(d, elementwise_affine=False, eps=1e-6)
        b.img_mlp = nn.Module()
        b.img_mlp.gate_layer = linear(d, hidden, False)
        b.img_mlp.proj = linear(d, hidden, False)
        b.img_mlp.out = linear(hidden, d, False)
        if fill:
            with torch.no_grad():
                b.attn.norm_q.weight.copy_(randn_bf16(next(seed), (32,), 0.5))
                b.attn.norm_k.weight.copy_(randn_bf16(next(seed), (32,), 0.5))
        return b

    m = nn.Module()
    m.img_in = linear(16, d, True)
    m.time_embed = nn.Module()
    m.time_embed.register_buffer("freqs", torch.arange(8, dtype=torch.float32))
    m.time_embed.linear_1 = linear(32, d, True)
    table = torch.zeros(12, 4, dtype=torch.float32) if not fill else randn_bf16(next(seed), (12, 4)).float()
    m.register_buffer("pos_table", table)
    m.register_buffer("pos_table_head", table[:3])
    m.transformer_blocks = nn.ModuleList([block() for _ in range(n_blocks)])
    m.norm_out = nn.Module()
    m.norm_out.linear = linear(d, 2 * d, True)
    m.proj_out = linear(d, 16, True)
    return m
