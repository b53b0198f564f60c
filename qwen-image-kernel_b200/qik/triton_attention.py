"""Block-causal flash attention on the sm_100a tensor core (no Triton inside).

Drop-in for ``qwen_image_kernel/triton_attention.py`` of gomezcojj-coder/
qwen-image-kernel: the module keeps the reference's name so imports resolve
unchanged, and ``block_causal_flash_attention`` keeps its signature, assertions
and semantics (triton_attention.py:171-260) while the arithmetic runs in the
tcgen05 kernel ``qik_block_causal_attention`` of libqik.so.

The allowed set of query row r is the prefix interval kv <= L[r] of the virtual
concatenation [cache ; fresh] (triton_attention.py:3-18); the e4m3 cache V is
dequantized in the loop as bf16(fl32(v8) * scale[b, h]).  bf16 and fp16 tensors are
both accepted, as in the reference (P is rounded to the tensors' type before P.V).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib as L


def block_causal_flash_attention(
    query: torch.Tensor,             # [B, SQ, H, D]
    key: torch.Tensor,               # [B, SN, H, D]  fresh keys
    value: torch.Tensor,             # [B, SN, H, D]
    prefix_lengths: torch.Tensor,    # [SQ] int32
    key_valid: torch.Tensor | None,  # [B, KV_TOTAL] bool or None
    cache_k: torch.Tensor | None = None,  # [B, P, H, D]
    cache_v: torch.Tensor | None = None,
    cache_v_scale: torch.Tensor | None = None,  # [B, H] fp32, only with fp8 cache V
    uniform_full: bool = False,  # caller guarantee: L == KV_TOTAL-1 for every row
    amax_out: torch.Tensor | None = None,  # int32 [1]: atomic max of the fp32 bits of max|out|
) -> torch.Tensor:
    """Exact block-causal attention via per-row prefix lengths.

    When ``cache_k``/``cache_v`` are given, keys/values are the *virtual* concat
    [cache, key]; ``key``/``value`` then hold only the fresh segment and
    ``prefix_lengths``/``key_valid`` are indexed in absolute (cache-aware) space.
    Rows with ``L = -1`` attend to nothing and produce zeros.  When
    ``cache_v_scale`` is given the cache V is fp8e4m3 dequantized per head.
    ``amax_out`` (int32 [1] on the query's device) receives, by atomic max, the fp32
    bits of max|out|: the dynamic scale of the FP8 out-projection that follows
    (``FP8Linear.forward_from_amax``) without another pass over ``out``.
    """
    assert query.dtype in (torch.bfloat16, torch.float16), "fp16/bf16 only"
    assert key.dtype == query.dtype and value.dtype == query.dtype, "q, k, v must share one dtype"
    B, SQ, H, D = query.shape
    if cache_k is not None:
        P = cache_k.shape[1]
        SN = key.shape[1]
        assert cache_k.shape[2] == H and key.shape[2] == H
        assert cache_k.dtype == key.dtype
    else:
        P = 0
        SN = key.shape[1]
    out = torch.empty_like(query)

    def unit_d(t: torch.Tensor) -> torch.Tensor:
        return t if t.stride(-1) == 1 else t.contiguous()

    q, k, v = unit_d(query), unit_d(key), unit_d(value)
    a = L.AttnArgs()
    flags = 0
    if key_valid is not None:
        kv_bytes = key_valid.to(torch.uint8).contiguous()
        flags |= L.ATTN_HAS_KEY_VALID
        a.key_valid = kv_bytes.data_ptr()
        a.kv_sb = kv_bytes.stride(0)
    v_fp8 = cache_v_scale is not None
    if v_fp8:
        assert cache_v is not None and cache_v.dtype == torch.float8_e4m3fn
    elif P > 0:
        assert cache_v.dtype == key.dtype
    if query.dtype == torch.float16:
        flags |= L.ATTN_F16
    if P > 0:
        ck, cv = unit_d(cache_k), unit_d(cache_v)
        flags |= L.ATTN_HAS_CACHE
        a.cache_k, a.cache_v = ck.data_ptr(), cv.data_ptr()
        a.ck_sb, a.ck_ss, a.ck_sh = ck.stride(0), ck.stride(1), ck.stride(2)
        a.cv_sb, a.cv_ss, a.cv_sh = cv.stride(0), cv.stride(1), cv.stride(2)
        if v_fp8:
            vs = cache_v_scale.to(torch.float32).contiguous()
            flags |= L.ATTN_V_FP8
            a.cache_v_scale = vs.data_ptr()
    uniform = uniform_full and key_valid is None
    if uniform:
        flags |= L.ATTN_UNIFORM
    Lt = prefix_lengths.to(device=query.device, dtype=torch.int32).contiguous()
    a.q, a.k, a.v, a.out, a.L = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), Lt.data_ptr()
    a.B, a.SQ, a.SN, a.P, a.H, a.D = B, SQ, SN, P, H, D
    a.q_sb, a.q_ss, a.q_sh = q.stride(0), q.stride(1), q.stride(2)
    a.k_sb, a.k_ss, a.k_sh = k.stride(0), k.stride(1), k.stride(2)
    a.v_sb, a.v_ss, a.v_sh = v.stride(0), v.stride(1), v.stride(2)
    a.o_sb, a.o_ss, a.o_sh = out.stride(0), out.stride(1), out.stride(2)
    a.sm_scale = D ** -0.5
    a.flags = flags
    if amax_out is not None:
        if amax_out.dtype != torch.int32 or amax_out.device != query.device:
            raise ValueError("block_causal_flash_attention: amax_out must be int32 on the query's device")
        a.amax_out = amax_out.data_ptr()
    lib = L.load()
    status = L.status_word(query.device)
    with torch.cuda.device(query.device):
        L.check(lib.qik_block_causal_attention(ctypes.byref(a), status.data_ptr(), L.stream_ptr()),
                "qik_block_causal_attention")
    # The temporaries (key-valid bytes, L, scales) return to torch's stream-ordered
    # allocator, which reuses them only for work queued after this launch.
    return out


def reference_block_causal_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    prefix_lengths: torch.Tensor,
    key_valid: torch.Tensor | None,
    cache_k: torch.Tensor | None = None,
    cache_v: torch.Tensor | None = None,
) -> torch.Tensor:
    """fp32 PyTorch statement of the attention semantics, exported because the
    reference module exports a function of this name and signature for its unit
    tests (triton_attention.py:266-293).  ``block_causal_flash_attention`` never calls
    it.  Keys and values are the concatenation [cache ; fresh]; query row r sees key j
    when j <= prefix_lengths[r] and, with ``key_valid`` [B, KV], key j of its sample
    is valid.  As in the reference, a row that sees no key comes out NaN (a softmax
    over an empty set), where the kernel writes zeros."""
    keys = key if cache_k is None else torch.cat((cache_k, key), dim=1)
    vals = value if cache_v is None else torch.cat((cache_v, value), dim=1)
    j = torch.arange(keys.shape[1], device=query.device)
    visible = j.view(1, 1, -1) <= prefix_lengths.to(query.device).view(1, -1, 1)       # [1, SQ, KV]
    if key_valid is not None:
        visible = visible & key_valid.to(torch.bool).view(key_valid.shape[0], 1, -1)   # [B, SQ, KV]
    logits = torch.einsum("bqhd,bkhd->bhqk", query.float(), keys.float()) * query.shape[-1] ** -0.5
    weights = logits.masked_fill(~visible.unsqueeze(1), float("-inf")).softmax(dim=-1)
    return torch.einsum("bhqk,bkhd->bqhd", weights, vals.float()).to(query.dtype)
