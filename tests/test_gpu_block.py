"""GPU checks of the attention processor and the fused transformer block
(qik.processors: QwenImage21KernelProcessor, QwenImage21KernelBlock,
convert_transformer_to_kernels) against a CPU composition of the oracle ops.

The modules are stand-ins with the attribute names the reference's processor and
block read (processors.py:50-126, 137-187): ``attn.heads``, ``attn.fused_qkv``,
``attn.norm_q/norm_k`` (weight, eps), ``attn.to_out[0/1]``, ``img_norm1/2`` (eps),
``img_mlp.fused_up/out``; the reference's own block test needs diffusers, which is
not installed.  Each stage of the oracle composition re-quantizes the previous
stage's bf16 output, so the end-to-end gate is a relative Frobenius error (1e-2 for
the processor, 2e-2 for the whole block); a wiring mistake (an offset, a view, a row
map) gives errors of order 1.
"""
import numpy as np
import pytest
import torch
import torch.nn as nn

import golden_inputs as GI
from oracle import oracle as O

pytestmark = pytest.mark.gpu

HEADS, HD = 4, 128
DIM = HEADS * HD  # model width = attention inner width
HIDDEN = 1024


class RMSNorm(nn.Module):
    def __init__(self, weight, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=False)
        self.eps = eps


class Attention(nn.Module):
    def __init__(self, fused_qkv, to_out, wq, wk):
        super().__init__()
        self.heads = HEADS
        self.fused_qkv = fused_qkv
        self.norm_q = RMSNorm(wq)
        self.norm_k = RMSNorm(wk)
        self.to_out = nn.ModuleList([to_out, nn.Identity()])
        self.processor = None

    def set_processor(self, p):
        self.processor = p

    def forward(self, hidden_states, **kw):
        return self.processor(self, hidden_states, **kw)


class MLP(nn.Module):
    def __init__(self, fused_up, out):
        super().__init__()
        self.fused_up = fused_up
        self.out = out


class Block(nn.Module):
    def __init__(self, attn, mlp):
        super().__init__()
        self.img_norm1 = nn.LayerNorm(DIM, elementwise_affine=False, eps=1e-6)
        self.img_norm2 = nn.LayerNorm(DIM, elementwise_affine=False, eps=1e-6)
        self.attn = attn
        self.img_mlp = mlp


def _fp8_linear(seed, n, k, bias=True):
    from qik.fp8 import FP8Linear
    lin = nn.Linear(k, n, bias=bias)
    with torch.no_grad():
        lin.weight.copy_(GI.randn_bf16(seed, (n, k), 0.04).float())
        if bias:
            lin.bias.copy_(GI.randn_bf16(seed + 1, (n,), 0.05).float())
    return FP8Linear.from_linear(lin.cuda())


def _block():
    from qik.processors import QwenImage21KernelProcessor
    attn = Attention(_fp8_linear(500, 3 * DIM, DIM), _fp8_linear(502, DIM, DIM),
                     (GI.randn_bf16(504, (HD,), 0.2) + 1.0), (GI.randn_bf16(505, (HD,), 0.2) + 1.0))
    attn.set_processor(QwenImage21KernelProcessor())
    mlp = MLP(_fp8_linear(506, 2 * HIDDEN, DIM), _fp8_linear(508, DIM, HIDDEN))
    return Block(attn, mlp).cuda()


def _freqs(S, D):
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2).float() / D))
    ang = torch.outer(torch.arange(S).float(), inv)
    return torch.polar(torch.ones_like(ang), ang)


# ---------------------------------------------------------------- oracle composition
def o_linear(x, lin):
    """FP8Linear.forward (fp8.py:78-90) on the CPU: dynamic e4m3 activation, fp32
    dequant GEMM, bf16 out."""
    shp = x.shape
    q, s = O.quantize_act(x.reshape(-1, shp[-1]).contiguous())
    wq = lin.weight.detach().cpu().view(torch.uint8).numpy()
    y = O.fp8_linear(q, s, wq, float(lin.weight_scale.item()), lin.bias)
    return y.to(torch.bfloat16).reshape(*shp[:-1], -1)


def o_attention_part(attn, x, fr, L, cache=None):
    B, S, _ = x.shape
    qkv = o_linear(x, attn.fused_qkv)
    q, k, v = qkv.unflatten(-1, (3 * HEADS, HD)).chunk(3, dim=-2)
    c, s = fr.real.float(), fr.imag.float()
    q = O.rms_norm_rope(q, attn.norm_q.weight.detach().cpu(), c, s, 1e-6)
    k = O.rms_norm_rope(k, attn.norm_k.weight.detach().cpu(), c, s, 1e-6)
    if cache is None:
        o = O.block_causal_attention(q, k, v, L)
    else:
        ck, cv, vs = cache
        o = O.block_causal_attention(q, k, v, L, None, ck, cv, vs)
    return o_linear(o.flatten(2, 3), attn.to_out[0]), k, v


# ---------------------------------------------------------------- processor
def test_processor_prefill_block_causal():
    """Prefill over text + two image blocks + target rows (processors.py:88-97)."""
    blk = _block()
    S = 384
    segments = [(0, 64, True), (64, 160, False), (160, 256, False)]
    x = GI.randn_bf16(510, (1, S, DIM))
    fr = _freqs(S, HD)
    out = blk.attn(hidden_states=x.cuda(), rotary_emb=fr.cuda(), segments=segments)
    torch.cuda.synchronize()
    L = O.build_prefix_lengths(segments, 256, S)
    ref, _, _ = o_attention_part(blk.attn, x, fr, L)
    r = O.relf(out.cpu(), ref)
    print("processor prefill relF", r)
    assert r <= 1e-2


def test_processor_extract_then_decode_through_fp8_slab():
    """Step 1 stores the prefix K/V in the slab (kv_cache_mode="extract",
    processors.py:84-85); later steps attend target rows over [slab ; fresh]
    (processors.py:99-111)."""
    from qik.kv_cache import ContiguousKVCache
    blk = _block()
    P, T = 256, 128
    S = P + T
    segments = [(0, 64, True), (64, P, False)]
    x = GI.randn_bf16(511, (1, S, DIM))
    fr = _freqs(S, HD)
    cache = ContiguousKVCache(1, 1, P, HEADS, HD, v_fp8=True, device="cuda")
    layer = cache.get_layer(0)
    blk.attn(hidden_states=x.cuda(), rotary_emb=fr.cuda(), segments=segments, layer_cache=layer,
             kv_cache_mode="extract", cache_write_slice=slice(0, P))
    # decode: only the target rows, rotary rows of the target positions
    xt = GI.randn_bf16(512, (1, T, DIM))
    fr_t = fr[P:].contiguous()
    out = blk.attn(hidden_states=xt.cuda(), rotary_emb=fr_t.cuda(), layer_cache=layer)
    torch.cuda.synchronize()
    ck, cv, vs = layer.views()
    # the slab holds the prefix keys / values of step 1
    _, k1, v1 = o_attention_part(blk.attn, x, fr, O.build_prefix_lengths(segments, P, S))
    d_k = (ck.cpu().float() - k1[:, :P].float()).abs().max().item()
    assert d_k <= 2.0 ** -6 * k1.float().abs().max().item()
    L = torch.full((T,), P + T - 1, dtype=torch.int32)
    ref, _, _ = o_attention_part(blk.attn, xt, fr_t, L, cache=(ck.cpu(), cv.cpu(), vs.cpu()))
    r = O.relf(out.cpu(), ref)
    print("processor decode relF", r)
    assert r <= 1e-2


def test_processor_without_cache_is_full_attention():
    blk = _block()
    S = 200
    x = GI.randn_bf16(513, (2, S, DIM))
    fr = _freqs(S, HD)
    out = blk.attn(hidden_states=x.cuda(), rotary_emb=fr.cuda())
    torch.cuda.synchronize()
    ref, _, _ = o_attention_part(blk.attn, x, fr, torch.full((S,), S - 1, dtype=torch.int32))
    assert O.relf(out.cpu(), ref) <= 1e-2


# ---------------------------------------------------------------- block
def test_fused_block_matches_oracle_composition():
    """QwenImage21KernelBlock.forward (processors.py:145-187): B=2 with a target mask
    (prefix positions use the t = 0 modulation rows B..2B-1)."""
    from qik.processors import QwenImage21KernelBlock
    torch.manual_seed(0)
    B, S = 2, 256
    blk = QwenImage21KernelBlock(_block())
    x = GI.randn_bf16(514, (B, S, DIM))
    mod = GI.randn_bf16(515, (2 * B, 4 * DIM), 0.2)
    tmask = torch.zeros(S, dtype=torch.bool)
    tmask[64:] = True
    fr = _freqs(S, HD)
    out = blk(x.cuda(), mod.cuda(), rotary_emb=fr.cuda(), target_token_mask=tmask.cuda())
    torch.cuda.synchronize()

    a = blk.attn
    img_mod = O.layer_norm_modulate(x, mod, 0, tmask, 1e-6)
    attn_out, _, _ = o_attention_part(a, img_mod, fr, torch.full((S,), S - 1, dtype=torch.int32))
    h = O.gate_residual(x, attn_out, mod, DIM, tmask)
    img_mod2 = O.layer_norm_modulate(h, mod, 2 * DIM, tmask, 1e-6)
    gate, up = o_linear(img_mod2, blk.img_mlp.fused_up).chunk(2, dim=-1)
    mlp_out = o_linear(O.swiglu(gate, up), blk.img_mlp.out)
    ref = O.gate_residual(h, mlp_out, mod, 3 * DIM, tmask)
    r = O.relf(out.cpu(), ref)
    print("block relF", r, "max-abs", (out.cpu().float() - ref.float()).abs().max().item())
    assert r <= 2e-2


def test_convert_transformer_to_kernels_swaps_blocks_and_processor():
    from qik.processors import QwenImage21KernelBlock, QwenImage21KernelProcessor, convert_transformer_to_kernels

    class T(nn.Module):
        def __init__(self):
            super().__init__()
            self.transformer_blocks = nn.ModuleList([_block(), _block()])

    t = T()
    assert convert_transformer_to_kernels(t) == 2
    assert all(isinstance(b, QwenImage21KernelBlock) for b in t.transformer_blocks)
    assert all(isinstance(b.attn.processor, QwenImage21KernelProcessor) for b in t.transformer_blocks)
    # state-dict names unchanged (submodules reused)
    assert any(k.startswith("0.attn.fused_qkv.weight") for k in t.transformer_blocks.state_dict())
