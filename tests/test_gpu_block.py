"""GPU checks of the attention processor and the fused transformer block
(qik.processors: QwenImage21KernelProcessor, QwenImage21KernelBlock,
convert_transformer_to_kernels) against a CPU composition of the oracle ops.

The modules are stand-ins with the attribute names the reference's processor and
block read (processors.py:50-126, 137-187): ``attn.heads``, ``attn.fused_qkv``,
``attn.norm_q/norm_k`` (weight, eps), ``attn.to_out[0/1]``, ``img_norm1/2`` (eps),
``img_mlp.fused_up/out``; the reference's own block test needs diffusers, which is
not installed.

Gates.  Every FP8 linear re-quantizes its bf16 input with a dynamic per-tensor scale,
so a last-bit difference in the largest element of an intermediate (a different but
equally exact summation order) moves the scale and re-rounds about half of the e4m3
codes: ~2% relative Frobenius error end to end with no error in any stage.  The
processor is therefore checked stage by stage on its own intermediates, captured at
the attention call: attention on the q / k / v the processor passed (relF <= 5e-3),
and the out-projection on the processor's own attention output (relF <= 5e-3, the
quantizer being bit-exact).  End to end against the oracle composition from the
hidden states the gate is 5e-2: it catches wiring mistakes (an offset, a view, a row
map), which give errors of order 1.
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


E2E_GATE = 5e-2    # end to end through re-quantizing FP8 linears (wiring check)
STAGE_GATE = 5e-3  # one stage on the product's own inputs


@pytest.fixture
def capture(monkeypatch):
    """Records each attention call the processor makes (inputs, options, output)."""
    import qik.processors as PR
    calls = []
    real = PR.block_causal_flash_attention

    def wrap(q, k, v, L, key_valid, **kw):
        out = real(q, k, v, L, key_valid, **kw)
        cpu = lambda t: None if t is None else t.detach().cpu()  # noqa: E731
        calls.append({"q": cpu(q), "k": cpu(k), "v": cpu(v), "L": cpu(L), "key_valid": cpu(key_valid),
                      "cache_k": cpu(kw.get("cache_k")), "cache_v": cpu(kw.get("cache_v")),
                      "cache_v_scale": cpu(kw.get("cache_v_scale")), "out": cpu(out)})
        return out

    monkeypatch.setattr(PR, "block_causal_flash_attention", wrap)
    return calls


def check_stages(attn, call, out, tag):
    """Attention on the processor's own q / k / v, and the out-projection on its own
    attention output."""
    ref_att = O.block_causal_attention(call["q"], call["k"], call["v"], call["L"], call["key_valid"],
                                       call["cache_k"], call["cache_v"], call["cache_v_scale"],
                                       out_dtype=torch.float32)
    r_att = O.relf(call["out"], ref_att)
    r_out = O.relf(out.cpu(), o_linear(call["out"].flatten(2, 3), attn.to_out[0]))
    print(f"{tag}: attention stage relF {r_att:.2e}, out-projection stage relF {r_out:.2e}")
    assert r_att <= STAGE_GATE and r_out <= STAGE_GATE


# ---------------------------------------------------------------- processor
def test_processor_prefill_block_causal(capture):
    """Prefill over text + two image blocks + target rows (processors.py:88-97)."""
    blk = _block()
    S = 384
    segments = [(0, 64, True), (64, 160, False), (160, 256, False)]
    x = GI.randn_bf16(510, (1, S, DIM))
    fr = _freqs(S, HD)
    out = blk.attn(hidden_states=x.cuda(), rotary_emb=fr.cuda(), segments=segments)
    torch.cuda.synchronize()
    check_stages(blk.attn, capture[-1], out, "prefill")
    L = O.build_prefix_lengths(segments, 256, S)
    assert torch.equal(capture[-1]["L"].long(), L.long())
    ref, _, _ = o_attention_part(blk.attn, x, fr, L)
    r = O.relf(out.cpu(), ref)
    print("processor prefill end-to-end relF", r)
    assert r <= E2E_GATE


def test_processor_extract_then_decode_through_fp8_slab(capture):
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
    check_stages(blk.attn, capture[-1], out, "decode")
    ck, cv, vs = layer.views()
    # the slab holds the prefix keys / values of step 1
    _, k1, v1 = o_attention_part(blk.attn, x, fr, O.build_prefix_lengths(segments, P, S))
    d_k = (ck.cpu().float() - k1[:, :P].float()).abs().max().item()
    assert d_k <= 2.0 ** -6 * k1.float().abs().max().item()
    L = torch.full((T,), P + T - 1, dtype=torch.int32)
    ref, _, _ = o_attention_part(blk.attn, xt, fr_t, L, cache=(ck.cpu(), cv.cpu(), vs.cpu()))
    r = O.relf(out.cpu(), ref)
    print("processor decode end-to-end relF", r)
    assert r <= E2E_GATE


def test_processor_without_cache_is_full_attention(capture):
    blk = _block()
    S = 200
    x = GI.randn_bf16(513, (2, S, DIM))
    fr = _freqs(S, HD)
    out = blk.attn(hidden_states=x.cuda(), rotary_emb=fr.cuda())
    torch.cuda.synchronize()
    check_stages(blk.attn, capture[-1], out, "no cache")
    ref, _, _ = o_attention_part(blk.attn, x, fr, torch.full((S,), S - 1, dtype=torch.int32))
    r = O.relf(out.cpu(), ref)
    print("processor without cache end-to-end relF", r)
    assert r <= E2E_GATE


# ---------------------------------------------------------------- block
def test_fused_block_matches_oracle_composition(capture):
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
    c = capture[-1]
    r_att = O.relf(c["out"], O.block_causal_attention(c["q"], c["k"], c["v"], c["L"], c["key_valid"],
                                                     out_dtype=torch.float32))
    print("block attention stage relF", r_att)
    assert r_att <= STAGE_GATE

    a = blk.attn
    img_mod = O.layer_norm_modulate(x, mod, 0, tmask, 1e-6)
    attn_out, _, _ = o_attention_part(a, img_mod, fr, torch.full((S,), S - 1, dtype=torch.int32))
    h = O.gate_residual(x, attn_out, mod, DIM, tmask)
    img_mod2 = O.layer_norm_modulate(h, mod, 2 * DIM, tmask, 1e-6)
    gate, up = o_linear(img_mod2, blk.img_mlp.fused_up).chunk(2, dim=-1)
    mlp_out = o_linear(O.swiglu(gate, up), blk.img_mlp.out)
    ref = O.gate_residual(h, mlp_out, mod, 3 * DIM, tmask)
    r = O.relf(out.cpu(), ref)
    print("block end-to-end relF", r, "max-abs", (out.cpu().float() - ref.float()).abs().max().item())
    assert r <= E2E_GATE


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
