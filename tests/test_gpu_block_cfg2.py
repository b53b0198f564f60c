"""BASELINE configs[2] at full size: the DiT block at 1024 px with CFG batch 2
(M = 2 x 4352 token rows, width 3072, 24 heads of 128) through the product API
(qik.processors.QwenImage21KernelBlock.forward), checked stage by stage against the
CPU oracle on the product's own intermediates.

Every kernel call the block makes is recorded (inputs and output) by wrapping the
module-level functions qik.processors calls; each recorded stage is then recomputed by
the oracle from the recorded inputs:

* gated residual (and RMSNorm + RoPE, SwiGLU where they run as kernels): the fused-op gate of test_gpu_fused.py
  (<= 0.5% of outputs differ, none by more than 2^-6 of the largest output, relF <=
  1e-3), and each amax output equal to the max |output|;
* the two LayerNorm + modulate stages, which emit the next linear's e4m3 input: codes
  and scale bit-identical to the bf16 layer-norm kernel followed by the oracle's
  quantizer on the same recorded input, and that bf16 output at the fused-op gate;
* every FP8 linear: its bf16 output within max-abs 2e-2 + half a bf16 ulp and relF
  <= 5e-3 of the fp32 dequant oracle on the same input, quantized by the oracle
  (bit-exact with the product's quantizer, tested elsewhere) with the amax the
  product's producer handed over, or on the e4m3 input and scale it was handed;
* the attention: max-abs <= 2e-2 and relF <= 5e-3 against the fp32 oracle on the q /
  k / v the processor passed, all 48 (sample, head) pairs;
* the fused QKV linear with the q / k RMSNorm + RoPE in its epilogue: bit-identical to
  the plain GEMM followed by the RMSNorm + RoPE kernel; against the oracle's dequant GEMM
  -> bf16 -> RMSNorm + RoPE, v within the linear gate, q and k within relF <= 5e-3 and
  no error above 2^-6 of the largest output (a last-bit change of a GEMM output moves
  its normalised value by up to two bf16 ulps);
* the out-projection and the down projection with the gated residual in their
  epilogues: bit-identical to the linear followed by the gated-residual kernel, and
  against the oracle's dequant GEMM -> bf16 -> gated residual within relF <= 5e-3 and no
  error above 2^-6 of the largest output (the residual stream grows to |x| ~ 8, where a
  last-bit change of a linear output moves a sum by one bf16 ulp of 2^-4); the gate
  tables within 2^-8 of tanh;
* the fused up projection with the SwiGLU in its epilogue: bit-identical (values and
  amax) to the plain GEMM's gate / up halves through the SwiGLU kernel, and at the
  fused-op gate against the oracle's SwiGLU of the bf16-rounded fp32 dequant GEMM.

The structure is the reference block's (processors.py:129-187): fused QKV 3072 -> 9216,
out-projection 3072 -> 3072, SwiGLU MLP with its fused up projection at BASELINE's
3072 -> 12288 and 6144 -> 3072 down.
"""
import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import oracle as O

pytestmark = pytest.mark.gpu

H, D, K, HALF, B, S = 24, 128, 3072, 6144, 2, 4352
LIN_MAX_ABS, LIN_RELF = 2e-2, 5e-3


class _Attn(nn.Module):
    def __init__(self, fused_qkv, to_out, wq, wk):
        super().__init__()
        self.heads = H
        self.fused_qkv = fused_qkv
        self.norm_q = nn.RMSNorm(D, eps=1e-6)
        self.norm_k = nn.RMSNorm(D, eps=1e-6)
        with torch.no_grad():
            self.norm_q.weight.copy_(wq)
            self.norm_k.weight.copy_(wk)
        self.to_out = nn.ModuleList([to_out, nn.Identity()])
        self.processor = None

    def set_processor(self, p):
        self.processor = p

    def forward(self, hidden_states, **kw):
        return self.processor(self, hidden_states, **kw)


def _lin(g, n_out, n_in, bias):
    from qik.fp8 import FP8Linear, quantize_weight_tensorwise
    f = FP8Linear(n_in, n_out, bias=bias).cuda()
    wq, sw = quantize_weight_tensorwise(torch.randn(n_out, n_in, device="cuda", generator=g) * 0.02)
    f.weight.copy_(wq)
    f.weight_scale.copy_(sw)
    if bias:
        f.bias.copy_((torch.randn(n_out, device="cuda", generator=g) * 0.05).to(torch.bfloat16))
    return f


@pytest.fixture
def recorder(monkeypatch):
    """Wraps the kernels qik.processors calls and records (name, inputs, output)."""
    import qik.processors as PR
    calls = []

    def cpu(t):
        if isinstance(t, torch.Tensor):
            return t.detach().cpu()
        return tuple(cpu(x) for x in t) if isinstance(t, tuple) else t

    def wrap(name, fn):
        def inner(*a, **kw):
            out = fn(*a, **kw)
            rec = {"name": name, "args": [cpu(x) for x in a], "kw": {k: cpu(v) for k, v in kw.items()}}
            if name in ("linear", "swiglu_linear", "qkv_rms_rope", "gate_linear"):
                rec["mod"] = a[0]
            if name == "qkv_rms_rope":
                rec["attn"] = a[4]
            torch.cuda.synchronize()
            rec["out"] = cpu(out)
            for k in ("amax_out",):
                if isinstance(kw.get(k), torch.Tensor):
                    rec["kw"][k] = kw[k].detach().cpu()
            if name == "swiglu_linear":
                rec["kw"]["amax_out"] = a[3].detach().cpu()  # positional, filled by the call
            calls.append(rec)
            return out
        return inner

    for name, attr in (("ln_mod", "fused_layer_norm_modulate"), ("ln_mod_e4m3", "fused_layer_norm_modulate_e4m3"),
                       ("rms_rope", "fused_rms_norm_rope"),
                       ("gate_res", "fused_gate_residual"), ("swiglu", "fused_swiglu"),
                       ("attention", "block_causal_flash_attention"), ("linear", "_linear"),
                       ("swiglu_linear", "_swiglu_linear"), ("qkv_rms_rope", "_qkv_rms_rope"),
                       ("gate_linear", "_gate_linear"), ("gate_table", "gate_table")):
        monkeypatch.setattr(PR, attr, wrap(name, getattr(PR, attr)))
    return calls


def _fused_gate(out, ref, tag):
    o, r = out.float(), ref.float()
    diff = (o - r).abs()
    frac = (diff > 0).float().mean().item()
    top = r.abs().max().item()
    relf = O.relf(o, r)
    print(f"{tag}: mismatch {frac:.2e} max-abs {diff.max().item():.3e} relF {relf:.2e}")
    assert frac <= 5e-3 and diff.max().item() <= top * 2.0 ** -6 and relf <= 1e-3, tag


def _amax_bits_of(t):
    return int(np.array([t.float().abs().max().item()], np.float32).view(np.int32)[0])


def test_dit_block_cfg2_full_size_stage_by_stage(recorder):
    from qik.processors import QwenImage21KernelBlock, QwenImage21KernelProcessor
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device="cuda").manual_seed(2024)
    attn = _Attn(_lin(g, 3 * K, K, True), _lin(g, K, K, True),
                 1.0 + 0.2 * torch.randn(D, device="cuda", generator=g),
                 1.0 + 0.2 * torch.randn(D, device="cuda", generator=g))
    attn.set_processor(QwenImage21KernelProcessor())
    shell = nn.Module()
    shell.img_norm1 = nn.LayerNorm(K, elementwise_affine=False, eps=1e-6)
    shell.img_norm2 = nn.LayerNorm(K, elementwise_affine=False, eps=1e-6)
    shell.attn = attn
    shell.img_mlp = nn.Module()
    shell.img_mlp.fused_up = _lin(g, 2 * HALF, K, False)
    shell.img_mlp.out = _lin(g, K, HALF, False)
    block = QwenImage21KernelBlock(shell)
    x = torch.randn(B, S, K, device="cuda", generator=g).to(torch.bfloat16)
    mod = (torch.randn(B, 4 * K, device="cuda", generator=g) * 0.3).to(torch.bfloat16)
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device="cuda").float() / D))
    freqs = torch.polar(torch.ones(S, D // 2, device="cuda"), torch.outer(torch.arange(S, device="cuda").float(), inv))
    out = block(x, mod, rotary_emb=freqs, segments=[(0, 256, True)])
    torch.cuda.synchronize()
    names = [c["name"] for c in recorder]
    # one gate_table launch covers both gates (modulation columns [K, 4K))
    assert names == ["gate_table", "ln_mod_e4m3", "qkv_rms_rope", "attention", "gate_linear",
                     "ln_mod_e4m3", "swiglu_linear", "gate_linear"], names
    assert recorder[-1]["out"].shape == (B, S, K) and torch.equal(recorder[-1]["out"], out.cpu())
    torch.set_num_threads(max(1, torch.get_num_threads()))
    cos, sin = freqs.real.float().cpu(), freqs.imag.float().cpu()
    for i, c in enumerate(recorder):
        a, kw, o = c["args"], c["kw"], c["out"]
        tag = f"stage {i} {c['name']}"
        if c["name"] == "ln_mod":
            xin, m, off = a[0], a[1], a[2]
            _fused_gate(o, O.layer_norm_modulate(xin, m, off, a[4], a[5]), tag)
            assert int(kw["amax_out"][0]) == _amax_bits_of(o), tag
        elif c["name"] == "ln_mod_e4m3":
            from qik.triton_fused import fused_layer_norm_modulate
            xin, m, off = a[0], a[1], a[2]
            ref = fused_layer_norm_modulate(xin.cuda(), m.cuda(), off, a[3], a[4], a[5]).cpu()
            q_o, s_o = O.quantize_act(ref)
            assert np.array_equal(o[0].view(torch.uint8).numpy().reshape(q_o.shape), q_o), tag
            assert np.float32(s_o) == np.float32(o[1].item()), tag
            _fused_gate(ref, O.layer_norm_modulate(xin, m, off, a[4], a[5]), tag)
        elif c["name"] == "rms_rope":
            _fused_gate(o, O.rms_norm_rope(a[0], a[1], cos, sin, a[3]), tag)
        elif c["name"] == "gate_res":
            _fused_gate(o, O.gate_residual(a[0], a[1], a[2], a[3], a[4]), tag)
        elif c["name"] == "swiglu":
            _fused_gate(o, O.swiglu(a[0], a[1]), tag)
            assert int(kw["amax_out"][0]) == _amax_bits_of(o), tag
        elif c["name"] == "gate_table":
            m, off, rows, width = a[0], a[1], a[2], a[3]
            ref = torch.tanh(m[:rows, off:off + width].float())
            assert (o.float() - ref).abs().max().item() <= 2.0 ** -8, tag
        elif c["name"] == "gate_linear":
            # bit-identical to the linear + the gated-residual kernel, and within the linear
            # gate of the oracle's dequant GEMM -> bf16 -> gated residual
            from qik.triton_fused import fused_gate_residual
            lin, xin, amax, resid, mask = c["mod"], a[1], a[2], a[3], a[5]
            off = K if i < 6 else 3 * K
            f = lin.forward_from_amax(xin.cuda(), None if amax is None else amax.cuda())
            ref = fused_gate_residual(resid.cuda(), f, mod, off, None if mask is None else mask.cuda()).cpu()
            assert torch.equal(o, ref), tag
            x2 = xin.reshape(-1, xin.shape[-1]).contiguous()
            if amax is not None:
                assert int(amax[0]) == _amax_bits_of(x2), tag
            q8, s8 = O.quantize_act(x2)
            y = O.fp8_linear(q8, s8, lin.weight.cpu(), float(lin.weight_scale.item()),
                             None if lin.bias is None else lin.bias.cpu()).to(torch.bfloat16).view(o.shape)
            oref = O.gate_residual(resid, y, mod.cpu(), off, mask).float()
            gf = o.float()
            d = (gf - oref).abs().max().item() / oref.abs().max().item()
            r = O.relf(gf, oref)
            print(f"{tag}: max-abs / max|ref| {d:.3e} relF {r:.3e}")
            assert d <= 2.0 ** -6 and r <= LIN_RELF, tag
        elif c["name"] == "qkv_rms_rope":
            # bit-identical to the plain GEMM + the RMSNorm + RoPE kernel on its q / k views,
            # and within the linear gate of the oracle's linear -> bf16 -> RMSNorm + RoPE
            from qik.fp8 import fp8_gemm
            from qik.triton_fused import fused_rms_norm_rope
            lin, xq, sx, heads, at = c["mod"], a[1], a[2], a[3], c["attn"]
            Bq, Sq, Kq = xq.shape
            x2 = xq.reshape(-1, Kq).cuda()
            plain = fp8_gemm(x2, sx.cuda(), lin.weight, lin.weight_scale, lin.bias).view(Bq, Sq, 3 * heads, D)
            pq, pk, pv = plain.chunk(3, dim=-2)
            rq = fused_rms_norm_rope(pq, at.norm_q.weight, freqs, at.norm_q.eps).cpu()
            rk = fused_rms_norm_rope(pk, at.norm_k.weight, freqs, at.norm_k.eps).cpu()
            oq, ok_, ov = o.chunk(3, dim=-2)
            assert torch.equal(oq, rq) and torch.equal(ok_, rk) and torch.equal(ov, pv.cpu()), tag
            q8, s8 = x2.view(torch.uint8).cpu().numpy(), float(sx.item())
            y = O.fp8_linear(q8, s8, lin.weight.cpu(), float(lin.weight_scale.item()),
                             None if lin.bias is None else lin.bias.cpu()).to(torch.bfloat16).view(Bq, Sq, 3 * heads, D)
            yq, yk, yv = y.chunk(3, dim=-2)
            refs = (O.rms_norm_rope(yq, at.norm_q.weight.detach().cpu(), cos, sin, at.norm_q.eps),
                    O.rms_norm_rope(yk, at.norm_k.weight.detach().cpu(), cos, sin, at.norm_k.eps), yv)
            for part, (got, ref) in zip("qkv", zip((oq, ok_, ov), refs)):
                gf, rf = got.float(), ref.float()
                r = O.relf(gf, rf)
                if part == "v":  # the linear's own output: the linear gate
                    d = ((gf - rf).abs() - 0.5 * O.bf16_ulp(rf)).max().item()
                    print(f"{tag} {part}: max-abs over half an ulp {d:.3e} relF {r:.3e}")
                    assert d <= LIN_MAX_ABS and r <= LIN_RELF, (tag, part)
                else:  # normalised heads (|out| up to ~5): errors relative to the largest output
                    d = (gf - rf).abs().max().item() / rf.abs().max().item()
                    print(f"{tag} {part}: max-abs / max|ref| {d:.3e} relF {r:.3e}")
                    assert d <= 2.0 ** -6 and r <= LIN_RELF, (tag, part)
        elif c["name"] == "swiglu_linear":
            # bit-identical to the plain GEMM's halves through the SwiGLU kernel, and
            # within the linear + elementwise gates of the oracle's composition
            from qik.fp8 import fp8_gemm
            from qik.triton_fused import fused_swiglu
            lin, xq, sx = c["mod"], a[1], a[2]
            x2 = xq.reshape(-1, xq.shape[-1]).cuda()
            gu = fp8_gemm(x2, sx.cuda(), lin.weight, lin.weight_scale, lin.bias)
            am = torch.zeros(1, dtype=torch.int32, device="cuda")
            ref = fused_swiglu(*gu.chunk(2, dim=-1), amax_out=am).cpu()
            y = o.reshape(-1, o.shape[-1])
            assert torch.equal(y, ref), tag
            assert int(kw["amax_out"][0]) == int(am[0]) == _amax_bits_of(y), tag
            q, s = x2.view(torch.uint8).cpu().numpy(), float(sx.item())
            gu_ref = O.fp8_linear(q, s, lin.weight.cpu(), float(lin.weight_scale.item()),
                                  None if lin.bias is None else lin.bias.cpu())
            h = gu_ref.shape[-1] // 2
            _fused_gate(y, O.swiglu(gu_ref[:, :h].to(torch.bfloat16), gu_ref[:, h:].to(torch.bfloat16)), tag)
        elif c["name"] == "linear":
            lin, xin, amax = c["mod"], a[1], a[2]
            x2 = xin.reshape(-1, xin.shape[-1]).contiguous()
            if xin.dtype == torch.float8_e4m3fn:  # handed its e4m3 input and scale
                q, s = x2.view(torch.uint8).numpy(), float(a[3].item())
            else:
                if amax is not None:  # the producer's amax is max|x| itself
                    assert int(amax[0]) == _amax_bits_of(x2), tag
                q, s = O.quantize_act(x2)
            ref = O.fp8_linear(q, s, lin.weight.cpu(), float(lin.weight_scale.item()),
                               None if lin.bias is None else lin.bias.cpu())
            y = o.reshape(-1, o.shape[-1]).float()
            d = ((y - ref).abs() - 0.5 * O.bf16_ulp(ref)).max().item()
            r = O.relf(y, ref)
            print(f"{tag}: {tuple(x2.shape)} -> {y.shape[-1]}: max-abs over half an ulp {d:.3e} relF {r:.3e}")
            assert d <= LIN_MAX_ABS and r <= LIN_RELF, tag
        elif c["name"] == "attention":
            q, k, v, L, kv = a[0], a[1], a[2], a[3], a[4]
            ref = O.block_causal_attention(q, k, v, L, kv, out_dtype=torch.float32)
            d = (o.float() - ref).abs().max().item()
            r = O.relf(o, ref)
            print(f"{tag}: max-abs {d:.3e} relF {r:.3e}")
            assert d <= 2e-2 and r <= 5e-3, tag
            if isinstance(kw.get("amax_out"), torch.Tensor):
                assert int(kw["amax_out"][0]) == _amax_bits_of(o), tag
