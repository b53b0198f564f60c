"""GPU parity of the fused elementwise kernels (csrc/qik_fused.cu) against the CPU
oracle, which restates the reference's Triton kernels (triton_fused.py) with their
rounding points, and against the stock expressions of the reference's own test
(tests/test_fused.py) at its bound.

Gates:
* vs the oracle: at most 0.5% of the bf16 outputs differ, none by more than 2^-6 of
  the largest |output|, and the relative Frobenius error is <= 1e-3.  The kernels and
  the oracle round at the same points; the remaining differences are last-bit
  differences of fp32 sums / rsqrt that flip a bf16 rounding.
* vs the stock expressions: max-abs < 4e-2 (tests/test_fused.py:33,59,81,94).
* amax outputs: bit-exact against the amax of the kernel's own output.
"""
import numpy as np
import pytest
import torch

import golden_inputs as GI
from oracle import oracle as O
from test_fused_oracle_cpu import stock_ln_modulate, stock_rms_norm_rope

pytestmark = pytest.mark.gpu

STOCK_BOUND = 4e-2


@pytest.fixture(scope="module")
def F():
    from qik import triton_fused
    return triton_fused


def _gate(out, ref, tag):
    o = out.detach().cpu().float()
    r = ref.float()
    diff = (o - r).abs()
    frac = (diff > 0).float().mean().item()
    top = r.abs().max().item()
    relf = O.relf(o, r)
    print(f"{tag}: mismatch {frac:.2e} max-abs {diff.max().item():.3e} (top {top:.3f}) relF {relf:.2e}")
    assert frac <= 5e-3, (tag, frac)
    assert diff.max().item() <= top * 2.0 ** -6, (tag, diff.max().item())
    assert relf <= 1e-3, (tag, relf)


def _freqs(S, D):
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2).float() / D))
    ang = torch.outer(torch.arange(S).float(), inv)
    return torch.polar(torch.ones_like(ang), ang)


def test_rms_rope_reference_case(F):
    """tests/test_fused.py:40-52 shape: B=1, S=300, H=32, D=128, fp32 weight."""
    B, S, H, D = 1, 300, 32, 128
    x = GI.randn_bf16(401, (B, S, H, D), 0.7)
    w = torch.from_numpy(np.random.default_rng(402).standard_normal(D).astype(np.float32) * 0.3)
    fr = _freqs(S, D)
    out = F.fused_rms_norm_rope(x.cuda(), w.cuda(), fr.cuda(), 1e-6)
    torch.cuda.synchronize()
    _gate(out, O.rms_norm_rope(x, w, fr.real.float(), fr.imag.float(), 1e-6), "rms_rope")
    assert (out.cpu().float() - stock_rms_norm_rope(x, w, fr, 1e-6).float()).abs().max().item() < STOCK_BOUND


@pytest.mark.parametrize("D", [64, 128, 256])
def test_rms_rope_strided_qkv_views(F, D):
    """q / k as the processor slices them from the fused QKV output
    (processors.py:69-70): [B, S, H, D] views with token stride 3 H D, read in place;
    bf16 norm weight (a bf16 checkpoint)."""
    B, S, H = 2, 77, 6
    qkv = GI.randn_bf16(403 + D, (B, S, 3 * H * D), 0.5)
    w = GI.randn_bf16(404, (D,), 0.3) + 1.0
    fr = _freqs(S, D)
    q_cpu, k_cpu, _ = qkv.unflatten(-1, (3 * H, D)).chunk(3, dim=-2)
    qkv_d = qkv.cuda()
    q, k, _ = qkv_d.unflatten(-1, (3 * H, D)).chunk(3, dim=-2)
    assert not q.is_contiguous()
    for name, t, tc in (("q", q, q_cpu), ("k", k, k_cpu)):
        out = F.fused_rms_norm_rope(t, w.cuda(), fr.cuda(), 1e-6)
        torch.cuda.synchronize()
        _gate(out, O.rms_norm_rope(tc, w, fr.real.float(), fr.imag.float(), 1e-6), f"rms_rope D={D} {name}")


def test_ln_modulate_reference_case(F):
    """tests/test_fused.py:61-75 shape: B=1, S=500, D=4096, R=B+1 rows, random mask."""
    B, S, D = 1, 500, 4096
    x = GI.randn_bf16(405, (B, S, D))
    mod = GI.randn_bf16(406, (B + 1, 4 * D), 0.2)
    tmask = torch.from_numpy(np.random.default_rng(407).random(S) > 0.5)
    amax = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = F.fused_layer_norm_modulate(x.cuda(), mod.cuda(), 0, 4 * D, tmask.cuda(), 1e-6, amax_out=amax)
    torch.cuda.synchronize()
    _gate(out, O.layer_norm_modulate(x, mod, 0, tmask, 1e-6), "ln_modulate")
    ref_stock = stock_ln_modulate(x, mod, 0, torch.where(tmask, 0, B), 1e-6)
    assert (out.cpu().float() - ref_stock.float()).abs().max().item() < STOCK_BOUND
    assert int(amax.item()) == int(out.float().abs().max().view(torch.int32).item())


@pytest.mark.parametrize("mask", [False, True])
def test_ln_modulate_batch2_dit_width(F, mask):
    """B=2 (CFG batch), D=3072 (the DiT width), scale of the second modulation
    (offset 2 * inner) with the t = 0 rows B..2B-1."""
    B, S, D = 2, 333, 3072
    x = GI.randn_bf16(408, (B, S, D), 2.0)
    mod = GI.randn_bf16(409, (2 * B, 4 * D), 0.3)
    tm = torch.from_numpy(np.random.default_rng(410).random(S) > 0.3) if mask else None
    out = F.fused_layer_norm_modulate(x.cuda(), mod.cuda(), 2 * D, 4 * D, None if tm is None else tm.cuda(), 1e-6)
    torch.cuda.synchronize()
    _gate(out, O.layer_norm_modulate(x, mod, 2 * D, tm, 1e-6), f"ln_modulate B=2 mask={mask}")


def test_ln_modulate_rejects_missing_t0_rows(F):
    from qik import _lib as L
    x = torch.zeros(2, 8, 64, dtype=torch.bfloat16, device="cuda")
    mod = torch.zeros(3, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(L.QikError, match="modulation rows"):
        F.fused_layer_norm_modulate(x, mod, 0, 256, torch.ones(8, dtype=torch.bool, device="cuda"), 1e-6)


@pytest.mark.parametrize("B,mask", [(1, True), (2, False), (2, True)])
def test_gate_residual(F, B, mask):
    """tests/test_fused.py:78-96 shape for B=1; gate of mod1 at offset D."""
    S, D = 500, 4096 if B == 1 else 3072
    x = GI.randn_bf16(411 + B, (B, S, D))
    f = GI.randn_bf16(413 + B, (B, S, D), 2.0)
    mod = GI.randn_bf16(415 + B, (2 * B, 4 * D), 0.2)
    tm = torch.from_numpy(np.random.default_rng(417).random(S) > 0.5) if mask else None
    out = F.fused_gate_residual(x.cuda(), f.cuda(), mod.cuda(), D, None if tm is None else tm.cuda())
    torch.cuda.synchronize()
    ref = O.gate_residual(x, f, mod, D, tm)
    _gate(out, ref, f"gate_residual B={B} mask={mask}")


def test_swiglu_reference_case(F):
    """tests/test_fused.py:99-108 shape: [1, 300, 12288]."""
    g = GI.randn_bf16(420, (1, 300, 12288))
    p = GI.randn_bf16(421, (1, 300, 12288))
    out = F.fused_swiglu(g.cuda(), p.cuda())
    torch.cuda.synchronize()
    _gate(out, O.swiglu(g, p), "swiglu")
    ref_stock = torch.nn.functional.silu(g) * p
    assert (out.cpu().float() - ref_stock.float()).abs().max().item() < STOCK_BOUND


def test_swiglu_fused_up_halves_and_amax(F):
    """gate / up as the two halves of the fused up-projection output
    (processors.py:182-186), read in place, with the down projection's amax."""
    M, N = 1000, 3072
    gu = GI.randn_bf16(422, (2, M // 2, 2 * N), 1.5)
    g_cpu, p_cpu = gu.chunk(2, dim=-1)
    g, p = gu.cuda().chunk(2, dim=-1)
    amax = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = F.fused_swiglu(g, p, amax_out=amax)
    torch.cuda.synchronize()
    _gate(out, O.swiglu(g_cpu, p_cpu), "swiglu halves")
    assert int(amax.item()) == int(out.float().abs().max().view(torch.int32).item())


def test_rms_rope_head_major_layout(F):
    """A [B, H, S, D] tensor seen as [B, S, H, D] (heads not contiguous within a token):
    the register-only kernel, same gate."""
    B, S, H, D = 2, 50, 5, 128
    base = GI.randn_bf16(420, (B, H, S, D), 0.7)
    x_cpu = base.transpose(1, 2)
    x = base.cuda().transpose(1, 2)
    w = GI.randn_bf16(421, (D,), 0.3) + 1.0
    fr = _freqs(S, D)
    out = F.fused_rms_norm_rope(x, w.cuda(), fr.cuda(), 1e-6)
    torch.cuda.synchronize()
    _gate(out, O.rms_norm_rope(x_cpu, w, fr.real.float(), fr.imag.float(), 1e-6), "rms_rope head-major")


def test_ln_modulate_full_t2i_block_shape(F):
    """The DiT block's shape (B = 2, S = 4352, D = 3072: 8704 rows streamed through the
    shared-memory ring, several rounds of every stage) with the amax output."""
    B, S, D = 2, 4352, 3072
    x = GI.randn_bf16(422, (B, S, D), 1.5)
    mod = GI.randn_bf16(423, (B, 4 * D), 0.3)
    amax = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = F.fused_layer_norm_modulate(x.cuda(), mod.cuda(), 0, 4 * D, None, 1e-6, amax_out=amax)
    torch.cuda.synchronize()
    _gate(out, O.layer_norm_modulate(x, mod, 0, None, 1e-6), "ln_modulate t2i")
    assert int(amax.item()) == int(out.float().abs().max().view(torch.int32).item())


# ---------------------------------------------------------------- layer norm -> e4m3
def _ln_e4m3_check(F, x, mod, off, tm, tag):
    """fused_layer_norm_modulate_e4m3 against the composition it replaces: the bf16
    layer-norm kernel followed by the activation quantizer (codes and scale
    bit-identical), and the oracle's quantizer on that bf16 output (bit-exact); the
    bf16 output itself passes the fused-op gate against the oracle."""
    from qik.fp8 import quantize_tensorwise
    xd, md = x.cuda(), mod.cuda()
    tmd = None if tm is None else tm.cuda()
    q, s = F.fused_layer_norm_modulate_e4m3(xd, md, off, mod.shape[1], tmd, 1e-6)
    ref = F.fused_layer_norm_modulate(xd, md, off, mod.shape[1], tmd, 1e-6)
    q_ref, s_ref = quantize_tensorwise(ref)
    torch.cuda.synchronize()
    qb = q.view(torch.uint8).cpu()
    mism = (qb != q_ref.view(torch.uint8).cpu()).sum().item()
    print(f"{tag}: scale {s.item():.6g} code mismatches {mism}")
    assert mism == 0, tag
    assert s.cpu().view(torch.int32).item() == s_ref.cpu().view(torch.int32).item(), tag
    q_o, s_o = O.quantize_act(ref.cpu())
    assert np.array_equal(qb.numpy().reshape(q_o.shape), q_o), tag
    assert np.float32(s_o) == np.float32(s.item()), tag
    _gate(ref, O.layer_norm_modulate(x, mod, off, tm, 1e-6), tag)
    return q, s


@pytest.mark.parametrize("mask", [False, True])
def test_ln_modulate_e4m3_batch2_ragged(F, mask):
    """B = 2, S = 333 (666 rows: the last 8-row group partial), D = 3072, the second
    modulation's scale with and without the t = 0 rows."""
    B, S, D = 2, 333, 3072
    x = GI.randn_bf16(430, (B, S, D), 2.0)
    mod = GI.randn_bf16(431, (2 * B, 4 * D), 0.3)
    tm = torch.from_numpy(np.random.default_rng(432).random(S) > 0.3) if mask else None
    _ln_e4m3_check(F, x, mod, 2 * D, tm, f"ln_e4m3 B=2 mask={mask}")


def test_ln_modulate_e4m3_reference_case_width_4096(F):
    """tests/test_fused.py:61-75's shape (B = 1, S = 500, D = 4096, random mask): a
    64 KB stage, so only two stages fit beside the table."""
    B, S, D = 1, 500, 4096
    x = GI.randn_bf16(433, (B, S, D))
    mod = GI.randn_bf16(434, (B + 1, 4 * D), 0.2)
    tm = torch.from_numpy(np.random.default_rng(435).random(S) > 0.5)
    _ln_e4m3_check(F, x, mod, 0, tm, "ln_e4m3 D=4096")


def test_ln_modulate_e4m3_tiny(F):
    """Fewer row groups than SMs (a grid of one CTA) and a narrow row."""
    x = GI.randn_bf16(436, (1, 3, 64))
    mod = GI.randn_bf16(437, (1, 256), 0.2)
    _ln_e4m3_check(F, x, mod, 64, None, "ln_e4m3 tiny")


def test_ln_modulate_e4m3_full_t2i_block_shape_calls_in_a_row(F):
    """The DiT block's shape (B = 2, S = 4352, D = 3072; each CTA makes two passes over
    7 or 8 groups), three calls in a row on one workspace with the amplitude changing
    (large, small, large): each call's grid barrier and amax slots start from what the
    last call left."""
    from qik import _lib as L
    B, S, D = 2, 4352, 3072
    mod = GI.randn_bf16(439, (B, 4 * D), 0.3)
    for i, amp in enumerate((3.0, 0.25, 1.5)):
        x = GI.randn_bf16(440 + i, (B, S, D), amp)
        _ln_e4m3_check(F, x, mod, 0, None, f"ln_e4m3 t2i call {i}")
    assert L.device_status(torch.device("cuda", 0)) == 0


def test_ln_modulate_e4m3_rejects_unaligned_codes(F):
    from qik import _lib as L
    lib = L.load()
    x = torch.zeros(1, 8, 64, dtype=torch.bfloat16, device="cuda")
    mod = torch.zeros(1, 256, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(8 * 64 + 16, dtype=torch.uint8, device="cuda")
    s = torch.empty(1, dtype=torch.float32, device="cuda")
    ws = torch.zeros(lib.qik_quant_workspace_bytes(), dtype=torch.uint8, device="cuda")
    rc = lib.qik_layer_norm_modulate_e4m3(x.data_ptr(), 1, 8, 64, mod.data_ptr(), 1, 256, 0, None, 1e-6,
                                          q.data_ptr() + 8, s.data_ptr(), ws.data_ptr(), None,
                                          L.stream_ptr())
    assert rc == 1 and b"16-byte aligned" in lib.qik_last_error()
