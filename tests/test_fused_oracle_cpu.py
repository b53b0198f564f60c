"""CPU checks of the fused elementwise oracle (oracle.rms_norm_rope, layer_norm_modulate,
gate_residual, swiglu) and of the host validation of their C entry points.

The reference has no golden vectors for these ops: its test (tests/test_fused.py)
compares the Triton kernels with plain-torch "stock" expressions at max-abs < 4e-2.
Those stock expressions are restated below (tests/test_fused.py:25-37, 47-58,
70-80, 88-93) and the oracle, which follows the kernels' own rounding points, must
meet the same bound against them on the same kind of inputs.
"""
import ctypes

import numpy as np
import pytest
import torch

import golden_inputs as GI
from oracle import oracle as O

BOUND = 4e-2  # tests/test_fused.py:33,59,81,94


def stock_rms_norm_rope(x, weight, freqs_cis, eps):
    """tests/test_fused.py:25-37."""
    var = x.float().pow(2).mean(-1, keepdim=True)
    y = x * torch.rsqrt(var + eps)
    y = y * weight.float()
    y = y.to(x.dtype)
    xc = torch.view_as_complex(y.float().reshape(*y.shape[:-1], -1, 2))
    rot = xc * freqs_cis.unsqueeze(1)
    return torch.view_as_real(rot).flatten(-2).to(x.dtype)


def stock_ln_modulate(x, modulation, scale_off, row_map, eps):
    """tests/test_fused.py:47-58 (one sample: rows are the row map)."""
    D = x.shape[-1]
    x32 = x.float()
    mu = x32.mean(-1, keepdim=True)
    var = x32.var(-1, unbiased=False, keepdim=True)
    y = ((x32 - mu) / torch.sqrt(var + eps)).to(torch.bfloat16)
    sel = modulation[row_map.long()][:, scale_off:scale_off + D]
    return y * (1 + sel)


def _freqs(S, D):
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2).float() / D))
    ang = torch.outer(torch.arange(S).float(), inv)
    return torch.polar(torch.ones_like(ang), ang)


def test_rms_rope_oracle_vs_stock():
    B, S, H, D = 1, 40, 4, 128
    x = GI.randn_bf16(301, (B, S, H, D), 0.7)
    w = torch.from_numpy(np.random.default_rng(302).standard_normal(D).astype(np.float32) * 0.3)
    fr = _freqs(S, D)
    mine = O.rms_norm_rope(x, w, fr.real.float(), fr.imag.float(), 1e-6)
    ref = stock_rms_norm_rope(x, w, fr, 1e-6)
    assert (mine.float() - ref.float()).abs().max().item() < BOUND


def test_ln_modulate_oracle_vs_stock():
    B, S, D = 1, 50, 512
    x = GI.randn_bf16(303, (B, S, D))
    mod = GI.randn_bf16(304, (B + 1, 4 * D), 0.2)
    tmask = torch.from_numpy(np.random.default_rng(305).random(S) > 0.5)
    row_map = torch.where(tmask, 0, B)
    mine = O.layer_norm_modulate(x, mod, 0, tmask, 1e-6)
    ref = stock_ln_modulate(x, mod, 0, row_map, 1e-6)
    assert (mine.float() - ref.float()).abs().max().item() < BOUND


def test_gate_residual_oracle_equals_stock():
    """The oracle's rounding chain is the stock expression's: bit-identical."""
    B, S, D = 1, 50, 512
    x = GI.randn_bf16(306, (B, S, D))
    f = GI.randn_bf16(307, (B, S, D), 2.0)
    mod = GI.randn_bf16(308, (B + 1, 4 * D), 0.2)
    tmask = torch.from_numpy(np.random.default_rng(309).random(S) > 0.5)
    mine = O.gate_residual(x, f, mod, D, tmask)
    sel = mod[torch.where(tmask, 0, B)][:, D:2 * D]
    ref = x + torch.tanh(sel) * f              # tests/test_fused.py:79
    assert (mine.float() - ref.float()).abs().max().item() < BOUND
    assert torch.equal(mine, ref[None] if ref.dim() == 2 else ref)


def test_swiglu_oracle_vs_stock():
    g = GI.randn_bf16(310, (1, 30, 1024))
    p = GI.randn_bf16(311, (1, 30, 1024))
    mine = O.swiglu(g, p)
    ref = torch.nn.functional.silu(g) * p      # tests/test_fused.py:92
    assert (mine.float() - ref.float()).abs().max().item() < BOUND


def test_modulation_rows_follow_row_map_plus_sample():
    """Row map 0 / B (triton_fused.py:141-151) plus the sample index the kernels add."""
    mask = torch.tensor([True, False, True])
    rows = O.modulation_rows(mask, 2, 3)
    assert rows.tolist() == [[0, 2, 0], [1, 3, 1]]
    assert O.modulation_rows(None, 2, 3).tolist() == [[0, 0, 0], [1, 1, 1]]


@pytest.fixture(scope="module")
def lib():
    from qik import _lib as L
    return L.load(require_cuda=False)


def test_fused_entry_points_validate_on_host(lib):
    p = ctypes.c_void_p(256)
    rc = lib.qik_rms_norm_rope(p, 1, 4, 2, 96, 768, 192, 96, p, p, p, ctypes.c_float(1e-6), p, 768, 192, 96, None)
    assert rc == 3 and b"head dim" in lib.qik_last_error()
    rc = lib.qik_rms_norm_rope(p, 1, 4, 2, 128, 1024, 256, 130, p, p, p, ctypes.c_float(1e-6), p, 1024, 256, 128,
                               None)
    assert rc == 1 and b"strides" in lib.qik_last_error()
    # a target mask needs the t = 0 rows B..2B-1
    rc = lib.qik_layer_norm_modulate(p, 2, 8, 64, p, 3, 256, 0, p, ctypes.c_float(1e-6), p, None, None)
    assert rc == 1 and b"modulation rows" in lib.qik_last_error()
    rc = lib.qik_layer_norm_modulate(p, 2, 8, 64, p, 4, 256, 200, None, ctypes.c_float(1e-6), p, None, None)
    assert rc == 1 and b"offset" in lib.qik_last_error()
    rc = lib.qik_gate_residual(p, p, 2, 8, 64, p, 1, 256, 64, None, p, None)
    assert rc == 1 and b"modulation rows" in lib.qik_last_error()
    rc = lib.qik_swiglu(p, 24, p, 24, 4, 12, p, 12, None, None)
    assert rc == 1 and b"multiples of 8" in lib.qik_last_error()
    # empty inputs are a no-op
    assert lib.qik_swiglu(None, 8, None, 8, 0, 8, None, 8, None, None) == 0
