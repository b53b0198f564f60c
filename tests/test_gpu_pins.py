"""Pins of the oracle's CUDA-side forms, evaluated on the GPU.

1. The reference computes its per-tensor scale with the torch expression
   ``(x.abs().amax().float() / 448.0).clamp_min(1e-12)`` on CUDA (fp8.py:24-26,
   fp8.py:58, kv_cache.py:38-39).  Evaluating that expression with torch on the GPU
   for every positive finite bf16 amax must give the oracle's SCALE_CUDA form.
2. The measured table of the reference's Triton reciprocal (act_reciprocal.npz,
   made by tests/golden/make_act_reciprocal.py on a B200) must be internally
   consistent, and the library's activation cast must reproduce it.
3. The weight path's torch cast (clamp, then .to(float8_e4m3fn)) on CUDA must equal
   the oracle's conversion.
"""
import numpy as np
import pytest
import torch

import golden_inputs as GI
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_scale_expression_on_cuda_is_reciprocal_form():
    bits = np.arange(1, 0x7F80, dtype=np.uint16)
    amax = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).cuda()
    s = (amax.float() / 448.0).clamp_min(1e-12).cpu().numpy()
    f = (bits.astype(np.uint32) << 16).view(np.float32)
    mine = np.array([O.scale_from_amax(float(a), O.SCALE_CUDA) for a in f], dtype=np.float32)
    assert np.array_equal(s.view(np.uint32), mine.view(np.uint32))
    cpu_form = np.array([O.scale_from_amax(float(a), O.SCALE_CPU) for a in f[::50]], dtype=np.float32)
    assert not np.array_equal(s[::50].view(np.uint32), cpu_form.view(np.uint32))


def test_weight_cast_on_cuda_matches_oracle():
    w = GI.randn_bf16(5, (512, 640), 0.02).cuda()
    s = (w.abs().amax().float() / 448.0).clamp_min(1e-12)
    q = (w.float() / s).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    q_ref, s_ref = O.quantize_weight(w.cpu(), O.SCALE_CUDA)
    assert np.float32(s_ref).view(np.uint32) == np.float32(s.item()).view(np.uint32)
    assert np.array_equal(q.cpu().view(torch.uint8).numpy(), q_ref)


def test_act_reciprocal_table_reproduced_by_library(golden_dir):
    path = golden_dir / "act_reciprocal.npz"
    if not path.exists():
        pytest.skip("act_reciprocal.npz not generated yet")
    g = np.load(path)
    assert int(g["torch_scale_mismatch"]) == 0
    assert int(g["cast_mismatch"]) == 0
    from qik import fp8
    # For a sample of scales in the table, build a tensor with that amax and check
    # the library's bytes against the oracle driven by the table's reciprocal.
    sb = g["scale_bits"]
    if sb.size == 0:
        return
    pick = sb[:: max(1, sb.size // 64)]
    for s_bits in pick:
        s = float(np.uint32(s_bits).view(np.float32))
        amax = np.float32(s * 448.0)
        x = GI.randn_bf16(int(s_bits) % 997, (4096,)).float() * float(amax) / 5.0
        x = x.clamp(-float(amax), float(amax)).to(torch.bfloat16)
        x[0] = torch.tensor(float(amax)).to(torch.bfloat16)
        q, sd = fp8.quantize_tensorwise(x.cuda())
        q_ref, s_ref = O.quantize_act(x, O.SCALE_CUDA, inv=O.act_reciprocal(O.compute_scale(x)))
        assert np.array_equal(q.cpu().view(torch.uint8).numpy(), q_ref)
