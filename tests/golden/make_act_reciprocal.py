"""Measure, on a GPU, how the reference's activation cast forms 1/s, for every scale
a bf16 tensor can produce, and write the exceptions to act_reciprocal.npz.

    python tests/golden/make_act_reciprocal.py        # on a B200 with triton installed

The reference's cast kernel (qwen_image_kernel/fp8.py:29-41) computes
``inv = 1.0 / tl.load(scale_ptr)`` as an fp32 division in Triton and then
``(x.to(tl.float32) * inv).to(float8e4nv)``; the scale comes from
``(x.abs().amax().float() / 448.0).clamp_min(1e-12)`` evaluated by torch on CUDA
(fp8.py:24-26).  Both expressions are restated here in the same technology (the
Triton kernel below is a restatement of those three lines, used only to measure
their arithmetic) and evaluated for every positive finite bf16 amax plus amax=0.

Output act_reciprocal.npz:
  scale_bits, inv_bits  -- the scales whose Triton reciprocal differs from the IEEE
                           round-to-nearest reciprocal, and the reciprocal the
                           reference computes for them (oracle.act_reciprocal);
  n_scales, n_diff      -- how many scales were measured / differ;
  torch_scale_mismatch  -- scales where torch-on-CUDA differs from the oracle's
                           SCALE_CUDA form (expected 0);
  cast_mismatch         -- bytes where the Triton cast differs from the oracle's
                           e4m3 satfinite cast on a large random tensor (expected 0).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch
import triton
import triton.language as tl

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
from oracle import oracle as O  # noqa: E402


@triton.jit
def _recip_kernel(s_ptr, out_ptr, n, BLOCK: tl.constexpr):
    offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    live = offs < n
    s = tl.load(s_ptr + offs, mask=live, other=1.0)
    tl.store(out_ptr + offs, 1.0 / s, mask=live)


@triton.jit
def _cast_kernel(x_ptr, out_ptr, s_ptr, n, BLOCK: tl.constexpr):
    offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    live = offs < n
    inv = 1.0 / tl.load(s_ptr)
    x = tl.load(x_ptr + offs, mask=live, other=0.0)
    tl.store(out_ptr + offs, (x.to(tl.float32) * inv).to(out_ptr.dtype.element_ty), mask=live)


def main() -> None:
    dev = torch.device("cuda")
    amax_bits = np.concatenate([[0], np.arange(1, 0x7F80)]).astype(np.uint16)
    amax = torch.from_numpy(amax_bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)
    # the reference's scale expression on CUDA, per amax value (one row each)
    scale = (amax.float() / 448.0).clamp_min(1e-12)
    oracle_scale = np.array([O.scale_from_amax(float(a), O.SCALE_CUDA)
                             for a in (amax_bits.astype(np.uint32) << 16).view(np.float32)], dtype=np.float32)
    torch_scale_mismatch = int((scale.cpu().numpy().view(np.uint32) != oracle_scale.view(np.uint32)).sum())

    inv = torch.empty_like(scale)
    n = scale.numel()
    _recip_kernel[(triton.cdiv(n, 1024),)](scale, inv, n, BLOCK=1024)
    torch.cuda.synchronize()
    s_np = scale.cpu().numpy()
    inv_np = inv.cpu().numpy()
    rn = (np.float32(1.0) / s_np).astype(np.float32)
    diff = inv_np.view(np.uint32) != rn.view(np.uint32)

    # the cast itself on a large random tensor with one fixed scale
    g = np.random.default_rng(0)
    x = torch.from_numpy(g.standard_normal(1 << 22, dtype=np.float32)).to(torch.bfloat16)
    x[:8] *= 20
    xd = x.to(dev)
    s = (xd.abs().amax().float() / 448.0).clamp_min(1e-12)
    q = torch.empty(xd.shape, dtype=torch.float8_e4m3fn, device=dev)
    _cast_kernel[(triton.cdiv(xd.numel(), 8192),)](xd, q, s, xd.numel(), BLOCK=8192, num_warps=8)
    inv_s = torch.empty(1, device=dev)
    _recip_kernel[(1,)](s.reshape(1), inv_s, 1, BLOCK=1024)
    q_ref, s_ref = O.quantize_act(x, O.SCALE_CUDA, inv=float(inv_s.item()))
    cast_mismatch = int((q.cpu().view(torch.uint8).numpy() != q_ref).sum())

    np.savez_compressed(HERE / "act_reciprocal.npz",
                        scale_bits=s_np.view(np.uint32)[diff], inv_bits=inv_np.view(np.uint32)[diff],
                        n_scales=np.int64(n), n_diff=np.int64(diff.sum()),
                        torch_scale_mismatch=np.int64(torch_scale_mismatch),
                        cast_mismatch=np.int64(cast_mismatch))
    print(f"scales measured {n}; reciprocal differs from IEEE RN for {int(diff.sum())}; "
          f"torch scale vs oracle mismatches {torch_scale_mismatch}; cast mismatches {cast_mismatch}")


if __name__ == "__main__":
    main()
