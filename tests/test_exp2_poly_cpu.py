"""The FMA-pipe 2^x of the attention softmax (exp2_poly2 in csrc/qik_device.cuh).

* Its cubic's coefficients are the ones tests/exp2_poly.py fits (float32 literals).
* Its steps, restated in float32 numpy (round-to-nearest shifter, exact reduction,
  Horner with fused multiply-adds, integer exponent add), stay within 7.6e-5
  relative of 2^x on [-125, 8] -- below half a bf16 ulp (2^-9) of P.
* Inputs below -125 (and -inf) give at most 2^-124, never more.
The kernel's outputs against MUFU ex2 over the same range are checked on the GPU by
the attention parity tests (every tile with all keys allowed uses it).
"""
import importlib.util
import re
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "qwen-image-kernel_b200" / "csrc"


def _fit_module():
    spec = importlib.util.spec_from_file_location("exp2_poly", Path(__file__).resolve().parent / "exp2_poly.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _kernel_coefficients():
    src = (CSRC / "qik_device.cuh").read_text()
    body = src[src.index("uint64_t exp2_poly2("):]
    body = body[:body.index("\n}\n")]
    lits = re.findall(r"f2_pack\((0x[0-9a-fA-F.p+-]+)f, \1f\)", body)
    vals = [np.float32(float.fromhex(v)) for v in lits]
    # order in the source: c3, c2, c1, c0
    assert len(vals) == 4, lits
    return vals[::-1]


def _fma32(a, b, c):
    return (a.astype(np.float64) * np.float64(b) + np.float64(c)).astype(np.float32)


def exp2_poly_ref(x, c):
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    shift = np.float32(12582912.0)
    r = (x + shift).astype(np.float32)
    n = (r - shift).astype(np.float32)
    f = (x - n).astype(np.float32)
    p = _fma32(f, c[3], c[2])
    p = (p.astype(np.float64) * f.astype(np.float64) + np.float64(c[1])).astype(np.float32)
    p = (p.astype(np.float64) * f.astype(np.float64) + np.float64(c[0])).astype(np.float32)
    bits = p.view(np.uint32) + (r.view(np.uint32) << np.uint32(23))
    return bits.view(np.float32)


def test_kernel_literals_are_the_fitted_coefficients():
    c_fit = np.float32(_fit_module().fit())
    c_k = _kernel_coefficients()
    assert all(a == b for a, b in zip(c_fit, c_k)), (c_fit, c_k)


def test_error_bound_and_underflow():
    c = _kernel_coefficients()
    x = np.linspace(-125.0, 8.0, 2_000_001, dtype=np.float32)
    y = exp2_poly_ref(x, c)
    rel = np.abs(y.astype(np.float64) / np.exp2(x.astype(np.float64)) - 1.0)
    assert rel.max() < 7.6e-5
    assert rel.max() < 2.0 ** -9
    lo = exp2_poly_ref(np.array([-125.5, -200.0, -1e30, -np.inf], dtype=np.float32), c)
    assert np.all(lo > 0) and np.all(lo <= 2.0 ** -124)
