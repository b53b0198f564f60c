"""CPU checks of the C ABI and the host-side logic (no compute, no GPU needed).

* libqik.so loads and exports every entry point include/qik.h declares, and the
  ctypes binding (qik/_lib.py) declares a signature for each of them;
* argument validation runs on the host and reports QIK_ERR_INVALID with a message,
  before any device work;
* compute calls raise instead of falling back to the CPU when no GPU is present;
* the prefix-length builder reproduces the reference's golden vectors.
"""
import ctypes
import re
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import PKG_DIR, ROOT

HEADER = ROOT / "include" / "qik.h"


def _declared() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(qik_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    so = PKG_DIR / "qik" / "libqik.so"
    if not so.exists():
        subprocess.run([sys.executable, str(PKG_DIR / "build.py")], check=True)
    from qik import _lib as L
    return L.load(require_cuda=False)


def test_header_declares_entry_points():
    names = _declared()
    for required in ("qik_quantize_act", "qik_quantize_weight", "qik_fp8_gemm", "qik_block_causal_attention",
                     "qik_kv_store", "qik_compute_scale", "qik_quantize_act_noalloc"):
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header(lib):
    from qik import _lib as L
    assert set(_declared()) <= set(L.SIGNATURES), set(_declared()) - set(L.SIGNATURES)
    assert L.missing_symbols() == []


def test_version_and_workspace(lib):
    assert lib.qik_version() >= 100
    assert lib.qik_quant_workspace_bytes() >= 4


def test_host_validation_reports_invalid(lib):
    rc = lib.qik_fp8_gemm(None, None, 128, 128, 128, 128, 128, None, None, None, None, 128, 0, 0, None, None, None)
    assert rc == 1 and b"NULL" in lib.qik_last_error()
    rc = lib.qik_fp8_gemm(ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 32, 24, 32, 32, ctypes.c_void_p(16),
                          ctypes.c_void_p(16), None, ctypes.c_void_p(16), 32, 0, 0, None, None, None)
    assert rc == 1 and b"K=24" in lib.qik_last_error()
    from qik import _lib as L
    a = L.AttnArgs()
    a.D = 64
    assert lib.qik_block_causal_attention(ctypes.byref(a), None, None) == 1
    assert b"head_dim" in lib.qik_last_error()
    rc = lib.qik_kv_store(None, None, 1, 10, 2, 128, 0, 0, 0, 0, 0, 0, None, None, 8, 1, None, None, None)
    assert rc == 1 and b"capacity" in lib.qik_last_error()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_compute_without_gpu_raises():
    from qik import _lib as L
    from qik import fp8
    with pytest.raises((L.QikError, ValueError)):
        fp8.quantize_tensorwise(torch.zeros(4, 4, dtype=torch.bfloat16))
    with pytest.raises(L.QikError):
        L.load()


def test_prefix_lengths_match_reference_golden(golden_dir):
    import golden_inputs as GI
    from qik.processors import _build_prefix_lengths
    g = np.load(golden_dir / "prefix_lengths.npz")
    for name, (segments, S) in GI.prefix_cases().items():
        prefix_end = segments[-1][1] if segments else 0
        L = _build_prefix_lengths(segments, prefix_end, S, torch.device("cpu"))
        assert np.array_equal(L.numpy(), g[name]), name
