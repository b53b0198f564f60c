"""GPU test of qik_quantize_act_noalloc, the activation quantizer for callers that
cannot allocate device memory (plugin hosts and serving runtimes that give a kernel
only its inputs and outputs, or launch paths where cudaMalloc is not allowed).

It is called through the C ABI (ctypes) twice in a row and compared with the
ordinary entry point qik_quantize_act, which takes a caller-allocated workspace
(zeroed before its first use, as that entry point requires).
The quantizer's tolerance is exact: bytes and scale bits must be equal.  The second
call uses an input with a much smaller amax than the first, so a scratch amax word
left over from the first call would show up as a wrong scale.

This file is collected last on purpose (tests/test_zz_*), and passes both alone in a
fresh process and after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest
import torch

import golden_inputs as GI

pytestmark = pytest.mark.gpu


def _reference_call(lib, x):
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(1, dtype=torch.float32, device=x.device)
    ws = torch.zeros(lib.qik_quant_workspace_bytes(), dtype=torch.uint8, device=x.device)
    rc = lib.qik_quantize_act(ctypes.c_void_p(x.data_ptr()), x.numel(), ctypes.c_void_p(q.data_ptr()),
                              ctypes.c_void_p(s.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.qik_last_error()
    return q, s


def _noalloc_call(lib, x):
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(1, dtype=torch.float32, device=x.device)
    rc = lib.qik_quantize_act_noalloc(ctypes.c_void_p(x.data_ptr()), x.numel(), ctypes.c_void_p(q.data_ptr()),
                                      ctypes.c_void_p(s.data_ptr()),
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.qik_last_error()
    return q, s


def test_noalloc_quantize_matches_workspace_entry_point_twice():
    from qik import _lib as L
    lib = L.load()
    inputs = [GI.outlier_activations(17, 4352, 3072).cuda(),          # amax ~ 100
              GI.randn_bf16(18, (333, 1001), 0.01).cuda()]           # amax ~ 0.05, ragged size
    for x in inputs:
        q_na, s_na = _noalloc_call(lib, x)
        q_ref, s_ref = _reference_call(lib, x)
        torch.cuda.synchronize()
        assert np.array_equal(s_na.cpu().numpy().view(np.uint32), s_ref.cpu().numpy().view(np.uint32))
        assert torch.equal(q_na.view(torch.uint8), q_ref.view(torch.uint8))


def test_noalloc_rejects_bad_arguments():
    from qik import _lib as L
    lib = L.load()
    s = torch.empty(1, dtype=torch.float32, device="cuda")
    rc = lib.qik_quantize_act_noalloc(None, 16, None, ctypes.c_void_p(s.data_ptr()), None)
    assert rc == 1                                                     # QIK_ERR_INVALID
    assert b"NULL" in lib.qik_last_error()
