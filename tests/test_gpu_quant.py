"""GPU parity: the e4m3 quantizers (qik_quantize_act / qik_quantize_weight /
qik_compute_scale) against the CPU oracle, bit-exact (bytes and scale bits)."""
import numpy as np
import pytest
import torch

import golden_inputs as GI
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fp8():
    from qik import fp8 as F
    return F


def _act_oracle(x: torch.Tensor):
    """Activation oracle with the device's 1/s (see test_gpu_pins.py for the pin of
    the reciprocal form; the oracle table of exceptions lives in the golden dir)."""
    return O.quantize_act(x, O.SCALE_CUDA, inv=O.act_reciprocal(O.compute_scale(x, O.SCALE_CUDA)))


def _check_act(fp8, x_cpu: torch.Tensor, dev_x: torch.Tensor | None = None):
    x = dev_x if dev_x is not None else x_cpu.cuda()
    q, s = fp8.quantize_tensorwise(x)
    torch.cuda.synchronize()
    q_ref, s_ref = _act_oracle(x_cpu)
    assert np.float32(s_ref).view(np.uint32) == s.cpu().numpy().view(np.uint32)[0]
    got = q.cpu().view(torch.uint8).numpy().reshape(q_ref.shape)
    bad = int((got != q_ref).sum())
    assert bad == 0, f"{bad} of {got.size} bytes differ"


@pytest.mark.parametrize("shape", [(1,), (17,), (3, 5), (128, 3072), (1000003,), (33, 97)])
def test_quantize_act_small(fp8, shape):
    x = GI.randn_bf16(hash(shape) % 1000, shape)
    _check_act(fp8, x)


def test_quantize_act_cfg1_outliers(fp8):
    """BASELINE config 1 activations: M=4352 x K=3072, 8 outlier channels x20."""
    x = GI.outlier_activations(0, 4352, 3072)
    _check_act(fp8, x)


def test_quantize_act_ffn_hidden_size(fp8):
    """The FFN hidden activation size (4352 x 12288), heavy-tailed values."""
    x = (GI.randn_bf16(5, (4352, 12288)).float() ** 3).to(torch.bfloat16)
    _check_act(fp8, x)


@pytest.mark.parametrize("M", [9472, 16384])
def test_quantize_act_cfg5_rows(fp8, M):
    """configs[4] row counts whose slices exceed shared memory: the remainder is read
    twice (L2 hints), the bytes must not change."""
    x = GI.outlier_activations(40 + M % 7, M, 3072)
    _check_act(fp8, x)


def test_quantize_act_state_reused_across_sizes(fp8):
    """One cached workspace serves calls with different grid sizes in a row: each
    call must leave the barrier ready for the next (no clearing between calls)."""
    shapes = [(256, 3072), (16384, 3072), (1,), (4352, 3072), (33, 97), (1024, 3072)]
    xs = [GI.randn_bf16(60 + i, sh, 0.5 + i) for i, sh in enumerate(shapes)]
    for _ in range(2):
        for x in xs:
            _check_act(fp8, x)


def test_quantize_act_zero_and_edge_values(fp8):
    _check_act(fp8, torch.zeros(1000, dtype=torch.bfloat16))         # amax 0 -> scale 1e-12
    x = GI.randn_bf16(9, (4096,))
    x[7] = 448.0
    x[9] = -3.0e38                                                    # near bf16 max
    x[11] = 1e-40                                                      # bf16 subnormal
    _check_act(fp8, x)


def test_quantize_act_unaligned_view(fp8):
    base = GI.randn_bf16(3, (1, 5003))
    dev = base.cuda()[:, 3:]                                           # 6-byte offset
    _check_act(fp8, base[:, 3:].contiguous(), dev_x=dev.contiguous())
    q, s = fp8.quantize_tensorwise(dev[0, 1:])
    q_ref, s_ref = _act_oracle(base[0, 4:].contiguous())
    assert np.array_equal(q.cpu().view(torch.uint8).numpy(), q_ref)


def test_compute_scale_matches_oracle(fp8):
    for seed, scale in [(1, 1.0), (2, 1e-3), (3, 300.0)]:
        x = GI.randn_bf16(seed, (257, 129), scale)
        s = fp8.compute_scale(x.cuda())
        assert np.float32(O.compute_scale(x)).view(np.uint32) == s.cpu().numpy().view(np.uint32)
    xf = GI.randn_bf16(4, (1000,)).float() * 1.2345
    s = fp8.compute_scale(xf.cuda())
    assert np.float32(O.compute_scale(xf)).view(np.uint32) == s.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("name", list(GI.weight_cases().keys()))
def test_quantize_weight_cases(fp8, name):
    w = GI.weight_cases()[name]
    q, s = fp8.quantize_weight_tensorwise(w.cuda())
    q_ref, s_ref = O.quantize_weight(w, O.SCALE_CUDA)
    assert np.float32(s_ref).view(np.uint32) == s.cpu().numpy().view(np.uint32)[0]
    assert np.array_equal(q.cpu().view(torch.uint8).numpy(), q_ref)


def test_quantize_weight_fused_qkv_shape(fp8):
    """Fused QKV weight of the DiT (3 x [3072, 3072] concatenated, one scale;
    quantize_offline.py:67-89) at BASELINE size."""
    w = torch.cat([GI.randn_bf16(40 + i, (3072, 3072), 0.02) for i in range(3)], 0)
    q, s = fp8.quantize_weight_tensorwise(w.cuda())
    q_ref, s_ref = O.quantize_weight(w, O.SCALE_CUDA)
    assert np.float32(s_ref).view(np.uint32) == s.cpu().numpy().view(np.uint32)[0]
    assert np.array_equal(q.cpu().view(torch.uint8).numpy(), q_ref)


def test_quantize_weight_from_cpu_tensor(fp8):
    w = GI.randn_bf16(50, (96, 320), 0.02)
    q, s = fp8.quantize_weight_tensorwise(w)                           # staged to the GPU
    assert q.device.type == "cpu" and s.device.type == "cpu"
    q_ref, s_ref = O.quantize_weight(w, O.SCALE_CUDA)
    assert np.array_equal(q.view(torch.uint8).numpy(), q_ref)
