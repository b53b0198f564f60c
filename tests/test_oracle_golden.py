"""Pin the CPU oracle against golden vectors produced by the reference's own code.

The fixtures under tests/golden/ were made by tests/golden/make_golden.py, which
ran the reference's CPU-runnable functions (fp8.py compute_scale and
quantize_weight_tensorwise, kv_cache.py ContiguousKVCache, triton_attention.py
reference_block_causal_attention, processors.py _build_prefix_lengths).  Those
ran on CPU tensors, so the per-tensor scale is the true-division form
(oracle.SCALE_CPU); the CUDA form is pinned on the GPU in test_gpu_pins.py.
"""
import numpy as np
import torch

import golden_inputs as GI
from oracle import oracle as O


def test_compute_scale_all_bf16_amax(golden_dir):
    g = np.load(golden_dir / "compute_scale_cpu.npz")
    amax = g["amax_bits"].astype(np.uint32) << 16
    amax_f = amax.view(np.float32)
    mine = np.array([O.scale_from_amax(float(a), O.SCALE_CPU) for a in amax_f], dtype=np.float32)
    assert np.array_equal(mine.view(np.uint32), g["scale"].view(np.uint32))
    assert np.float32(O.scale_from_amax(0.0, O.SCALE_CPU)) == g["zero_scale"]


def test_cuda_scale_form_differs_from_cpu_form(golden_dir):
    """Documents the evaluation-form hazard: amax * fl32(1/448) and amax / 448 differ
    in the last bit for about half of all bf16 amax values."""
    g = np.load(golden_dir / "compute_scale_cpu.npz")
    amax_f = (g["amax_bits"].astype(np.uint32) << 16).view(np.float32)
    cuda = amax_f * O._RECIP_448
    cuda = np.maximum(cuda, np.float32(1e-12))
    diff = int((cuda.view(np.uint32) != g["scale"].view(np.uint32)).sum())
    assert 0.3 * amax_f.size < diff < 0.7 * amax_f.size
    mine = np.array([O.scale_from_amax(float(a), O.SCALE_CUDA) for a in amax_f[::97]], dtype=np.float32)
    assert np.array_equal(mine.view(np.uint32), cuda[::97].view(np.uint32))


def test_weight_quant_golden(golden_dir):
    g = np.load(golden_dir / "weight_quant.npz")
    for name, w in GI.weight_cases().items():
        q, s = O.quantize_weight(w, O.SCALE_CPU)
        assert np.float32(s).view(np.uint32) == g[f"{name}__s"].view(np.uint32)[0], name
        assert np.array_equal(q, g[f"{name}__q"]), name


def test_kv_cache_store_golden(golden_dir):
    g = np.load(golden_dir / "kv_cache.npz")
    for name, (k, v, pmax, layers, layer) in GI.kv_cases().items():
        B, P, H, D = k.shape
        # bf16 V: plain transpose into [L, B, H, Pmax, D]
        tag = f"{name}__fp80"
        kb = g[f"{tag}__k_buf"].reshape(layers, B, H, pmax, D)
        kt = k.transpose(1, 2).contiguous().view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(kb[layer, :, :, :P], kt)
        assert np.array_equal(g[f"{tag}__v_buf"].reshape(layers, B, H, pmax, D)[layer, :, :, :P],
                              v.transpose(1, 2).contiguous().view(torch.int16).numpy().view(np.uint16))
        assert int(g[f"{tag}__lengths"][layer]) == P
        # fp8 V: per-(b, h) scale and bytes
        tag = f"{name}__fp81"
        v8, sc = O.slab_v_store(v, pmax, O.SCALE_CPU)
        ref_v8 = g[f"{tag}__v_buf"].reshape(layers, B, H, pmax, D)[layer]
        assert np.array_equal(v8[:, :, :P], ref_v8[:, :, :P]), name
        assert np.array_equal(sc.view(np.uint32), g[f"{tag}__v_scale"][layer].view(np.uint32)), name
        # views(): [B, P, H, D] with strides (H*Pmax*D, D, Pmax*D, 1)
        st = g[f"{tag}__views_strides"]
        assert tuple(st[:4]) == (H * pmax * D, D, pmax * D, 1)


def test_prefix_lengths_golden(golden_dir):
    g = np.load(golden_dir / "prefix_lengths.npz")
    for name, (segments, S) in GI.prefix_cases().items():
        prefix_end = segments[-1][1] if segments else 0
        L = O.build_prefix_lengths(segments, prefix_end, S)
        assert np.array_equal(L.numpy(), g[name]), name


def test_cfg4_prefix_lengths_semantics(golden_dir):
    """text rows L=q, cond block L=2559, target rows L=6655."""
    L = np.load(golden_dir / "prefix_lengths.npz")["cfg4_edit_768"]
    assert L.shape == (6656,)
    assert np.array_equal(L[:256], np.arange(256))
    assert (L[256:2560] == 2559).all() and (L[2560:] == 6655).all()
    pairs = int((L.astype(np.int64) + 1).sum())
    assert pairs == 33_194_112


def test_attention_oracle_golden(golden_dir):
    g = np.load(golden_dir / "attention.npz")
    for name, c in GI.attention_cases().items():
        if c.get("slab_fp8"):
            v8 = torch.from_numpy(g[f"{name}__v8"]).view(torch.float8_e4m3fn)
            vsc = torch.from_numpy(g[f"{name}__vsc"])
            # the oracle's own slab store must reproduce the reference store first
            mine_v8, mine_sc = O.slab_v_store(c["cache_v"], c["cache_v"].shape[1], O.SCALE_CPU)
            assert np.array_equal(mine_v8.transpose(0, 2, 1, 3), g[f"{name}__v8"])
            assert np.array_equal(mine_sc, g[f"{name}__vsc"])
            out = O.block_causal_attention(c["q"], c["k"], c["v"], c["L"], c["key_valid"], c["cache_k"],
                                           v8, vsc)
        else:
            out = O.block_causal_attention(c["q"], c["k"], c["v"], c["L"], c["key_valid"], c["cache_k"],
                                           c["cache_v"])
        ref = torch.from_numpy(g[f"{name}__out"].view(np.int16)).view(torch.bfloat16).reshape(out.shape)
        d = (out.float() - ref.float()).abs().max().item()
        # both are fp32 math cast to bf16; per-head vs batched matmul may flip a bf16 ulp
        assert d <= 2e-3, (name, d)
        assert O.relf(out, ref) < 1e-3, name


def test_activation_quant_roundtrip_bound():
    """quantize_tensorwise semantics at a BASELINE-like shape: dequant error bound of
    e4m3 (half an e4m3 ulp relative, 2^-4) and saturation never triggers."""
    x = GI.outlier_activations(7, 256, 3072)
    q, s = O.quantize_act(x)
    deq = O.dequant(q, s)
    xf = x.float()
    err = (deq - xf).abs()
    assert (err <= xf.abs() * 2.0 ** -4 + s * 2.0 ** -9 + 1e-30).all()
    assert int(q.view(np.uint8).max()) != 0x7F
    assert O.amax(x) == xf.abs().max().item()


def test_e4m3_conversion_matches_torch_cast():
    bits = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    v = np.clip(bits[np.isfinite(bits)], -448, 448)[::3]
    t = torch.from_numpy(v.copy()).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.e4m3_from_f32_torch(v), t)


def test_fp8_linear_oracle_reference_bound():
    """The reference's own FP8Linear gate (tests/test_fp8.py:16-30): relF < 0.06 vs the
    unquantized fp32 product, here on the oracle's dequant path."""
    M, K, N = 128, 512, 256
    x = GI.randn_bf16(31, (M, K))
    w = GI.randn_bf16(32, (N, K), 0.02)
    xq, sx = O.quantize_act(x)
    wq, sw = O.quantize_weight(w)
    y = O.fp8_linear(xq, sx, wq, sw)
    ref = x.float() @ w.float().t()
    assert O.relf(y, ref) < 0.06


def test_exported_reference_attention_matches_golden(golden_dir):
    """qik.triton_attention.reference_block_causal_attention (the compatibility export
    of triton_attention.py:266-293) reproduces the reference function's outputs."""
    from qik.triton_attention import reference_block_causal_attention
    g = np.load(golden_dir / "attention.npz")
    for name, c in GI.attention_cases().items():
        if c.get("slab_fp8"):
            continue
        out = reference_block_causal_attention(c["q"], c["k"], c["v"], c["L"], c["key_valid"], c["cache_k"],
                                               c["cache_v"])
        ref = torch.from_numpy(g[f"{name}__out"].view(np.int16)).view(torch.bfloat16).reshape(out.shape)
        assert (out.float() - ref.float()).abs().max().item() <= 2e-3, name
        assert O.relf(out, ref) < 1e-3, name
