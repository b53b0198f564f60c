"""CPU tests of the e4m3 cache format (qik.quantize_offline) and the drop-in
installer (qik.patch).  The weight quantizer is the oracle here (the library's GPU
quantizer is checked byte for byte against it in test_gpu_quant.py)."""
import importlib
import sys
import textwrap

import torch

from oracle import oracle as O


def _oracle_quant(w):
    q, s = O.quantize_weight(w.cpu(), O.SCALE_CUDA)
    return torch.from_numpy(q).view(torch.float8_e4m3fn), torch.tensor([s], dtype=torch.float32)


class _Attn(torch.nn.Module):
    def __init__(self, d, bias):
        super().__init__()
        self.to_q = torch.nn.Linear(d, d, bias=bias, dtype=torch.bfloat16)
        self.to_k = torch.nn.Linear(d, d, bias=bias, dtype=torch.bfloat16)
        self.to_v = torch.nn.Linear(d, d, bias=bias, dtype=torch.bfloat16)
        self.to_out = torch.nn.ModuleList([torch.nn.Linear(d, d, bias=True, dtype=torch.bfloat16),
                                           torch.nn.Dropout(0.0)])


class _Mlp(torch.nn.Module):
    def __init__(self, d, h):
        super().__init__()
        self.gate_layer = torch.nn.Linear(d, h, bias=False, dtype=torch.bfloat16)
        self.proj = torch.nn.Linear(d, h, bias=False, dtype=torch.bfloat16)
        self.out = torch.nn.Linear(h, d, bias=False, dtype=torch.bfloat16)


class _Block(torch.nn.Module):
    def __init__(self, d=64, h=128, bias=True):
        super().__init__()
        self.attn = _Attn(d, bias)
        self.img_mlp = _Mlp(d, h)
        self.register_buffer("freqs", torch.ones(4))


def _model():
    torch.manual_seed(0)
    m = torch.nn.Module()
    m.transformer_blocks = torch.nn.ModuleList([_Block(), _Block()])
    m.proj_out = torch.nn.Linear(64, 32, bias=True, dtype=torch.bfloat16)
    return m


def test_fused_cache_keys_layout_and_roundtrip(tmp_path):
    from safetensors import safe_open
    from qik import quantize_offline as QO
    from qik.fp8 import FP8Linear
    m = _model()
    wq_ref = torch.cat([m.transformer_blocks[0].attn.to_q.weight, m.transformer_blocks[0].attn.to_k.weight,
                        m.transformer_blocks[0].attn.to_v.weight], 0).detach().clone()
    for blk in m.transformer_blocks:
        QO._fuse_block_linears(blk, quantize=_oracle_quant)
    QO._convert_module_fp8(m, quantize=_oracle_quant)
    path = tmp_path / "fp8_cache" / "transformer_fused_fp8.safetensors"
    n = QO.save_fp8_cache(m, str(path))
    with safe_open(str(path), framework="pt") as f:
        keys = set(f.keys())
        w = f.get_tensor("transformer_blocks.0.attn.fused_qkv.weight")
        s = f.get_tensor("transformer_blocks.0.attn.fused_qkv.weight_scale")
        assert w.dtype == torch.float8_e4m3fn and tuple(w.shape) == (192, 64)
        assert s.dtype == torch.float32 and tuple(s.shape) == (1,)
        assert f.get_tensor("transformer_blocks.0.attn.fused_qkv.bias").dtype == torch.bfloat16
    assert len(keys) == n
    assert not any(".freqs" in k for k in keys)
    assert not any("to_q" in k or "gate_layer" in k for k in keys)
    for must in ("transformer_blocks.1.img_mlp.fused_up.weight", "transformer_blocks.1.img_mlp.out.weight_scale",
                 "transformer_blocks.0.attn.to_out.0.weight", "proj_out.bias"):
        assert must in keys
    # one scale over the concatenated Q/K/V weight, bytes = the oracle's quantization of the cat
    q_exp, s_exp = _oracle_quant(wq_ref)
    assert torch.equal(w.view(torch.uint8), q_exp.view(torch.uint8)) and float(s) == float(s_exp)
    # loads into FP8Linear shells with assign=True (runtime.py:196-200)
    shell = FP8Linear(64, 192, bias=True)
    from safetensors.torch import load_file
    sd = load_file(str(path))
    missing, unexpected = shell.load_state_dict(
        {k.split("attn.fused_qkv.")[1]: v for k, v in sd.items() if k.startswith("transformer_blocks.0.attn.fused_qkv.")},
        strict=True, assign=True)
    assert not missing and not unexpected


def test_sd_for_save_dealiases():
    from qik import quantize_offline as QO
    m = torch.nn.Module()
    base = torch.arange(8, dtype=torch.float32)
    m.register_buffer("a", base)
    m.register_buffer("b", base[:4])
    sd = QO._sd_for_save(m)
    assert sd["a"].untyped_storage().data_ptr() != sd["b"].untyped_storage().data_ptr()


def test_patch_install_binds_qik_modules(tmp_path):
    from qik import patch
    pkg = tmp_path / "qwen_image_kernel"
    pkg.mkdir()
    (pkg / "__init__.py").write_text("")
    (pkg / "runtime.py").write_text(textwrap.dedent("""
        from .fp8 import FP8Linear
        from .kv_cache import ContiguousKVCache
        from .triton_attention import block_causal_flash_attention
    """))
    sys.path.insert(0, str(tmp_path))
    try:
        for k in [k for k in sys.modules if k.startswith("qwen_image_kernel")]:
            del sys.modules[k]
        patch.install()
        rt = importlib.import_module("qwen_image_kernel.runtime")
        import qik.fp8
        import qik.kv_cache
        import qik.triton_attention
        assert rt.FP8Linear is qik.fp8.FP8Linear
        assert rt.ContiguousKVCache is qik.kv_cache.ContiguousKVCache
        assert rt.block_causal_flash_attention is qik.triton_attention.block_causal_flash_attention
    finally:
        patch.uninstall()
        for k in [k for k in sys.modules if k.startswith("qwen_image_kernel")]:
            del sys.modules[k]
        sys.path.remove(str(tmp_path))


def test_fp8linear_buffers_match_reference_contract():
    from qik.fp8 import FP8Linear
    m = FP8Linear(256, 96, bias=True)
    assert m.weight.dtype == torch.float8_e4m3fn and tuple(m.weight.shape) == (96, 256)
    assert m.weight_scale.dtype == torch.float32 and tuple(m.weight_scale.shape) == (1,)
    assert m.bias.dtype == torch.bfloat16
    assert FP8Linear(256, 96).bias is None
    assert set(m.state_dict()) == {"weight", "weight_scale", "bias"}
