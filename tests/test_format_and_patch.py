"""CPU tests of the e4m3 cache format (qik.quantize_offline) against a file the
reference's own writer produced (tests/golden/fp8_cache_ref.safetensors), and of the
drop-in installer (qik.patch).  The weight quantizer is the oracle here (the library's
GPU quantizer is checked byte for byte against it in test_gpu_quant.py)."""
import importlib
import sys
import textwrap

import pytest
import torch

from oracle import oracle as O


GOLDEN_CACHE = "fp8_cache_ref.safetensors"


def _oracle_quant(mode):
    def quant(w):
        q, s = O.quantize_weight(w.cpu(), mode)
        return torch.from_numpy(q).view(torch.float8_e4m3fn), torch.tensor([s], dtype=torch.float32)
    return quant


def test_writer_reproduces_reference_cache_bytes(tmp_path, golden_dir):
    """The reference's writer (quantize_offline.py:29-131, run on CPU by
    tests/golden/make_golden.py over golden_inputs.standin_dit) and this writer, fed
    the same tree and the same (CPU-form) weight quantizer, produce the same file
    byte for byte."""
    import golden_inputs as GI
    from qik import quantize_offline as QO
    m = GI.standin_dit()
    QO.convert_model_fp8(m, quantize=_oracle_quant(O.SCALE_CPU))
    path = tmp_path / "fp8_cache" / "transformer_fused_fp8.safetensors"
    n = QO.write_fp8_cache(m, str(path))
    mine, ref = path.read_bytes(), (golden_dir / GOLDEN_CACHE).read_bytes()
    assert len(mine) == len(ref) and mine == ref
    assert n == 38


def test_reference_cache_layout(golden_dir):
    """Key schema of the reference-written file: fused groups with one scale, the
    members absent, ``.freqs`` dropped, e4m3 / f32 / bf16 dtypes."""
    import golden_inputs as GI
    from safetensors.torch import load_file
    sd = load_file(str(golden_dir / GOLDEN_CACHE))
    assert not any(".freqs" in k for k in sd)
    assert not any(f".{m}." in k for k in sd for m in ("to_q", "to_k", "to_v", "gate_layer", "proj"))
    for i in range(2):
        w = sd[f"transformer_blocks.{i}.attn.fused_qkv.weight"]
        assert w.dtype == torch.float8_e4m3fn and tuple(w.shape) == (192, 64)
        assert sd[f"transformer_blocks.{i}.attn.fused_qkv.weight_scale"].shape == (1,)
        assert sd[f"transformer_blocks.{i}.attn.fused_qkv.bias"].dtype == torch.bfloat16
        assert tuple(sd[f"transformer_blocks.{i}.img_mlp.fused_up.weight"].shape) == (192, 64)
        assert f"transformer_blocks.{i}.img_mlp.fused_up.bias" not in sd
    assert sd["pos_table_head"].shape == (3, 4)
    # one scale over the concatenated Q/K/V weights of block 0, in the oracle's CPU form
    src = GI.standin_dit()
    a = src.transformer_blocks[0].attn
    q_exp, s_exp = _oracle_quant(O.SCALE_CPU)(torch.cat([a.to_q.weight, a.to_k.weight, a.to_v.weight]).detach())
    assert torch.equal(sd["transformer_blocks.0.attn.fused_qkv.weight"].view(torch.uint8), q_exp.view(torch.uint8))
    assert sd["transformer_blocks.0.attn.fused_qkv.weight_scale"].item() == s_exp.item()


def test_reader_loads_reference_cache(golden_dir):
    """A skeleton built on the meta device takes the reference-written file through the
    shells (runtime.py:76-123,196-200): no missing or unexpected key, nothing left on
    the meta device, fused shells where the file has fused keys."""
    import golden_inputs as GI
    from safetensors.torch import load_file
    from qik import quantize_offline as QO
    from qik.fp8 import FP8Linear
    with torch.device("meta"):
        m = GI.standin_dit(fill=False)
    QO.load_fp8_cache(m, str(golden_dir / GOLDEN_CACHE))
    sd = load_file(str(golden_dir / GOLDEN_CACHE))
    blk = m.transformer_blocks[1]
    assert isinstance(blk.attn.fused_qkv, FP8Linear) and isinstance(blk.attn.to_q, torch.nn.Identity)
    assert isinstance(blk.img_mlp.fused_up, FP8Linear) and blk.img_mlp.fused_up.bias is None
    assert isinstance(m.img_in, FP8Linear) and isinstance(blk.attn.to_out[0], FP8Linear)
    got = m.state_dict()
    for k, t in sd.items():
        assert torch.equal(got[k].view(torch.uint8), t.view(torch.uint8)), k


def test_reader_rejects_mismatched_cache(golden_dir):
    import golden_inputs as GI
    from safetensors.torch import load_file
    from qik import quantize_offline as QO
    sd = load_file(str(golden_dir / GOLDEN_CACHE))
    broken = dict(sd)
    del broken["proj_out.weight_scale"]
    with torch.device("meta"):
        m = GI.standin_dit(fill=False)
    with pytest.raises(ValueError, match="missing"):
        QO.load_fp8_cache(m, broken)
    extra = dict(sd)
    extra["proj_out.stray"] = torch.zeros(1)
    with torch.device("meta"):
        m = GI.standin_dit(fill=False)
    with pytest.raises(ValueError, match="unexpected"):
        QO.load_fp8_cache(m, extra)


def test_cache_state_dict_copies_out_shared_storage():
    from qik import quantize_offline as QO
    m = torch.nn.Module()
    base = torch.arange(8, dtype=torch.float32)
    m.register_buffer("a", base)
    m.register_buffer("b", base[:4])
    m.register_buffer("c", torch.ones(3))
    sd = QO.cache_state_dict(m)
    assert sd["a"].untyped_storage().data_ptr() != sd["b"].untyped_storage().data_ptr()
    assert sd["c"].data_ptr() == m.c.data_ptr()          # sole owner of a whole storage: not copied
    assert torch.equal(sd["b"], base[:4])


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
