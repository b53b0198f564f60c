"""The e4m3 cache written with the library's GPU weight quantizer (qik_quantize_weight,
the path quantize_offline.py:19-26 takes on a CUDA machine) is byte-identical to the
same cache written with the oracle's CUDA-form quantizer; the CPU test
test_format_and_patch.py pins the writer itself to the reference's own file."""
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _oracle_cuda_form(w):
    q, s = O.quantize_weight(w.cpu(), O.SCALE_CUDA)
    return torch.from_numpy(q).view(torch.float8_e4m3fn), torch.tensor([s], dtype=torch.float32)


def test_cache_written_on_gpu_matches_oracle(tmp_path):
    import golden_inputs as GI
    from qik import quantize_offline as QO
    a, b = GI.standin_dit(d=256, hidden=384), GI.standin_dit(d=256, hidden=384)
    QO.convert_model_fp8(a)                                   # product quantizer (GPU)
    QO.convert_model_fp8(b, quantize=_oracle_cuda_form)
    QO.write_fp8_cache(a, str(tmp_path / "gpu.safetensors"))
    QO.write_fp8_cache(b, str(tmp_path / "oracle.safetensors"))
    assert (tmp_path / "gpu.safetensors").read_bytes() == (tmp_path / "oracle.safetensors").read_bytes()
    # and the GPU-quantized cache loads back into a meta skeleton, forward-ready
    with torch.device("meta"):
        m = GI.standin_dit(d=256, hidden=384, fill=False)
    QO.load_fp8_cache(m, str(tmp_path / "gpu.safetensors"))
    lin = m.transformer_blocks[0].attn.fused_qkv.cuda()     # (time_embed.freqs stays on meta: dropped)
    x = GI.randn_bf16(77, (2, 40, 256)).cuda()
    y = lin(x)
    assert y.shape == (2, 40, 768) and torch.isfinite(y.float()).all()
