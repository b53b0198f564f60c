"""qik.host_pipeline.HostPipeline: the FP8 FFN pair over pinned host batches, with the
copies of neighbouring batches overlapping the kernels, gives bit-identical results to
calling the FFN on each batch directly (the pipeline moves only copies), through slot
reuse at depths 1-3; unpinned host buffers are refused."""
import pytest
import torch

import golden_inputs as GI

pytestmark = pytest.mark.gpu

M, K, HID = 384, 512, 1536


@pytest.fixture(scope="module")
def ffn():
    from qik import fp8 as F
    dev = torch.device("cuda", 0)
    up = F.FP8Linear(K, HID).to(dev)
    down = F.FP8Linear(HID, K).to(dev)
    for lin, seed in ((up, 601), (down, 602)):
        wq, sw = F.quantize_weight_tensorwise(GI.randn_bf16(seed, (lin.out_features, lin.in_features), 0.04).to(dev))
        lin.weight.copy_(wq)
        lin.weight_scale.copy_(sw)
    return F, up, down


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_pipeline_matches_direct_calls(ffn, depth):
    from qik.host_pipeline import HostPipeline
    F, up, down = ffn
    xs = [GI.outlier_activations(610 + i, M, K).pin_memory() for i in range(7)]
    ys = [torch.empty(M, K, dtype=torch.bfloat16).pin_memory() for _ in xs]
    pipe = HostPipeline(lambda xd, yd: F.fp8_ffn_gelu(xd, up, down, out=yd), (M, K), (M, K),
                        device="cuda:0", depth=depth)
    events = [pipe.submit(x, y) for x, y in zip(xs, ys)]
    events[-1].synchronize()
    pipe.synchronize()
    for i, (x, y) in enumerate(zip(xs, ys)):
        ref = F.fp8_ffn_gelu(x.cuda(), up, down).cpu()
        assert torch.equal(y, ref), f"batch {i} differs from the direct call"


def test_pipeline_refuses_unpinned_buffers(ffn):
    from qik.host_pipeline import HostPipeline
    F, up, down = ffn
    pipe = HostPipeline(lambda xd, yd: F.fp8_ffn_gelu(xd, up, down, out=yd), (M, K), (M, K), device="cuda:0")
    with pytest.raises(ValueError, match="pinned"):
        pipe.submit(torch.zeros(M, K, dtype=torch.bfloat16), torch.zeros(M, K, dtype=torch.bfloat16).pin_memory())
    with pytest.raises(ValueError, match="contiguous"):
        pipe.submit(torch.zeros(M, K + 8, dtype=torch.bfloat16).pin_memory(),
                    torch.zeros(M, K, dtype=torch.bfloat16).pin_memory())
