"""GPU parity: the tcgen05 FP8 GEMM (qik_fp8_gemm) and FP8Linear against the oracle.

Gates: the fp32 (pre-cast) GEMM output within
max-abs <= 2e-2 and relative Frobenius <= 5e-3 of the fp32 dequant oracle; the
bf16 production output within 1 bf16 ulp (+1e-6) of bf16(oracle) element-wise and
relF <= 5e-3.  Small-integer operands make fp32 accumulation exact, so those cases
must match bit for bit whatever the summation order.
"""
import numpy as np
import pytest
import torch

import golden_inputs as GI
from oracle import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
RELF = 5e-3


@pytest.fixture(scope="module")
def fp8():
    from qik import fp8 as F
    return F


def _e4m3_small_ints(seed: int, shape, lo=-4, hi=4) -> torch.Tensor:
    g = np.random.default_rng(seed)
    return torch.from_numpy(g.integers(lo, hi + 1, size=shape).astype(np.float32)).to(torch.float8_e4m3fn)


def _one():
    return torch.ones(1, dtype=torch.float32, device="cuda")


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (128, 256, 256), (256, 512, 384), (1, 16, 16),
                                   (2, 48, 32), (127, 272, 112), (129, 256, 144), (300, 3072, 3072),
                                   (4352, 256, 128), (512, 1024, 12288), (2, 18432, 3072), (256, 3072, 3072),
                                   (1000, 1040, 2048)])
def test_gemm_exact_small_ints(fp8, M, N, K):
    """Exact integer products: any layout/descriptor/tail error shows up as a mismatch."""
    a = _e4m3_small_ints(M * 7 + K, (M, K))
    b = _e4m3_small_ints(N * 3 + K, (N, K))
    ref = a.float() @ b.float().t()
    y = fp8.fp8_gemm(a.cuda(), _one(), b.cuda(), _one(), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), ref)


TILE_CFGS = [1, 2, 3, 4]   # qik._lib.GEMM_TILE_PAIR_256 .. GEMM_TILE_SINGLE_64


@pytest.mark.parametrize("cfg", TILE_CFGS)
@pytest.mark.parametrize("M,N,K", [(300, 736, 384), (600, 3072, 256), (4352, 3072, 512), (257, 1936, 128)])
def test_gemm_every_tile_config_exact(fp8, cfg, M, N, K):
    """Every tile configuration forced (qik_fp8_gemm_tiled), exact small-integer products,
    fp32 and bf16 outputs, partial row and column tiles and a 16-column chunk at the
    matrix edge (N = 736, 1936)."""
    a = _e4m3_small_ints(M + 5 * K, (M, K)).cuda()
    b = _e4m3_small_ints(N + 7 * K, (N, K)).cuda()
    ref = a.cpu().float() @ b.cpu().float().t()
    y = fp8.fp8_gemm(a, _one(), b, _one(), out_dtype=torch.float32, tile_cfg=cfg)
    yb = fp8.fp8_gemm(a, _one(), b, _one(), tile_cfg=cfg)
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), ref)
    assert torch.equal(yb.cpu(), ref.to(torch.bfloat16))


@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (2, 18432, 3072), (5, 736, 384), (16, 1936, 256), (2, 3072, 12288)])
def test_gemm_swapped_tiny_m_exact(fp8, M, N, K):
    """The tiny-M configuration (QIK_GEMM_TILE_SWAP_16, the default for M <= 16: weights
    as the tile rows, the activation rows as a 16-wide tile, the output stored
    transposed): exact small-integer products in fp32 and bf16, equal to the untransposed
    128 x 64 configuration, with bias, GELU and the amax output."""
    from qik import _lib as L
    a = _e4m3_small_ints(M + 13 * K, (M, K)).cuda()
    b = _e4m3_small_ints(N + 17 * K, (N, K)).cuda()
    ref = a.cpu().float() @ b.cpu().float().t()
    y = fp8.fp8_gemm(a, _one(), b, _one(), out_dtype=torch.float32, tile_cfg=L.GEMM_TILE_SWAP_16)
    yb = fp8.fp8_gemm(a, _one(), b, _one(), tile_cfg=L.GEMM_TILE_SWAP_16)
    y_auto = fp8.fp8_gemm(a, _one(), b, _one())  # the default for M <= 16
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), ref)
    assert torch.equal(yb.cpu(), ref.to(torch.bfloat16))
    assert torch.equal(y_auto.cpu(), ref.to(torch.bfloat16))
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(N)) * 4).to(torch.bfloat16).cuda()
    for epi in (L.EPI_SCALE, L.EPI_GELU_TANH):
        am_s, am_u = (torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(2))
        ys = fp8.fp8_gemm(a, _one(), b, _one(), bias=bias, epilogue=epi, amax_out=am_s,
                          tile_cfg=L.GEMM_TILE_SWAP_16)
        yu = fp8.fp8_gemm(a, _one(), b, _one(), bias=bias, epilogue=epi, amax_out=am_u,
                          tile_cfg=L.GEMM_TILE_SINGLE_64)
        torch.cuda.synchronize()
        assert torch.equal(ys, yu), epi
        assert int(am_s.item()) == int(am_u.item()) == int(ys.float().abs().max().view(torch.int32).item())


def test_gemm_swapped_tiny_m_rejects_larger_m(fp8):
    from qik import _lib as L
    a = torch.zeros(17, 128, dtype=torch.float8_e4m3fn, device="cuda")
    b = torch.zeros(128, 128, dtype=torch.float8_e4m3fn, device="cuda")
    with pytest.raises(L.QikError, match="M <= 16"):
        fp8.fp8_gemm(a, _one(), b, _one(), tile_cfg=L.GEMM_TILE_SWAP_16)


@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (300, 512, 256), (513, 12288, 3072), (4352, 24576, 3072)])
def test_gemm_swiglu_epilogue_matches_gemm_then_swiglu(fp8, M, N, K):
    """QIK_EPI_SWIGLU (the fused gate / up projection with silu(gate) * up applied in the
    epilogue, the gate / up output never written) is bit-identical, values and amax, to
    the plain GEMM on the same CTA-pair tiles followed by the SwiGLU kernel on its two
    halves; with and without bias, ragged M (a partial last 256-row tile)."""
    from qik import _lib as L
    from qik.triton_fused import fused_swiglu
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    wq, sw = fp8.quantize_weight_tensorwise(torch.randn(N, K, device="cuda", generator=g) * 0.02)
    xq, sx = fp8.quantize_tensorwise(torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16))
    bias = (torch.randn(N, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    for b in (None, bias):
        gu = fp8.fp8_gemm(xq, sx, wq, sw, b, tile_cfg=L.GEMM_TILE_PAIR_256)
        am_ref, am = (torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(2))
        ref = fused_swiglu(*gu.chunk(2, dim=-1), amax_out=am_ref)
        y = fp8.fp8_gemm(xq, sx, wq, sw, b, epilogue=L.EPI_SWIGLU, amax_out=am)
        torch.cuda.synchronize()
        assert y.shape == (M, N // 2)
        assert torch.equal(y, ref), b is None
        assert int(am.item()) == int(am_ref.item()) == int(y.float().abs().max().view(torch.int32).item())


@pytest.mark.parametrize("B,S,H,rope", [(2, 4352, 24, True), (1, 300, 2, True), (3, 77, 3, True), (1, 256, 4, False)])
def test_qkv_rms_rope_epilogue_matches_gemm_then_rms_rope(fp8, B, S, H, rope):
    """qik_fp8_gemm_qkv_rms_rope (the fused QKV linear with the per-head RMSNorm + RoPE of
    q and k in its epilogue) is bit-identical to the plain GEMM on the same CTA-pair tiles
    followed by the RMSNorm + RoPE kernel on its q and k views, its v columns equal to the
    GEMM's: the configs[2] shape, ragged M (a partial last 256-row tile), an odd head
    count (a tile holding the last q head and the first k head, a partial last v tile),
    and no rotary table (the identity rotation)."""
    from qik import _lib as L
    from qik.triton_fused import fused_rms_norm_rope
    D, K = 128, 384 if H < 8 else 3072
    g = torch.Generator(device="cuda").manual_seed(B * S + H)
    lin = fp8.FP8Linear(K, 3 * H * D, bias=True).cuda()
    wq8, sw = fp8.quantize_weight_tensorwise(torch.randn(3 * H * D, K, device="cuda", generator=g) * 0.05)
    lin.weight.copy_(wq8)
    lin.weight_scale.copy_(sw)
    lin.bias.copy_((torch.randn(3 * H * D, device="cuda", generator=g) * 0.3).to(torch.bfloat16))
    xq, sx = fp8.quantize_tensorwise(torch.randn(B * S, K, device="cuda", generator=g).to(torch.bfloat16))
    xq = xq.view(B, S, K)
    w_q = 1.0 + 0.2 * torch.randn(D, device="cuda", generator=g)
    w_k = 1.0 + 0.2 * torch.randn(D, device="cuda", generator=g)
    freqs = None
    if rope:
        inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device="cuda").float() / D))
        freqs = torch.polar(torch.ones(S, D // 2, device="cuda"),
                            torch.outer(torch.arange(S, device="cuda").float(), inv))
    out = lin.forward_qkv_rms_rope_e4m3(xq, sx, H, w_q, w_k, freqs, 1e-6)
    plain = fp8.fp8_gemm(xq.view(B * S, K), sx, lin.weight, lin.weight_scale, lin.bias,
                         tile_cfg=L.GEMM_TILE_PAIR_256).view(B, S, 3 * H, D)
    q, k, v = plain.chunk(3, dim=-2)
    ref_q = fused_rms_norm_rope(q, w_q, freqs, 1e-6)
    ref_k = fused_rms_norm_rope(k, w_k, freqs, 1e-6)
    torch.cuda.synchronize()
    oq, ok, ov = out.chunk(3, dim=-2)
    assert out.shape == (B, S, 3 * H, D)
    assert torch.equal(oq, ref_q), "q"
    assert torch.equal(ok, ref_k), "k"
    assert torch.equal(ov, v), "v"


@pytest.mark.parametrize("B,S,K,N,masked", [(2, 4352, 3072, 3072, False), (2, 4352, 6144, 3072, True),
                                            (1, 77, 256, 256, True), (3, 50, 384, 144, False)])
def test_gate_residual_epilogue_matches_linear_then_gate_residual(fp8, B, S, K, N, masked):
    """qik_fp8_gemm_gate_residual (an FP8 linear with the DiT block's gated residual in
    its epilogue) is bit-identical to the linear followed by the gated-residual kernel:
    the configs[2] out-projection and down-projection shapes (with the t = 0 modulation
    rows of a target mask), and small ragged shapes (partial tiles, a partial column
    chunk, a bias)."""
    from qik.triton_fused import fused_gate_residual, gate_table
    g = torch.Generator(device="cuda").manual_seed(B * S + K + N)
    lin = fp8.FP8Linear(K, N, bias=True).cuda()
    wq8, sw = fp8.quantize_weight_tensorwise(torch.randn(N, K, device="cuda", generator=g) * 0.03)
    lin.weight.copy_(wq8)
    lin.weight_scale.copy_(sw)
    lin.bias.copy_((torch.randn(N, device="cuda", generator=g) * 0.2).to(torch.bfloat16))
    x = torch.randn(B, S, K, device="cuda", generator=g).to(torch.bfloat16)
    res = (torch.randn(B, S, N, device="cuda", generator=g) * 2).to(torch.bfloat16)
    mod = (torch.randn(2 * B, 4 * N, device="cuda", generator=g) * 0.8).to(torch.bfloat16)
    mask = (torch.rand(S, device="cuda", generator=g) < 0.7) if masked else None
    amax = fp8.amax_bits(x.reshape(-1, K))
    for off in (N, 3 * N):
        table = gate_table(mod, off, 2 * B if masked else B, N)
        out = lin.forward_gate_residual(x, amax, res, table, mask)
        ref = fused_gate_residual(res, lin.forward_from_amax(x, amax), mod, off, mask)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), off
    # the table is bf16(tanh(gate)) (fp32 tanh, one rounding)
    t = gate_table(mod, N, 2 * B, N).float()
    r = torch.tanh(mod[:, N:2 * N].float())
    assert (t - r).abs().max().item() <= 2.0 ** -8


def test_qkv_rms_rope_rejects(fp8):
    lin = fp8.FP8Linear(256, 3 * 2 * 64).cuda()
    xq = torch.zeros(1, 16, 256, dtype=torch.float8_e4m3fn, device="cuda")
    w = torch.ones(128, device="cuda")
    with pytest.raises(ValueError, match="heads"):
        lin.forward_qkv_rms_rope_e4m3(xq, _one(), 2, w, w, None, 1e-6)


def test_gemm_swiglu_epilogue_rejects(fp8):
    from qik import _lib as L
    a = torch.zeros(64, 128, dtype=torch.float8_e4m3fn, device="cuda")
    b = torch.zeros(384, 128, dtype=torch.float8_e4m3fn, device="cuda")
    with pytest.raises(L.QikError, match="N % 256 == 0"):
        fp8.fp8_gemm(a, _one(), b, _one(), epilogue=L.EPI_SWIGLU)
    b = torch.zeros(512, 128, dtype=torch.float8_e4m3fn, device="cuda")
    with pytest.raises(L.QikError, match="CTA-pair tiles only"):
        fp8.fp8_gemm(a, _one(), b, _one(), epilogue=L.EPI_SWIGLU, tile_cfg=L.GEMM_TILE_SINGLE_128)
    with pytest.raises(L.QikError, match="BF16 output"):
        fp8.fp8_gemm(a, _one(), b, _one(), epilogue=L.EPI_SWIGLU, out_dtype=torch.float32)


@pytest.mark.parametrize("cfg", [1, 3])
@pytest.mark.parametrize("raster", [1, 3, 16, 255])
def test_gemm_raster_groups_exact(fp8, cfg, raster):
    """The tile raster (QIK_GEMM_RASTER(g): groups of g row tiles walked column by
    column) only reorders tiles: exact small-integer products for group sizes that
    divide the row tiles unevenly (4352 rows = 17 pair tiles, 34 single tiles), equal
    them, and exceed them."""
    M, N, K = 4352, 1280, 256
    a = _e4m3_small_ints(M + 3 * K, (M, K)).cuda()
    b = _e4m3_small_ints(N + 11 * K, (N, K)).cuda()
    ref = a.cpu().float() @ b.cpu().float().t()
    y = fp8.fp8_gemm(a, _one(), b, _one(), out_dtype=torch.float32, tile_cfg=cfg | (raster << 8))
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), ref)


def test_gemm_deterministic(fp8):
    """Repeated launches give bitwise-identical results (fixed schedule, no atomics)."""
    M, N, K = 640, 768, 6144
    a = _e4m3_small_ints(11, (M, K)).cuda()
    b = _e4m3_small_ints(12, (N, K)).cuda()
    x = GI.randn_bf16(13, (M, K)).cuda()
    xq, sx = fp8.quantize_tensorwise(x)
    y1 = fp8.fp8_gemm(xq, sx, b, _one())
    y2 = fp8.fp8_gemm(xq, sx, b, _one())
    assert torch.equal(y1, y2)
    assert torch.equal(fp8.fp8_gemm(a, _one(), b, _one(), out_dtype=torch.float32).cpu(),
                       a.cpu().float() @ b.cpu().float().t())


def test_gemm_scales_and_bias(fp8):
    M, N, K = 200, 320, 256
    a = _e4m3_small_ints(1, (M, K))
    b = _e4m3_small_ints(2, (N, K))
    bias = GI.randn_bf16(3, (N,))
    sa = torch.tensor([0.25], device="cuda")
    sb = torch.tensor([0.5], device="cuda")
    y = fp8.fp8_gemm(a.cuda(), sa, b.cuda(), sb, bias=bias.cuda(), out_dtype=torch.float32)
    ref = (a.float() @ b.float().t()) * 0.125 + bias.float()
    assert torch.allclose(y.cpu(), ref, rtol=0, atol=1e-5)
    yb = fp8.fp8_gemm(a.cuda(), sa, b.cuda(), sb, bias=bias.cuda())
    assert torch.equal(yb.cpu(), ref.to(torch.bfloat16))


def _linear_case(seed, M, N, K, outliers=True):
    x = GI.outlier_activations(seed, M, K) if outliers else GI.randn_bf16(seed, (M, K))
    w = GI.randn_bf16(seed + 1, (N, K), 0.02)
    return x, w


@pytest.mark.parametrize("M,N,K", [(4352, 3072, 3072), (256, 9216, 3072), (1024, 12288, 3072),
                                   (256, 3072, 12288), (2, 18432, 3072)])
def test_fp8_linear_parity(fp8, M, N, K):
    """BASELINE config 1 (and sweep shapes): dynamic activation quant + FP8 GEMM vs the
    fp32 dequant path of the reference, on the same quantized operands."""
    x, w = _linear_case(M + N, M, N, K)
    lin = fp8.FP8Linear(K, N).cuda()
    wq, sw = fp8.quantize_weight_tensorwise(w.cuda())
    lin.weight.copy_(wq)
    lin.weight_scale.copy_(sw)
    xd = x.cuda()
    y32 = lin.forward_fp32(xd)
    y16 = lin(xd)
    torch.cuda.synchronize()
    xq, sx = fp8.quantize_tensorwise(xd)
    ref = O.fp8_linear(xq.cpu(), float(sx.item()), wq.cpu(), float(sw.item()))
    d = (y32.cpu() - ref).abs().max().item()
    r = O.relf(y32.cpu(), ref)
    print(f"M={M} N={N} K={K}: fp32 max-abs {d:.3e} relF {r:.3e} max|ref| {ref.abs().max().item():.2f}")
    assert d <= MAX_ABS, d
    assert r <= RELF
    # the bf16 output is the round-to-nearest of the kernel's own fp32 result ...
    assert torch.equal(y16.cpu(), y32.cpu().to(torch.bfloat16))
    # ... and within the gates of the reference's bf16 output (whose own bf16 cast
    # already costs up to half a bf16 ulp of |y|)
    assert O.relf(y16.cpu(), ref) <= RELF
    assert ((y16.cpu().float() - ref).abs() <= MAX_ABS + 0.5 * O.bf16_ulp(ref)).all()
    # the reference's own gate vs the unquantized product (tests/test_fp8.py:27-28)
    assert O.relf(y16.cpu(), x.float() @ w.float().t()) < 0.06


CFG5_SHAPES = [(M, N) for N in (3072, 9216, 12288, 18432) for M in (256, 1024, 4352, 9472, 16384)]


@pytest.mark.parametrize("M,N", CFG5_SHAPES)
def test_gemm_cfg5_all_shapes(fp8, M, N):
    """Every configs[4] shape (K = 3072): the fp32 (pre-cast) GEMM output of the
    product's own e4m3 operands against the fp32 dequant product computed by plain
    PyTorch on the GPU (TF32 off: an fp32 reference of the same op), max-abs <= 2e-2 and
    relF <= 5e-3; the bf16 output is the kernel's fp32 result rounded.  The CPU oracle
    pins the same computation at the configs[1] shape above."""
    K = 3072
    g = torch.Generator(device="cuda").manual_seed(M * 31 + N)
    x = torch.randn(M, K, device="cuda", generator=g)
    x[:, :8] *= 20.0
    w = torch.randn(N, K, device="cuda", generator=g) * 0.02
    xq, sx = fp8.quantize_tensorwise(x.to(torch.bfloat16))
    wq, sw = fp8.quantize_weight_tensorwise(w.to(torch.bfloat16))
    y32 = fp8.fp8_gemm(xq, sx, wq, sw, out_dtype=torch.float32)
    y16 = fp8.fp8_gemm(xq, sx, wq, sw)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = (xq.float() * sx) @ (wq.float() * sw).t()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    d = (y32 - ref).abs().max().item()
    r = ((y32 - ref).norm() / ref.norm()).item()
    print(f"M={M} N={N}: fp32 max-abs {d:.3e} relF {r:.3e}")
    assert d <= MAX_ABS and r <= RELF
    assert torch.equal(y16, y32.to(torch.bfloat16))


def test_fp8_linear_bias_and_leading_dims(fp8):
    x = GI.randn_bf16(70, (2, 37, 512))
    w = GI.randn_bf16(71, (384, 512), 0.02)
    b = GI.randn_bf16(72, (384,), 0.1)
    lin = torch.nn.Linear(512, 384, bias=True, dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(b)
    f = fp8.FP8Linear.from_linear(lin.cuda())
    y = f(x.cuda())
    assert y.shape == (2, 37, 384) and y.dtype == torch.bfloat16
    xq, sx = fp8.quantize_tensorwise(x.cuda().reshape(-1, 512))
    ref = O.fp8_linear(xq.cpu(), float(sx.item()), f.weight.cpu(), float(f.weight_scale.item()), b)
    assert O.relf(y.reshape(-1, 384).cpu(), ref) <= RELF


def test_fp8_linear_skinny_k_dequant_path(fp8):
    """in_features < 256 follows the reference's dequantized bf16 linear."""
    lin = torch.nn.Linear(64, 128, bias=False, dtype=torch.bfloat16).cuda()
    f = fp8.FP8Linear.from_linear(lin)
    x = GI.randn_bf16(80, (10, 64)).cuda()
    w = (f.weight.to(torch.bfloat16).float() * f.weight_scale).to(torch.bfloat16)
    assert torch.equal(f(x), torch.nn.functional.linear(x, w))


def test_gelu_epilogue_and_amax(fp8):
    """GEMM1 of the FFN: y = gelu_tanh(bf16(acc*s)), amax of the bf16 output."""
    M, N, K = 512, 1024, 3072
    x, w = _linear_case(5, M, N, K)
    xq, sx = fp8.quantize_tensorwise(x.cuda())
    wq, sw = fp8.quantize_weight_tensorwise(w.cuda())
    amax = torch.zeros(1, dtype=torch.int32, device="cuda")
    from qik import _lib as L
    h = fp8.fp8_gemm(xq, sx, wq, sw, epilogue=L.EPI_GELU_TANH, amax_out=amax)
    plain = fp8.fp8_gemm(xq, sx, wq, sw)
    torch.cuda.synchronize()
    # GELU-tanh evaluated in fp64 on the kernel's own bf16 linear output, rounded to
    # bf16; torch's fp32 form is also accepted within an absolute 1e-6 (it loses
    # relative accuracy where 1 + tanh(u) cancels, x < -5).
    xd = plain.double().cpu()
    ref64 = 0.5 * xd * (1.0 + torch.tanh(0.7978845608028654 * (xd + 0.044715 * xd ** 3)))
    ref_h = ref64.to(torch.bfloat16).float()
    d = (h.cpu().float() - ref_h).abs()
    assert (d <= O.bf16_ulp(ref_h) + 1e-6).all(), d.max().item()
    torch_h = torch.nn.functional.gelu(plain.float(), approximate="tanh").to(torch.bfloat16).cpu().float()
    assert ((h.cpu().float() - torch_h).abs() <= O.bf16_ulp(torch_h) + 1e-6).all()
    got_amax = np.array([amax.item()], dtype=np.int32).view(np.float32)[0]
    assert got_amax == h.float().abs().max().item()


def test_ffn_pair_parity(fp8):
    """BASELINE config 2 at reduced M: FFN 3072 -> 12288 (GELU-tanh) -> 3072, both FP8,
    hidden re-quantized dynamically; vs the fp32 dequant oracle on the same operands."""
    M, K, Hd = 512, 3072, 12288
    x = GI.outlier_activations(90, M, K)
    up = fp8.FP8Linear(K, Hd).cuda()
    down = fp8.FP8Linear(Hd, K).cuda()
    for lin, seed in ((up, 91), (down, 92)):
        wq, sw = fp8.quantize_weight_tensorwise(GI.randn_bf16(seed, (lin.out_features, lin.in_features), 0.02).cuda())
        lin.weight.copy_(wq)
        lin.weight_scale.copy_(sw)
    y = fp8.fp8_ffn_gelu(x.cuda(), up, down)
    torch.cuda.synchronize()
    # oracle: same dynamic quantizations, fp32 dequant GEMMs, bf16 rounding points of
    # the reference module chain (linear -> bf16, gelu -> bf16, linear -> bf16)
    xq, sx = O.quantize_act(x)
    y1 = O.fp8_linear(xq, sx, up.weight.cpu(), float(up.weight_scale.item())).to(torch.bfloat16)
    h = O.gelu_tanh(y1)
    hq, sh = O.quantize_act(h, inv=O.act_reciprocal(O.compute_scale(h)))
    ref = O.fp8_linear(hq, sh, down.weight.cpu(), float(down.weight_scale.item()))
    assert (y.cpu().float() - ref).abs().max().item() <= 5 * MAX_ABS
    assert O.relf(y.cpu(), ref) <= RELF
    # max|x| supplied by x's producer (qik_fp8_ffn_from_amax): the chain starts at the
    # pack of x and gives the same bytes
    xd = x.cuda()
    amax = torch.tensor([int(np.array([xd.float().abs().max().item()], np.float32).view(np.int32)[0])],
                        dtype=torch.int32, device="cuda")
    y2 = fp8.fp8_ffn_gelu(xd, up, down, x_amax=amax)
    torch.cuda.synchronize()
    assert torch.equal(y2, y)


def test_ffn_pair_from_layer_norm_amax(fp8):
    """The DiT block's second half: LayerNorm + modulate accumulating max|out|, fed to
    the FFN chain as its input amax -- identical to the chain computing it itself."""
    from qik.triton_fused import fused_layer_norm_modulate
    M, K, Hd = 384, 3072, 12288
    h = GI.randn_bf16(95, (1, M, K)).cuda()
    mod = GI.randn_bf16(96, (1, 4 * K), 0.2).cuda()
    up = fp8.FP8Linear(K, Hd).cuda()
    down = fp8.FP8Linear(Hd, K).cuda()
    for lin, seed in ((up, 97), (down, 98)):
        wq, sw = fp8.quantize_weight_tensorwise(GI.randn_bf16(seed, (lin.out_features, lin.in_features), 0.02).cuda())
        lin.weight.copy_(wq)
        lin.weight_scale.copy_(sw)
    amax = torch.zeros(1, dtype=torch.int32, device="cuda")
    hm = fused_layer_norm_modulate(h, mod, 2 * K, 4 * K, None, 1e-6, amax_out=amax)
    y_fused = fp8.fp8_ffn_gelu(hm.reshape(M, K), up, down, x_amax=amax)
    y_plain = fp8.fp8_ffn_gelu(hm.reshape(M, K), up, down)
    torch.cuda.synchronize()
    assert torch.equal(y_fused, y_plain)


def test_ffn_pair_from_layer_norm_e4m3(fp8):
    """The DiT block's second half with the LayerNorm emitting the FFN's e4m3 input
    (qik_layer_norm_modulate_e4m3 -> qik_fp8_ffn_e4m3): identical to the chain on the
    bf16 LayerNorm output."""
    from qik.triton_fused import fused_layer_norm_modulate, fused_layer_norm_modulate_e4m3
    M, K, Hd = 384, 3072, 12288
    h = GI.randn_bf16(99, (1, M, K)).cuda()
    mod = GI.randn_bf16(100, (1, 4 * K), 0.2).cuda()
    up = fp8.FP8Linear(K, Hd).cuda()
    down = fp8.FP8Linear(Hd, K).cuda()
    for lin, seed in ((up, 101), (down, 102)):
        wq, sw = fp8.quantize_weight_tensorwise(GI.randn_bf16(seed, (lin.out_features, lin.in_features), 0.02).cuda())
        lin.weight.copy_(wq)
        lin.weight_scale.copy_(sw)
    hq, hs = fused_layer_norm_modulate_e4m3(h, mod, 2 * K, 4 * K, None, 1e-6)
    y_e4m3 = fp8.fp8_ffn_gelu(hq.reshape(M, K), up, down, x_scale=hs)
    y_plain = fp8.fp8_ffn_gelu(fused_layer_norm_modulate(h, mod, 2 * K, 4 * K, None, 1e-6).reshape(M, K), up, down)
    torch.cuda.synchronize()
    assert torch.equal(y_e4m3, y_plain)
    # an FP8 linear handed the same codes and scale (FP8Linear.forward_e4m3) equals forward
    assert torch.equal(up.forward_e4m3(hq, hs), up(fused_layer_norm_modulate(h, mod, 2 * K, 4 * K, None, 1e-6)))


def test_gemm_rejects_bad_shapes(fp8):
    from qik import _lib as L
    a = torch.zeros(4, 24, dtype=torch.float8_e4m3fn, device="cuda")
    b = torch.zeros(32, 24, dtype=torch.float8_e4m3fn, device="cuda")
    with pytest.raises(L.QikError):
        fp8.fp8_gemm(a, _one(), b, _one())                               # K % 16 != 0
    a = torch.zeros(4, 32, dtype=torch.float8_e4m3fn, device="cuda")
    b = torch.zeros(40, 32, dtype=torch.float8_e4m3fn, device="cuda")
    with pytest.raises(L.QikError):
        fp8.fp8_gemm(a, _one(), b, _one())                               # N % 16 != 0
