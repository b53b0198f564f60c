"""GPU parity: the tcgen05 block-causal attention (qik_block_causal_attention) vs the
CPU oracle and the reference's own golden outputs.

Gate: max-abs <= 2e-2 and relative Frobenius <= 5e-3
against the fp32 reference path (oracle.block_causal_attention, which restates
reference_block_causal_attention, triton_attention.py:266-293, with the kernel's
fp8 slab-V dequant).  The reference's own test gate is max-abs < 2e-2
(tests/test_attention.py:132).
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
def attn():
    from qik import triton_attention as A
    return A


def _cuda(t):
    return None if t is None else t.cuda()


def _check(out, ref32, heads=None, tag=""):
    o = out.cpu().float()
    if heads is not None:
        o = o[:, :, heads]
        ref32 = ref32[:, :, heads]
    d = (o - ref32).abs().max().item()
    r = O.relf(o, ref32)
    print(f"{tag}: max-abs {d:.3e} relF {r:.3e}")
    assert d <= MAX_ABS, (tag, d)
    assert r <= RELF, (tag, r)


@pytest.mark.parametrize("name", list(GI.attention_cases().keys()))
def test_golden_cases(attn, golden_dir, name):
    c = GI.attention_cases()[name]
    g = np.load(golden_dir / "attention.npz")
    if c.get("slab_fp8"):
        v8 = torch.from_numpy(g[f"{name}__v8"]).view(torch.float8_e4m3fn)
        vsc = torch.from_numpy(g[f"{name}__vsc"])
        out = attn.block_causal_flash_attention(c["q"].cuda(), c["k"].cuda(), c["v"].cuda(), c["L"].cuda(),
                                                _cuda(c["key_valid"]), c["cache_k"].cuda(), v8.cuda(),
                                                vsc.cuda(), uniform_full=True)
        ref32 = O.block_causal_attention(c["q"], c["k"], c["v"], c["L"], c["key_valid"], c["cache_k"], v8, vsc,
                                         out_dtype=torch.float32)
        exact = O.block_causal_attention(c["q"], c["k"], c["v"], c["L"], c["key_valid"], c["cache_k"], v8, vsc,
                                         out_dtype=torch.float32, slab_v_bf16=False)
        _check(out.cpu(), exact, tag=name + " vs fp32 dequant")
    else:
        out = attn.block_causal_flash_attention(c["q"].cuda(), c["k"].cuda(), c["v"].cuda(), c["L"].cuda(),
                                                _cuda(c["key_valid"]), _cuda(c["cache_k"]), _cuda(c["cache_v"]))
        ref32 = O.block_causal_attention(c["q"], c["k"], c["v"], c["L"], c["key_valid"], c["cache_k"],
                                         c["cache_v"], out_dtype=torch.float32)
    torch.cuda.synchronize()
    _check(out, ref32, tag=name)
    golden = torch.from_numpy(g[f"{name}__out"].view(np.int16)).view(torch.bfloat16).reshape(out.shape)
    assert (out.cpu().float() - golden.float()).abs().max().item() <= MAX_ABS


def _layout_case(layout, batch=1, heads=4, pad=False, seed=0):
    segs, pos = [], 0
    for kind, n in layout:
        segs.append((pos, pos + n, kind == "text"))
        pos += n
    S = pos
    q = GI.randn_bf16(seed, (batch, S, heads, 128), 0.3)
    k = GI.randn_bf16(seed + 1, (batch, S, heads, 128), 0.3)
    v = GI.randn_bf16(seed + 2, (batch, S, heads, 128), 0.3)
    kv = None
    if pad:
        first_text_end = next(e for s, e, t in segs if t)
        kv = torch.ones(batch, S, dtype=torch.bool)
        kv[:, first_text_end - 5:first_text_end] = False
    L = torch.arange(S, dtype=torch.int32)
    for s, e, is_text in segs:
        if not is_text:
            L[s:e] = e - 1
    L[segs[-1][1]:] = S - 1
    return q, k, v, L, kv


# the reference's own test layouts (tests/test_attention.py:154-159), full size
@pytest.mark.parametrize("name,layout,batch,pad", [
    ("t2i prefill", [("text", 256), ("img", 1024)], 1, False),
    ("edit prefill", [("text", 64), ("img", 4096), ("text", 32), ("img", 256)], 1, False),
    ("padded prompt", [("text", 128), ("img", 512)], 1, True),
    ("batch=2", [("text", 96), ("img", 200)], 2, False),
])
def test_reference_prefill_layouts(attn, name, layout, batch, pad):
    q, k, v, L, kv = _layout_case(layout, batch=batch, pad=pad, seed=len(name))
    out = attn.block_causal_flash_attention(q.cuda(), k.cuda(), v.cuda(), L.cuda(), _cuda(kv))
    torch.cuda.synchronize()
    ref32 = O.block_causal_attention(q, k, v, L, kv, out_dtype=torch.float32)
    _check(out, ref32, tag=name)


@pytest.mark.parametrize("P,T", [(256, 512), (1024, 1024), (200, 77)])
def test_reference_decode_layouts(attn, P, T):
    """tests/test_attention.py:137-150: decode over a bf16 cache + fresh target."""
    H = 4
    q = GI.randn_bf16(P, (1, T, H, 128), 0.3)
    kn = GI.randn_bf16(P + 1, (1, T, H, 128), 0.3)
    vn = GI.randn_bf16(P + 2, (1, T, H, 128), 0.3)
    ck = GI.randn_bf16(P + 3, (1, P, H, 128), 0.3)
    cv = GI.randn_bf16(P + 4, (1, P, H, 128), 0.3)
    L = torch.full((T,), P + T - 1, dtype=torch.int32)
    ref32 = O.block_causal_attention(q, kn, vn, L, None, ck, cv, out_dtype=torch.float32)
    for uniform in (False, True):
        out = attn.block_causal_flash_attention(q.cuda(), kn.cuda(), vn.cuda(), L.cuda(), None, ck.cuda(),
                                                cv.cuda(), uniform_full=uniform)
        torch.cuda.synchronize()
        _check(out, ref32, tag=f"decode P={P} T={T} uniform={uniform}")


@pytest.mark.parametrize("P", [0, 300])
def test_no_fresh_keys(attn, P):
    """SN == 0: the query rows attend to the cache alone (P > 0, uniform and per-row
    limits), or to no key at all (P == 0: zeros); the empty fresh K / V are never read."""
    H, T = 2, 200
    q = GI.randn_bf16(70 + P, (1, T, H, 128), 0.3)
    kn = torch.empty(1, 0, H, 128, dtype=torch.bfloat16)
    vn = torch.empty(1, 0, H, 128, dtype=torch.bfloat16)
    if P == 0:
        L = torch.full((T,), -1, dtype=torch.int32)
        out = attn.block_causal_flash_attention(q.cuda(), kn.cuda(), vn.cuda(), L.cuda(), None)
        torch.cuda.synchronize()
        assert torch.count_nonzero(out).item() == 0
        return
    ck = GI.randn_bf16(71 + P, (1, P, H, 128), 0.3)
    cv = GI.randn_bf16(72 + P, (1, P, H, 128), 0.3)
    for L, uniform in ((torch.full((T,), P - 1, dtype=torch.int32), True),
                       (torch.arange(T, dtype=torch.int32) + (P - T), False)):
        ref32 = O.block_causal_attention(q, kn, vn, L, None, ck, cv, out_dtype=torch.float32)
        out = attn.block_causal_flash_attention(q.cuda(), kn.cuda(), vn.cuda(), L.cuda(), None, ck.cuda(),
                                                cv.cuda(), uniform_full=uniform)
        torch.cuda.synchronize()
        _check(out, ref32, tag=f"no fresh keys P={P} uniform={uniform}")


def test_fp8_slab_through_kv_cache(attn):
    """tests/test_kv_cache.py:40-60: fp8-V slab stored by ContiguousKVCache, attention
    vs the oracle with the same dequantized V, and vs the bf16-V result (rel < 0.03)."""
    from qik.kv_cache import ContiguousKVCache
    B, P, Q, H, D = 1, 640, 256, 32, 128
    k = GI.randn_bf16(1, (B, P, H, D))
    v = GI.randn_bf16(2, (B, P, H, D))
    q = GI.randn_bf16(3, (B, Q, H, D), 0.3)
    kn = GI.randn_bf16(4, (B, Q, H, D), 0.3)
    vn = GI.randn_bf16(5, (B, Q, H, D), 0.3)
    L = torch.full((Q,), P + Q - 1, dtype=torch.int32)
    cache = ContiguousKVCache(2, B, P + 16, H, D, v_fp8=True, device="cuda")
    cache.get_layer(1).store(k.cuda(), v.cuda())
    ck8, cv8, vs = cache.get_layer(1).views()
    out8 = attn.block_causal_flash_attention(q.cuda(), kn.cuda(), vn.cuda(), L.cuda(), None, ck8, cv8, vs,
                                             uniform_full=True)
    out16 = attn.block_causal_flash_attention(q.cuda(), kn.cuda(), vn.cuda(), L.cuda(), None, k.cuda(), v.cuda())
    torch.cuda.synchronize()
    ref32 = O.block_causal_attention(q, kn, vn, L, None, ck8.cpu(), cv8.cpu(), vs.cpu(), out_dtype=torch.float32)
    _check(out8, ref32, tag="fp8 slab")
    exact = O.block_causal_attention(q, kn, vn, L, None, ck8.cpu(), cv8.cpu(), vs.cpu(), out_dtype=torch.float32,
                                     slab_v_bf16=False)
    _check(out8, exact, tag="fp8 slab vs fp32 dequant")
    assert O.relf(out8.cpu(), out16.cpu()) < 0.03


def test_cfg4_prefill_form(attn):
    """BASELINE config 4, prefill form: B=1, H=24, D=128, 256 text (L=q) + 2304 cond
    (L=2559) + 4096 target (L=6655), Q/K/V ~ N(0,1).  Oracle checked on all 24 heads
    (head by head, fp32 on the CPU)."""
    H, S = 24, 6656
    q = GI.randn_bf16(41, (1, S, H, 128))
    k = GI.randn_bf16(42, (1, S, H, 128))
    v = GI.randn_bf16(43, (1, S, H, 128))
    L = torch.arange(S, dtype=torch.int32)
    L[256:2560] = 2559
    L[2560:] = S - 1
    out = attn.block_causal_flash_attention(q.cuda(), k.cuda(), v.cuda(), L.cuda(), None)
    torch.cuda.synchronize()
    heads = list(range(H))
    ref32 = O.block_causal_attention(q, k, v, L, None, heads=heads, out_dtype=torch.float32)
    _check(out, ref32, heads=heads, tag="cfg4 prefill")


def test_cfg4_decode_form_fp8_slab(attn):
    """BASELINE config 4, decode form: 4096 target queries over the e4m3-V slab of the
    2560 prefix tokens (stored per head with amax/448 scales) + 4096 fresh keys."""
    from qik.kv_cache import ContiguousKVCache
    H, P, T = 24, 2560, 4096
    kp = GI.randn_bf16(51, (1, P, H, 128))
    vp = GI.randn_bf16(52, (1, P, H, 128))
    q = GI.randn_bf16(53, (1, T, H, 128))
    kn = GI.randn_bf16(54, (1, T, H, 128))
    vn = GI.randn_bf16(55, (1, T, H, 128))
    cache = ContiguousKVCache(1, 1, P, H, 128, v_fp8=True, device="cuda")
    cache.get_layer(0).store(kp.cuda(), vp.cuda())
    ck, cv, vs = cache.get_layer(0).views()
    L = torch.full((T,), P + T - 1, dtype=torch.int32)
    out = attn.block_causal_flash_attention(q.cuda(), kn.cuda(), vn.cuda(), L.cuda(), None, ck, cv, vs,
                                            uniform_full=True)
    torch.cuda.synchronize()
    heads = list(range(H))
    ref32 = O.block_causal_attention(q, kn, vn, L, None, ck.cpu(), cv.cpu(), vs.cpu(), heads=heads,
                                     out_dtype=torch.float32)
    _check(out, ref32, heads=heads, tag="cfg4 decode fp8 slab")
    exact = O.block_causal_attention(q, kn, vn, L, None, ck.cpu(), cv.cpu(), vs.cpu(), heads=heads,
                                     out_dtype=torch.float32, slab_v_bf16=False)
    _check(out, exact, heads=heads, tag="cfg4 decode fp8 slab vs fp32 dequant")


def test_edge_rows_and_ragged_tiles(attn):
    """L = -1 rows give zeros, SQ / P / SN not multiples of 128, key-valid holes that
    empty whole rows, decode with key_valid (non-uniform path)."""
    H, P, SN, SQ = 2, 70, 131, 131
    q = GI.randn_bf16(61, (2, SQ, H, 128), 0.3)
    kn = GI.randn_bf16(62, (2, SN, H, 128), 0.3)
    vn = GI.randn_bf16(63, (2, SN, H, 128), 0.3)
    ck = GI.randn_bf16(64, (2, P, H, 128), 0.3)
    cv = GI.randn_bf16(65, (2, P, H, 128), 0.3)
    g = np.random.default_rng(66)
    L = torch.from_numpy(g.integers(-1, P + SN, size=SQ).astype(np.int32))
    L[:5] = -1
    kv = torch.from_numpy(g.random((2, P + SN)) > 0.2)
    kv[1, :3] = False                                   # rows with L < 3 in batch 1 see nothing
    out = attn.block_causal_flash_attention(q.cuda(), kn.cuda(), vn.cuda(), L.cuda(), kv.cuda(), ck.cuda(),
                                            cv.cuda())
    torch.cuda.synchronize()
    ref32 = O.block_causal_attention(q, kn, vn, L, kv, ck, cv, out_dtype=torch.float32)
    _check(out, ref32, tag="edge")
    assert (out[:, :5].float() == 0).all()


def test_fp8_slab_rows_ending_inside_slab(attn):
    """Block-causal rows over an fp8-V slab where some query tiles never reach the
    fresh keys (their whole range lies in the slab) and others cross the boundary."""
    from qik.kv_cache import ContiguousKVCache
    H, P, SN, SQ = 2, 300, 100, 260
    kp = GI.randn_bf16(71, (1, P, H, 128))
    vp = GI.randn_bf16(72, (1, P, H, 128))
    q = GI.randn_bf16(73, (1, SQ, H, 128), 0.5)
    kn = GI.randn_bf16(74, (1, SN, H, 128), 0.5)
    vn = GI.randn_bf16(75, (1, SN, H, 128), 0.5)
    cache = ContiguousKVCache(1, 1, P, H, 128, v_fp8=True, device="cuda")
    cache.get_layer(0).store(kp.cuda(), vp.cuda())
    ck, cv, vs = cache.get_layer(0).views()
    L = torch.arange(SQ, dtype=torch.int32)            # rows 0..127 end inside the slab
    L[200:] = P + SN - 1
    out = attn.block_causal_flash_attention(q.cuda(), kn.cuda(), vn.cuda(), L.cuda(), None, ck, cv, vs)
    torch.cuda.synchronize()
    exact = O.block_causal_attention(q, kn, vn, L, None, ck.cpu(), cv.cpu(), vs.cpu(), out_dtype=torch.float32,
                                     slab_v_bf16=False)
    _check(out, exact, tag="fp8 slab partial")


@pytest.mark.parametrize("slab", [False, True])
def test_running_max_jumps_in_some_rows(attn, slab):
    """Rows whose running max grows by far more than 2^8 (log2 units) in a later key
    tile while their warp neighbours' does not: O is rescaled in TMEM for some rows
    of a warp only (factor 1 for the others), after the first tile and, with the fp8
    slab, at the same time as the slab-scale boundary."""
    from qik.kv_cache import ContiguousKVCache
    H, S = 2, 640
    P = 256 if slab else 0
    q = GI.randn_bf16(81, (1, S, H, 128), 0.3)
    k = GI.randn_bf16(82, (1, S, H, 128), 0.3)
    v = GI.randn_bf16(83, (1, S, H, 128), 0.5)
    rows = torch.arange(0, S, 3)
    q[0, rows, :, 0] = 4.0
    k[0, 400, :, 0] = 40.0          # raw score ~160 -> ~20 log2 units above the rest
    k[0, 130, :, 0] = -40.0
    L = torch.full((S,), P + S - 1, dtype=torch.int32)
    L[:200] = torch.arange(P, P + 200, dtype=torch.int32)   # causal head rows see the jump only later
    if slab:
        cache = ContiguousKVCache(1, 1, P, H, 128, v_fp8=True, device="cuda")
        cache.get_layer(0).store(GI.randn_bf16(84, (1, P, H, 128), 0.3).cuda(),
                                 GI.randn_bf16(85, (1, P, H, 128), 0.5).cuda())
        ck, cv, vs = cache.get_layer(0).views()
        out = attn.block_causal_flash_attention(q.cuda(), k.cuda(), v.cuda(), L.cuda(), None, ck, cv, vs)
        ref32 = O.block_causal_attention(q, k, v, L, None, ck.cpu(), cv.cpu(), vs.cpu(), out_dtype=torch.float32,
                                         slab_v_bf16=False)
    else:
        out = attn.block_causal_flash_attention(q.cuda(), k.cuda(), v.cuda(), L.cuda(), None)
        ref32 = O.block_causal_attention(q, k, v, L, None, out_dtype=torch.float32)
    torch.cuda.synchronize()
    _check(out, ref32, tag=f"max jumps slab={slab}")
    from qik import _lib as QL
    assert QL.device_status() == 0


def test_status_word_clean(attn):
    from qik import _lib as L
    assert L.device_status() == 0


def test_amax_out_is_max_abs_of_the_output():
    """amax_out (the FP8 out-projection's dynamic scale input) holds the fp32 bits of
    max|out| exactly, for a block-causal prefill and for a decode over the e4m3 slab
    (rows with no allowed key give 0 and do not count)."""
    from qik.kv_cache import ContiguousKVCache
    from qik.triton_attention import block_causal_flash_attention as attn
    B, S, H, D = 2, 300, 3, 128
    q, k, v = (GI.randn_bf16(700 + i, (B, S, H, D), 1.0 + i).cuda() for i in range(3))
    L = torch.arange(S, dtype=torch.int32)
    L[40:] = S - 1
    L[5] = -1
    amax = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = attn(q, k, v, L.cuda(), None, amax_out=amax)
    torch.cuda.synchronize()
    want = np.array([out.float().abs().max().item()], np.float32).view(np.int32)[0]
    assert int(amax.item()) == int(want)
    P, T = 256, 128
    cache = ContiguousKVCache(1, B, P, H, D, v_fp8=True, device="cuda")
    cache.get_layer(0).store(GI.randn_bf16(710, (B, P, H, D)).cuda(), GI.randn_bf16(711, (B, P, H, D), 3.0).cuda())
    ck, cv, vs = cache.get_layer(0).views()
    amax.zero_()
    Ld = torch.full((T,), P + T - 1, dtype=torch.int32, device="cuda")
    out = attn(q[:, :T].contiguous(), k[:, :T].contiguous(), v[:, :T].contiguous(), Ld, None, ck, cv, vs,
               uniform_full=True, amax_out=amax)
    torch.cuda.synchronize()
    want = np.array([out.float().abs().max().item()], np.float32).view(np.int32)[0]
    assert int(amax.item()) == int(want)


@pytest.mark.parametrize("name", ["t2i_prefill", "edit_prefill", "padded_prompt", "batch2", "decode_bf16_slab",
                                  "decode_fp8_slab"])
def test_fp16_tensors(attn, golden_dir, name):
    """The reference accepts fp16 as well as bf16 (triton_attention.py:190): the golden
    layouts with fp16 q / k / v (and fp16 cache K / V, or the golden e4m3 slab V with its
    scales), fp16 output, against the fp32 oracle on the same fp16 values."""
    c = GI.attention_cases()[name]
    h = lambda t: None if t is None else t.to(torch.float16)  # noqa: E731
    q, k, v, ck = h(c["q"]), h(c["k"]), h(c["v"]), h(c["cache_k"])
    L, kv = c["L"], c["key_valid"]
    if c.get("slab_fp8"):
        g = np.load(golden_dir / "attention.npz")
        cv = torch.from_numpy(g[f"{name}__v8"]).view(torch.float8_e4m3fn)
        vsc = torch.from_numpy(g[f"{name}__vsc"])
        out = attn.block_causal_flash_attention(q.cuda(), k.cuda(), v.cuda(), L.cuda(), _cuda(kv), ck.cuda(),
                                                cv.cuda(), vsc.cuda(), uniform_full=True)
        ref32 = O.block_causal_attention(q, k, v, L, kv, ck, cv, vsc, out_dtype=torch.float32, slab_v_bf16=False)
    else:
        cv = h(c["cache_v"])
        out = attn.block_causal_flash_attention(q.cuda(), k.cuda(), v.cuda(), L.cuda(), _cuda(kv), _cuda(ck),
                                                _cuda(cv))
        ref32 = O.block_causal_attention(q, k, v, L, kv, ck, cv, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16 and out.shape == q.shape
    _check(out, ref32, tag=f"fp16 {name}")


def test_fp16_amax_out_and_dtype_checks(attn):
    """amax_out for fp16 output holds the fp32 bits of max|out|; mixed q / k / v types
    are refused, as the reference's single-dtype kernel requires."""
    q, k, v = (GI.randn_bf16(300 + i, (1, 300, 2, 128), 0.5).to(torch.float16).cuda() for i in range(3))
    L = torch.full((300,), 299, dtype=torch.int32, device="cuda")
    amax = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = attn.block_causal_flash_attention(q, k, v, L, None, uniform_full=True, amax_out=amax)
    torch.cuda.synchronize()
    got = np.array([amax.item()], dtype=np.int32).view(np.float32)[0]
    assert got == out.float().abs().max().item()
    with pytest.raises(AssertionError):
        attn.block_causal_flash_attention(q, k.to(torch.bfloat16), v, L, None)
