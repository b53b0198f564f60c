"""CPU oracle for the Qwen-Image FP8 DiT hot path.

TEST INFRASTRUCTURE ONLY.  This module restates the reference's arithmetic on the
CPU so the CUDA kernels can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg (and its
``--impl reference`` arm) may import it; the product path (``qik``) never does.

Byte-exact parts (quantizers) live in ``qik_oracle.c`` (built by the Makefile
next to this file into ``_build/libqik_oracle.so``) and are reached through
ctypes.  Floating-point parts (the fp32 dequant GEMM and attention) are restated
in PyTorch fp32 on CPU.

Reference = gomezcojj-coder/qwen-image-kernel; every function cites the lines it
follows.  Parity pins: ``tests/golden/make_golden.py`` produced the committed
fixtures by running the reference's own CPU-runnable functions; see
``tests/test_oracle_golden.py``.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np
import torch

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libqik_oracle.so"

SCALE_CUDA = 0   # amax * fl32(1/448): how the reference's expression evaluates on CUDA
SCALE_CPU = 1    # amax / 448 (true division): the same expression on CPU tensors
E4M3_MAX = 448.0
_RECIP_448 = np.float32(1.0) / np.float32(448.0)


def build() -> Path:
    """Compile the C restatement if needed (gcc, no fast-math)."""
    src = _HERE / "qik_oracle.c"
    if not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(_LIB_PATH))
        f32, i64, vp, i32 = ctypes.c_float, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
        L.qik_oracle_e4m3_satfinite.argtypes = [f32]
        L.qik_oracle_e4m3_satfinite.restype = ctypes.c_uint8
        L.qik_oracle_e4m3_torch.argtypes = [f32]
        L.qik_oracle_e4m3_torch.restype = ctypes.c_uint8
        L.qik_oracle_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.qik_oracle_e4m3_to_f32.restype = f32
        L.qik_oracle_amax_bf16.argtypes = [vp, i64]
        L.qik_oracle_amax_bf16.restype = f32
        L.qik_oracle_amax_f32.argtypes = [vp, i64]
        L.qik_oracle_amax_f32.restype = f32
        L.qik_oracle_scale_from_amax.argtypes = [f32, i32]
        L.qik_oracle_scale_from_amax.restype = f32
        L.qik_oracle_pack_act_bf16.argtypes = [vp, i64, f32, vp]
        L.qik_oracle_pack_act_bf16.restype = None
        L.qik_oracle_pack_div_bf16.argtypes = [vp, i64, f32, vp]
        L.qik_oracle_pack_div_bf16.restype = None
        L.qik_oracle_pack_div_f32.argtypes = [vp, i64, f32, vp]
        L.qik_oracle_pack_div_f32.restype = None
        L.qik_oracle_slab_v_store.argtypes = [vp, i64, i64, i64, i64, i64, i64, i64, i64, vp, vp, i32]
        L.qik_oracle_slab_v_store.restype = None
        _lib = L
    return _lib


# ----------------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------------
def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    assert t.dtype == torch.bfloat16
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def e4m3_bytes_to_f32(q: np.ndarray) -> np.ndarray:
    """Exact decode of e4m3 bytes (table of all 256 codes)."""
    table = np.array([lib().qik_oracle_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)
    return table[q]


def e4m3_from_f32_torch(x: np.ndarray) -> np.ndarray:
    """c10's fp32 -> float8_e4m3fn conversion (round-to-nearest-even, overflow -> NaN)."""
    f = lib().qik_oracle_e4m3_torch
    flat = np.ascontiguousarray(x, dtype=np.float32).ravel()
    return np.fromiter((f(float(v)) for v in flat), dtype=np.uint8, count=flat.size).reshape(np.shape(x))


def e4m3_from_f32_satfinite(x: np.ndarray) -> np.ndarray:
    """Device cvt.rn.satfinite fp32 -> e4m3 (round-to-nearest-even, saturating)."""
    f = lib().qik_oracle_e4m3_satfinite
    flat = np.ascontiguousarray(x, dtype=np.float32).ravel()
    return np.fromiter((f(float(v)) for v in flat), dtype=np.uint8, count=flat.size).reshape(np.shape(x))


# ----------------------------------------------------------------------------------
# quantizers (byte-exact)
# ----------------------------------------------------------------------------------
def amax(x: torch.Tensor) -> float:
    """max|x| over all elements (fp8.py:26 `x.abs().amax()`); NaN propagates."""
    if x.dtype == torch.bfloat16:
        bits = _bf16_bits(x).ravel()
        return float(lib().qik_oracle_amax_bf16(_ptr(bits), bits.size))
    a = x.detach().cpu().contiguous().float().numpy().ravel()
    return float(lib().qik_oracle_amax_f32(_ptr(a), a.size))


def scale_from_amax(a: float, mode: int = SCALE_CUDA) -> float:
    """compute_scale's arithmetic (fp8.py:24-26): clamp_min(fl32(amax)/448, 1e-12)."""
    return float(lib().qik_oracle_scale_from_amax(a, mode))


def compute_scale(x: torch.Tensor, mode: int = SCALE_CUDA) -> float:
    """fp8.py:24-26 / fp8.py:58 (weights) / kv_cache.py:38-39 (per-head slab V)."""
    return scale_from_amax(amax(x), mode)


def reciprocal_rn(s: float) -> float:
    """IEEE round-to-nearest fp32 1/s."""
    return float(np.float32(1.0) / np.float32(s))


def quantize_act(x: torch.Tensor, mode: int = SCALE_CUDA, inv: float | None = None):
    """quantize_tensorwise (fp8.py:44-53): s = compute_scale(x); q = e4m3(x * (1/s)).

    ``inv`` is the fp32 value of ``1/s`` the device formed (fp8.py:39); by default
    the reference's form (act_reciprocal).  Returns (q uint8 ndarray, s float).
    """
    bits = _bf16_bits(x)
    s = compute_scale(x, mode)
    if inv is None:
        inv = act_reciprocal(s)
    q = np.empty(bits.shape, dtype=np.uint8)
    lib().qik_oracle_pack_act_bf16(_ptr(bits), bits.size, inv, _ptr(q))
    return q, s


def quantize_weight(w: torch.Tensor, mode: int = SCALE_CUDA):
    """quantize_weight_tensorwise (fp8.py:56-60): q = e4m3(clamp(fl32(w) / s, +-448))."""
    s = compute_scale(w, mode)
    q = np.empty(tuple(w.shape), dtype=np.uint8)
    if w.dtype == torch.bfloat16:
        bits = _bf16_bits(w)
        lib().qik_oracle_pack_div_bf16(_ptr(bits), bits.size, s, _ptr(q))
    else:
        a = w.detach().cpu().contiguous().float().numpy()
        lib().qik_oracle_pack_div_f32(_ptr(a), a.size, s, _ptr(q))
    return q, s


def slab_v_store(v: torch.Tensor, pmax: int, mode: int = SCALE_CUDA):
    """_LayerView.store's fp8-V branch (kv_cache.py:36-42).

    v: [B, P, H, D] bf16 (any strides).  Returns (v8 uint8 [B, H, pmax, D] with rows
    >= P left zero, scale float32 [B, H]).
    """
    assert v.dtype == torch.bfloat16 and v.dim() == 4
    B, P, H, D = v.shape
    vc = v.detach().cpu().contiguous()
    bits = vc.view(torch.int16).numpy().view(np.uint16)
    v8 = np.zeros((B, H, pmax, D), dtype=np.uint8)
    scale = np.zeros((B, H), dtype=np.float32)
    lib().qik_oracle_slab_v_store(_ptr(bits), B, P, H, D, P * H * D, H * D, D, pmax,
                                  _ptr(v8), _ptr(scale), mode)
    return v8, scale


# ----------------------------------------------------------------------------------
# fp32 restatements (floating point)
# ----------------------------------------------------------------------------------
def dequant(q: np.ndarray | torch.Tensor, s: float) -> torch.Tensor:
    """fl32(q) * s in fp32."""
    if isinstance(q, torch.Tensor):
        q = q.detach().cpu().contiguous().view(torch.uint8).numpy()
    return torch.from_numpy(e4m3_bytes_to_f32(np.asarray(q))) * np.float32(s)


def fp8_linear(xq, sx: float, wq, sw: float, bias: torch.Tensor | None = None) -> torch.Tensor:
    """The fp32-accumulated dequant path of FP8Linear.forward (fp8.py:85-90):
    y32 = (fl32(xq) * sx) @ (fl32(wq) * sw)^T (+ bias), in fp32."""
    a = dequant(xq, sx)
    b = dequant(wq, sw)
    y = a @ b.t()
    if bias is not None:
        y = y + bias.detach().cpu().float()
    return y


def gelu_tanh(y: torch.Tensor) -> torch.Tensor:
    """GELU with the tanh approximation, evaluated in fp32 on the bf16 input, rounded
    to bf16 (torch.nn.functional.gelu(approximate='tanh') on a bf16 tensor).  The
    reference has no GELU path; configs 2-3 of the benchmark ask for it."""
    return torch.nn.functional.gelu(y.float(), approximate="tanh").to(torch.bfloat16)


def build_prefix_lengths(segments, prefix_len: int, seq_len: int) -> torch.Tensor:
    """processors.py:22-36: per-row inclusive kv limit L (text: causal, image block:
    end-1, target rows: S-1)."""
    L = torch.arange(seq_len, dtype=torch.int32)
    for start, end, is_text in segments:
        if not is_text:
            L[start:end] = end - 1
    L[prefix_len:] = seq_len - 1
    return L


def block_causal_attention(query, key, value, prefix_lengths, key_valid=None, cache_k=None,
                           cache_v=None, cache_v_scale=None, heads=None,
                           out_dtype=torch.bfloat16, slab_v_bf16: bool = True) -> torch.Tensor:
    """reference_block_causal_attention (triton_attention.py:266-293) on the CPU in fp32,
    extended with the fp8 slab-V dequant of the kernel (triton_attention.py:154-159):
    slab V = bf16(fl32(v8) * vsc[b, h]).  Computed head by head to bound memory.

    query [B,SQ,H,D] bf16, key/value [B,SN,H,D], prefix_lengths [SQ] int32 (absolute
    kv index), key_valid [B,P+SN] bool or None, cache_k [B,P,H,D] bf16, cache_v
    [B,P,H,D] bf16 or e4m3 (then cache_v_scale [B,H] fp32).  Rows with no allowed key
    produce zeros (the kernel's `l == 0` epilogue, triton_attention.py:166).
    Returns [B,SQ,H,D] in ``out_dtype`` (bf16 like the reference, or fp32 for
    tolerance checks on the pre-cast values).  ``slab_v_bf16=False`` keeps the slab V
    dequant in fp32 (fl32(v8) * vsc, the fp32-accumulated dequant path parity is gated on) instead of
    the reference kernel's per-element bf16 rounding.
    """
    B, SQ, H, D = query.shape
    P = 0 if cache_k is None else cache_k.shape[1]
    if cache_v is not None and cache_v.dtype == torch.float8_e4m3fn:
        assert cache_v_scale is not None
        cv = cache_v.detach().cpu().float() * cache_v_scale.detach().cpu().float()[:, None, :, None]
        cache_v = cv.to(torch.bfloat16) if slab_v_bf16 else cv
        value = value if slab_v_bf16 else value.detach().cpu().float()
    k_all = key if cache_k is None else torch.cat([cache_k.cpu(), key.cpu()], dim=1)
    v_all = value if cache_v is None else torch.cat([cache_v.cpu(), value.cpu()], dim=1)
    KV = k_all.shape[1]
    Lr = prefix_lengths.detach().cpu().to(torch.int64)
    idx = torch.arange(KV)
    allowed = idx[None, :] <= Lr[:, None]                       # [SQ, KV]
    out = torch.zeros(B, SQ, H, D, dtype=torch.float32)
    hs = range(H) if heads is None else heads
    for b in range(B):
        allow_b = allowed
        if key_valid is not None:
            allow_b = allowed & key_valid[b].detach().cpu().to(torch.bool)[None, :]
        empty = ~allow_b.any(dim=1)
        for h in hs:
            q = query[b, :, h].detach().cpu().float()
            k = k_all[b, :, h].detach().cpu().float()
            v = v_all[b, :, h].detach().cpu().float()
            s = (q @ k.t()) * (D ** -0.5)
            s = s.masked_fill(~allow_b, float("-inf"))
            p = torch.softmax(s, dim=-1)
            p = torch.nan_to_num(p, nan=0.0)
            o = p @ v
            o[empty] = 0.0
            out[b, :, h] = o
    return out if out_dtype == torch.float32 else out.to(out_dtype)


def attention_flops(prefix_lengths: torch.Tensor, key_valid_rows: int | None, B: int, H: int, D: int,
                    kv_total: int) -> float:
    """Algorithmic FLOPs 4*D*H*B*sum_rows(min(L, KV-1)+1) (QK^T + PV over allowed pairs)."""
    L = prefix_lengths.detach().cpu().to(torch.int64).clamp(min=-1, max=kv_total - 1)
    return 4.0 * D * H * B * float((L + 1).sum())


def relf(a: torch.Tensor, b: torch.Tensor) -> float:
    """Relative Frobenius error ||a-b|| / ||b||."""
    a = a.float()
    b = b.float()
    den = b.norm().item()
    return (a - b).norm().item() / den if den > 0 else (a - b).norm().item()


def bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 numbers at |x| (for the <= 1 ulp output gate)."""
    a = x.float().abs().clamp_min(2.0 ** -126)
    e = torch.floor(torch.log2(a))
    return torch.pow(2.0, e - 7)



_RECIP_TABLE: dict[int, int] | None = None


def act_reciprocal(s: float) -> float:
    """fp32 value of ``1.0 / s`` as the reference's activation cast forms it
    (fp8.py:39, an fp32 division inside a Triton kernel).

    It equals the IEEE round-to-nearest reciprocal except for the scales listed in
    tests/golden/act_reciprocal.npz, which tests/golden/make_act_reciprocal.py measured
    on a B200 by evaluating that same Triton expression for every scale a bf16
    tensor can produce.  Without the table this is the IEEE reciprocal."""
    global _RECIP_TABLE
    if _RECIP_TABLE is None:
        path = _HERE.parent / "tests" / "golden" / "act_reciprocal.npz"
        _RECIP_TABLE = {}
        if path.exists():
            g = np.load(path)
            _RECIP_TABLE = dict(zip(g["scale_bits"].tolist(), g["inv_bits"].tolist()))
    sb = int(np.float32(s).view(np.uint32))
    if sb in _RECIP_TABLE:
        return float(np.uint32(_RECIP_TABLE[sb]).view(np.float32))
    return reciprocal_rn(s)


# ---------------------------------------------------------------- fused elementwise ops
# Restatements of the reference's fused Triton kernels (qwen_image_kernel/triton_fused.py)
# in fp32 on the CPU with bf16 roundings at the points the kernels round.

def _rb(t: torch.Tensor) -> torch.Tensor:
    """Round an fp32 tensor to bf16 (nearest-even) and back to fp32."""
    return t.to(torch.bfloat16).float()


def modulation_rows(target_token_mask: torch.Tensor | None, B: int, S: int) -> torch.Tensor:
    """[B, S] modulation row of each (sample, position): the row map of
    _modulation_row_map (triton_fused.py:141-151, 0 for target positions, B
    otherwise) plus the sample index, as the kernels add it (triton_fused.py:127,199)."""
    if target_token_mask is None:
        base = torch.zeros(S, dtype=torch.int64)
    else:
        base = torch.where(target_token_mask.cpu().to(torch.bool), 0, B).to(torch.int64)
    return base[None, :] + torch.arange(B, dtype=torch.int64)[:, None]


def rms_norm_rope(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                  eps: float) -> torch.Tensor:
    """rms_rope_kernel (triton_fused.py:28-69): per (b, s, h) row of D,
    rrms = rsqrt(sum(x^2) / D + eps); n = bf16((x * rrms) * w) in fp32; the pairs
    (n[2i], n[2i+1]) rotate by (cos[s, i], sin[s, i]); bf16 out.
    x: [B, S, H, D] bf16 (any strides); weight: [D]; cos, sin: [S, D/2] fp32."""
    x = x.cpu().float()
    D = x.shape[-1]
    ss = (x * x).sum(-1, keepdim=True)
    rrms = torch.rsqrt(ss / D + eps)
    n = _rb((x * rrms) * weight.cpu().float())
    ne, no = n[..., 0::2], n[..., 1::2]
    c = cos.cpu().float()[None, :, None, :]
    s = sin.cpu().float()[None, :, None, :]
    oe = ne * c - no * s
    oo = ne * s + no * c
    return torch.stack([oe, oo], -1).flatten(-2).to(torch.bfloat16)


def layer_norm_modulate(x: torch.Tensor, modulation: torch.Tensor, scale_off: int,
                        target_token_mask: torch.Tensor | None, eps: float) -> torch.Tensor:
    """ln_modulate_kernel (triton_fused.py:111-138): LayerNorm without affine in fp32
    (mean, then the centred variance), y = bf16(xc * rsqrt(var + eps)), then
    bf16(y * bf16(1 + scale)) with scale = modulation[row, scale_off : scale_off + D].
    x: [B, S, D] bf16; modulation: [R, >= scale_off + D] bf16."""
    x = x.cpu().float()
    B, S, D = x.shape
    mean = x.sum(-1, keepdim=True) / D
    xc = x - mean
    var = (xc * xc).sum(-1, keepdim=True) / D
    y = _rb(xc * torch.rsqrt(var + eps))
    rows = modulation_rows(target_token_mask, B, S)
    sc = modulation.cpu()[rows][..., scale_off:scale_off + D].float()
    return (y * _rb(1.0 + sc)).to(torch.bfloat16)


def gate_residual(x: torch.Tensor, f: torch.Tensor, modulation: torch.Tensor, gate_off: int,
                  target_token_mask: torch.Tensor | None) -> torch.Tensor:
    """gate_residual_kernel (triton_fused.py:183-209): g = bf16(tanh(gate)) with gate =
    modulation[row, gate_off : gate_off + D]; y = x + g * f in bf16 arithmetic (the
    product rounded to bf16, then the sum), as the stock expression rounds."""
    x = x.cpu().float()
    B, S, D = x.shape
    rows = modulation_rows(target_token_mask, B, S)
    g = _rb(torch.tanh(modulation.cpu()[rows][..., gate_off:gate_off + D].float()))
    t = _rb(g * f.cpu().float())
    return (x + t).to(torch.bfloat16)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """swiglu_kernel (triton_fused.py:237-249): s = bf16(g * sigmoid(g)) in fp32, then
    bf16(s * up)."""
    g = gate.cpu().float()
    s = _rb(g * torch.sigmoid(g))
    return (s * up.cpu().float()).to(torch.bfloat16)
