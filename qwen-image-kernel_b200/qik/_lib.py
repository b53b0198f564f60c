"""ctypes binding of libqik.so (the C ABI declared in include/qik.h).

The library is built in-tree by ``qwen-image-kernel_b200/build.py``.  There is no
fallback: if the library is missing, or no CUDA device is present, the first call
raises instead of computing anything elsewhere.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libqik.so"

QIK_OK = 0
DTYPE_BF16, DTYPE_F32, DTYPE_E4M3 = 0, 1, 2
EPI_SCALE, EPI_GELU_TANH, EPI_SCATTER, EPI_SWIGLU = 0, 1, 2, 3
GEMM_TILE_AUTO, GEMM_TILE_PAIR_256, GEMM_TILE_SINGLE_256, GEMM_TILE_SINGLE_128, GEMM_TILE_SINGLE_64, GEMM_TILE_SWAP_16 = range(6)
TP_MAX_WORLD = 8
ATTN_HAS_CACHE, ATTN_HAS_KEY_VALID, ATTN_UNIFORM, ATTN_V_FP8, ATTN_F16 = 1, 2, 4, 8, 16
STATUS_OK, STATUS_TIMEOUT = 0, 1

_i64, _i32, _f32, _vp, _u64 = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_uint64


class AttnArgs(ctypes.Structure):
    """Mirror of ``qik_attn_args`` (include/qik.h)."""
    _fields_ = [
        ("q", _vp), ("k", _vp), ("v", _vp), ("cache_k", _vp), ("cache_v", _vp), ("cache_v_scale", _vp),
        ("L", _vp), ("key_valid", _vp), ("out", _vp),
        ("B", _i64), ("SQ", _i64), ("SN", _i64), ("P", _i64), ("H", _i64), ("D", _i64),
        ("q_sb", _i64), ("q_ss", _i64), ("q_sh", _i64),
        ("k_sb", _i64), ("k_ss", _i64), ("k_sh", _i64),
        ("v_sb", _i64), ("v_ss", _i64), ("v_sh", _i64),
        ("ck_sb", _i64), ("ck_ss", _i64), ("ck_sh", _i64),
        ("cv_sb", _i64), ("cv_ss", _i64), ("cv_sh", _i64),
        ("o_sb", _i64), ("o_ss", _i64), ("o_sh", _i64),
        ("kv_sb", _i64),
        ("sm_scale", _f32),
        ("flags", _i32),
        ("amax_out", _vp),
    ]


# name -> (restype, argtypes)
SIGNATURES = {
    "qik_version": (_i32, []),
    "qik_last_error": (ctypes.c_char_p, []),
    "qik_quant_workspace_bytes": (ctypes.c_size_t, []),
    "qik_compute_scale": (_i32, [_vp, _i32, _i64, _vp, _vp, _vp]),
    "qik_amax": (_i32, [_vp, _i32, _i64, _vp, _vp]),
    "qik_quantize_act": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp]),
    "qik_quantize_act_from_amax": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp]),
    "qik_quantize_act_noalloc": (_i32, [_vp, _i64, _vp, _vp, _vp]),
    "qik_quantize_weight": (_i32, [_vp, _i32, _i64, _vp, _vp, _vp, _vp]),
    "qik_fp8_gemm": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _vp,
                            _vp, _vp]),
    "qik_fp8_gemm_tiled": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _i32, _i32,
                                  _vp, _i32, _vp, _vp]),
    "qik_fp8_gemm_qkv_rms_rope": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _i32, _i32,
                                         _vp, _vp, _vp, _vp, _i64, _f32, _vp, _vp]),
    "qik_gate_table": (_i32, [_vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "qik_fp8_gemm_gate_residual": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _vp, _i64,
                                          _vp, _i64, _i64, _vp, _i64, _vp, _vp]),
    "qik_fp8_ffn_workspace_bytes": (ctypes.c_size_t, [_i64, _i64, _i64]),
    "qik_fp8_ffn": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp,
                           _vp]),
    "qik_fp8_ffn_from_amax": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                     ctypes.c_size_t, _vp, _vp]),
    "qik_fp8_ffn_e4m3": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                ctypes.c_size_t, _vp, _vp]),
    "qik_block_causal_attention": (_i32, [ctypes.POINTER(AttnArgs), _vp, _vp]),
    "qik_kv_store": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _i64,
                            _i32, _vp, _vp, _vp]),
    "qik_rms_norm_rope": (_i32, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _f32, _vp, _i64,
                                 _i64, _i64, _vp]),
    "qik_layer_norm_modulate": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _f32, _vp, _vp,
                                       _vp]),
    "qik_layer_norm_modulate_e4m3": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _f32, _vp, _vp,
                                            _vp, _vp, _vp]),
    "qik_gate_residual": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "qik_swiglu": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp]),
    "qik_selftest_wait_timeout": (_i32, [_vp, _u64, _vp]),
    "qik_ipc_handle_bytes": (ctypes.c_size_t, []),
    "qik_ipc_export": (_i32, [_vp, _vp, ctypes.POINTER(_u64)]),
    "qik_ipc_open": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "qik_ipc_close": (_i32, [_vp]),
    "qik_fp8_gemm_scatter_signals": (_i64, [_i64, _i64, _i64, _i32]),
    "qik_fp8_gemm_scatter": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _i32, _i64, _vp, _vp, _vp,
                                    _vp]),
    "qik_tp_reduce_gather": (_i32, [_vp, _vp, ctypes.c_uint32, _i32, _i32, _i64, _i64, _i64, _vp, _vp, _vp, _i32,
                                    _vp, _vp]),
    "qik_tp_wait": (_i32, [_vp, ctypes.c_uint32, _i32, _vp, _vp]),
    "qik_rows_bias_bf16": (_i32, [_vp, _i64, _i64, _vp, _vp, _vp, _vp]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class QikError(RuntimeError):
    pass


def load(require_cuda: bool = True) -> ctypes.CDLL:
    """Load libqik.so.  With ``require_cuda`` (every compute call) a CUDA device must
    be present: the kernels have no CPU path."""
    global _lib
    if require_cuda and not torch.cuda.is_available():
        raise QikError("qik: no CUDA device; the qik kernels run only on sm_100a GPUs")
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise QikError(f"qik: {LIB_PATH} is missing; build it with qwen-image-kernel_b200/build.py")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                try:
                    fn = getattr(lib, name)
                except AttributeError:
                    continue   # reported by missing_symbols(); calling it raises
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def missing_symbols() -> list[str]:
    """Entry points of include/qik.h that the loaded library does not export."""
    lib = load(require_cuda=False)
    return [n for n in SIGNATURES if not hasattr(lib, n)]


def check(rc: int, what: str) -> None:
    if rc != QIK_OK:
        msg = load(require_cuda=False).qik_last_error()
        raise QikError(f"{what} failed (status {rc}): {msg.decode() if msg else ''}")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_status: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word the kernels write on a failed bounded wait."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def device_status(device: torch.device | None = None) -> int:
    """Read (synchronizing) the device status word; 0 means no kernel gave up a wait."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    return int(status_word(dev)[0].item())


_quant_state: dict[tuple[int, int], torch.Tensor] = {}


def quant_state(device: torch.device, stream: int | None = None) -> torch.Tensor:
    """The workspace qik_quantize_act keeps between calls, one per (device, stream):
    zeroed when first made, then passed to every call on that stream (each completed
    call leaves its grid-barrier state ready for the next, so no call clears it)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, stream_ptr(torch.device("cuda", idx)) if stream is None else stream)
    t = _quant_state.get(key)
    if t is None:
        t = torch.zeros(load().qik_quant_workspace_bytes(), dtype=torch.uint8, device=torch.device("cuda", idx))
        _quant_state[key] = t
    return t


def reset_quant_state() -> None:
    """Zero every cached quantizer workspace (needed after a call that failed)."""
    for t in _quant_state.values():
        t.zero_()

