"""qik -- B200-native (sm_100a) FP8 DiT hot path of Qwen-Image.

Host-side mirror of the reference's operator interface (gomezcojj-coder/
qwen-image-kernel): ``qik.fp8`` (FP8Linear and the e4m3 quantizers),
``qik.triton_attention`` (block_causal_flash_attention), ``qik.kv_cache``
(ContiguousKVCache) and ``qik.quantize_offline`` (the e4m3 weight-cache format).
All arithmetic runs in the CUDA kernels of ``libqik.so`` (C ABI: include/qik.h).
"""
from . import _lib  # noqa: F401

__version__ = "0.1.0"
