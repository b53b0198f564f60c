"""Drop qik into an unmodified checkout of gomezcojj-coder/qwen-image-kernel.

``install()`` registers the qik modules under the reference's module names before
the reference package is imported:

    qwen_image_kernel.fp8               -> qik.fp8
    qwen_image_kernel.triton_attention  -> qik.triton_attention
    qwen_image_kernel.kv_cache          -> qik.kv_cache
    qwen_image_kernel.quantize_offline  -> qik.quantize_offline
    qwen_image_kernel.triton_fused      -> qik.triton_fused
    qwen_image_kernel.processors        -> qik.processors

The reference's own relative imports (``from .fp8 import FP8Linear`` and
``from .processors import QwenImage21KernelBlock, QwenImage21KernelProcessor`` in
runtime.py:33-35, ``from .kv_cache import ContiguousKVCache`` in runtime.py:34)
resolve through ``sys.modules`` and therefore bind the qik implementations;
everything else in the reference package (the runtime, metrics, the web UI) loads
from the checkout as before.
"""
from __future__ import annotations

import importlib
import sys

MODULES = {
    "fp8": "qik.fp8",
    "triton_attention": "qik.triton_attention",
    "kv_cache": "qik.kv_cache",
    "quantize_offline": "qik.quantize_offline",
    "triton_fused": "qik.triton_fused",
    "processors": "qik.processors",
}


def install(package: str = "qwen_image_kernel") -> dict[str, object]:
    """Register the qik modules as ``<package>.<name>``.  Call before importing the
    reference package; if the package is already imported its attributes are
    replaced too.  Returns the mapping that was installed."""
    installed = {}
    for name, target in MODULES.items():
        mod = importlib.import_module(target)
        sys.modules[f"{package}.{name}"] = mod
        installed[f"{package}.{name}"] = mod
        parent = sys.modules.get(package)
        if parent is not None:
            setattr(parent, name, mod)
    return installed


def uninstall(package: str = "qwen_image_kernel") -> None:
    for name, target in MODULES.items():
        key = f"{package}.{name}"
        if sys.modules.get(key) is sys.modules.get(target):
            del sys.modules[key]
