"""Prefix-length construction of the block-causal mask.

``_build_prefix_lengths`` follows qwen_image_kernel/processors.py:22-36: the
block-causal mask of a joint [prefix ; target] sequence collapses to one inclusive
key limit per query row -- text rows are causal (L = q), image-block rows see the
whole prefix up to the end of their block (L = end - 1), target rows see everything
(L = S - 1).  BASELINE's "causal length" is the exclusive count L + 1.
"""
from __future__ import annotations

import torch


def _build_prefix_lengths(segments: list[tuple[int, int, bool]], prefix_len: int, seq_len: int,
                          device: torch.device) -> torch.Tensor:
    """Per-row inclusive kv limit L: row q attends iff kv <= L[q]."""
    L = torch.arange(seq_len, dtype=torch.int32, device=device)
    for start, end, is_text in segments:
        if not is_text:
            L[start:end] = end - 1
    L[prefix_len:] = seq_len - 1
    return L
