"""Rotary position embedding tables for the decode step.

A Llama-style model rotates q and k by position before attention, and the
reference quantizes the post-RoPE keys (scripts/validate_llama.py:23-31). The
rotation itself runs on the GPU, fused into the step's cache append
(``int4kv_cache_append_rope``) or as ``int4kv_rope`` for prefill rows; this
module only builds its parameter table once, like a weight:
``cos[p, i] = cos(p * base^(-2i/D))`` and ``sin`` likewise, for i < D/2,
angles in float64 and the values rounded to float32 (Llama-2: base 10000).
"""

import math

import numpy as np
import torch


def rope_table(max_positions: int, head_dim: int, base: float = 10000.0, device="cuda"):
    """(cos, sin) float32 [max_positions, head_dim // 2] on `device`."""
    if head_dim % 8 or head_dim <= 0 or max_positions <= 0:
        raise ValueError("rope tables need head_dim % 8 == 0 and max_positions > 0")
    if not (base > 1.0 and math.isfinite(base)):
        raise ValueError("rope base must be a finite number > 1")
    inv = base ** (-np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)
    ang = np.arange(max_positions, dtype=np.float64)[:, None] * inv[None, :]
    cos = torch.from_numpy(np.cos(ang).astype(np.float32)).to(device)
    sin = torch.from_numpy(np.sin(ang).astype(np.float32)).to(device)
    return cos, sin
