"""Rotary position embedding of the decode step (test infrastructure).

The reference quantizes POST-RoPE keys: its model path hooks the cache update
of a Hugging Face Llama, which applies the rotary embedding first
(scripts/validate_llama.py:23-31, 123-175; transformers pinned ">=4.36" in
pyproject.toml:44). The rotation is transformers'
``models.llama.modeling_llama.apply_rotary_pos_emb`` in its rotate-half form:

    x_embed = (x * cos) + (rotate_half(x) * sin),
    rotate_half(x) = cat(-x[..., D/2:], x[..., :D/2]),
    cos = cat(c, c), sin = cat(s, s) for the per-position half tables c, s,

evaluated in float32, each product and the sum rounded separately. This is a
NumPy restatement of that expression; ``tests/test_rope_oracle.py`` pins it
bit for bit against transformers' own function on the same tables.
"""

import numpy as np

_F32 = np.float32


def apply_rope(x, positions, cos_half, sin_half):
    """x [rows, heads, D] float32 rotated at positions [rows] with tables
    cos_half / sin_half [max_positions, D/2] float32."""
    x = np.asarray(x, dtype=_F32)
    pos = np.asarray(positions, dtype=np.int64)
    d = x.shape[-1]
    half = d // 2
    c = np.asarray(cos_half, dtype=_F32)[pos][:, None, :]  # [rows, 1, D/2]
    s = np.asarray(sin_half, dtype=_F32)[pos][:, None, :]
    lo, hi = x[..., :half], x[..., half:]
    out = np.empty_like(x)
    # (x * cos) + (rotate_half(x) * sin): -hi * s is exactly -(hi * s)
    out[..., :half] = (lo * c) - (hi * s)
    out[..., half:] = (hi * c) + (lo * s)
    return out


def rope_table_f32(max_positions, head_dim, base=10000.0):
    """The half tables of the checker's cases: angles pos * base^(-2i/D) in
    float64, cos / sin rounded to float32 (any table works for parity: the
    kernel and this oracle take it as an input)."""
    inv = base ** (-np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)
    ang = np.arange(max_positions, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(_F32), np.sin(ang).astype(_F32)
