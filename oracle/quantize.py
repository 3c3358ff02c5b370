"""Quantizer oracle: per-channel asymmetric INT4 (test infrastructure only).

Restates ``src/quantize_int4_ref.py`` of the reference:

* ``quantize_int4``   -- ``quantize_int4_ref`` (per_channel=True), :23-84
* ``dequantize_int4`` -- ``dequantize_int4_ref`` (per_channel=True), :87-136
* ``quantize_grouped`` -- the grouped driver the benchmark configs need: the
  reference realises "per block" by calling ``quantize_int4_ref`` once per
  block on a 2-D ``[rows, head_dim]`` slice (``src/vllm_integration.py:51``,
  ``benchmarks/bench_three_backend.py:120-124``); here the block is a
  128-token group of one head.

All arithmetic is float32 with IEEE rounding: ``range = max(max-min, 1e-8)``,
``scale = range / 15``, ``zp = -min / scale``,
``q = clip(rint((x - min) / scale), 0, 15)`` (round half to even, as
``np.round`` does).
"""

import numpy as np

_F32 = np.float32
_EPS = np.float32(1e-8)   # src/quantize_int4_ref.py:66
_LEVELS = np.float32(15.0)  # src/quantize_int4_ref.py:67


def quantize_int4(kv):
    """(q uint8 same shape, scale [C], zp [C]) reducing over all leading axes.

    Restates src/quantize_int4_ref.py:46-84 for per_channel=True: min/max over
    every axis but the last (:51-56), float32 throughout (:49).
    """
    x = np.asarray(kv)
    if x.ndim < 2:
        raise ValueError(f"KV must be at least 2D, got {x.ndim}D")
    if x.dtype not in (np.float32, np.float16):
        raise ValueError(f"Expected FP32/FP16, got {x.dtype}")
    x = x.astype(_F32)
    lead = tuple(range(x.ndim - 1))
    lo = np.min(x, axis=lead, keepdims=True)
    hi = np.max(x, axis=lead, keepdims=True)
    scale = np.maximum(hi - lo, _EPS) / _LEVELS
    zp = -lo / scale
    q = np.clip(np.rint((x - lo) / scale), 0, 15).astype(np.uint8)
    c = x.shape[-1]
    return q, scale.reshape(c), zp.reshape(c)


def dequantize_int4(q, scale, zp):
    """k = q*scale - zp*scale in float32 (src/quantize_int4_ref.py:109-131)."""
    qf = np.asarray(q).astype(_F32)
    s = np.asarray(scale).astype(_F32)
    z = np.asarray(zp).astype(_F32)
    return qf * s - z * s


def quantize_grouped(kv, group=128):
    """Per-(group, head, channel) quantizer for kv[N, H, D] float32.

    Each group of ``group`` consecutive tokens of one head is quantized as an
    independent 2-D ``[rows, D]`` array, exactly as one ``quantize_int4_ref``
    call on ``kv[g*group:(g+1)*group, h, :]`` would; the last group may be
    partial and then uses only its own rows.

    Returns (q [N, H, D] uint8 one value per byte, scale [G, H, D], zp [G, H, D]).
    The reductions are vectorised over groups and heads; min/max are exact and
    the elementwise float32 operations are the same per element as the
    per-call form, so the result is bit-identical to it.
    """
    x = np.asarray(kv)
    if x.ndim != 3:
        raise ValueError(f"kv must be [tokens, heads, head_dim], got {x.shape}")
    x = x.astype(_F32)
    n, h, d = x.shape
    if n == 0:
        raise ValueError("kv must have at least one token")
    g_full = n // group
    tail = n - g_full * group
    qs, ss, zs = [], [], []
    if g_full:
        blk = x[: g_full * group].reshape(g_full, group, h, d)
        lo = blk.min(axis=1, keepdims=True)
        hi = blk.max(axis=1, keepdims=True)
        scale = np.maximum(hi - lo, _EPS) / _LEVELS
        zp = -lo / scale
        q = np.clip(np.rint((blk - lo) / scale), 0, 15).astype(np.uint8)
        qs.append(q.reshape(g_full * group, h, d))
        ss.append(scale.reshape(g_full, h, d))
        zs.append(zp.reshape(g_full, h, d))
    if tail:
        blk = x[g_full * group:]
        lo = blk.min(axis=0, keepdims=True)
        hi = blk.max(axis=0, keepdims=True)
        scale = np.maximum(hi - lo, _EPS) / _LEVELS
        zp = -lo / scale
        q = np.clip(np.rint((blk - lo) / scale), 0, 15).astype(np.uint8)
        qs.append(q)
        ss.append(scale.reshape(1, h, d))
        zs.append(zp.reshape(1, h, d))
    return np.concatenate(qs), np.concatenate(ss), np.concatenate(zs)
