"""Nibble packing oracle (test infrastructure only).

Restates ``src/int4_pack.py`` of the reference: along the last axis, even
index -> low nibble, odd index -> high nibble (:27-29); an odd last axis is
zero-padded first (:23-25); ``unpack`` strips the pad (:41-47).
"""

import numpy as np


def pack_int4(q):
    """uint8 values in [0, 15] -> uint8 [..., ceil(n/2)] (src/int4_pack.py:14-29)."""
    q = np.asarray(q)
    if q.dtype != np.uint8:
        raise AssertionError(f"expected uint8, got {q.dtype}")
    if q.size and q.max() > 15:
        raise AssertionError("values must fit in 4 bits")
    if q.shape[-1] % 2:
        q = np.concatenate([q, np.zeros(q.shape[:-1] + (1,), np.uint8)], axis=-1)
    return (q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8)


def unpack_int4(packed, last_dim):
    """Inverse of pack_int4 (src/int4_pack.py:32-47)."""
    p = np.asarray(packed)
    if p.dtype != np.uint8:
        raise AssertionError(f"expected uint8, got {p.dtype}")
    out = np.empty(p.shape[:-1] + (2 * p.shape[-1],), np.uint8)
    out[..., 0::2] = p & 0x0F
    out[..., 1::2] = p >> 4
    return out[..., :last_dim]


def packed_nbytes(shape):
    """Bytes of the packed form of an unpacked shape (src/int4_pack.py:50-56)."""
    n = (shape[-1] + 1) // 2
    for d in shape[:-1]:
        n *= d
    return n
