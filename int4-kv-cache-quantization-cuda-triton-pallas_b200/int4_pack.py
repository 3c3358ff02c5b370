"""Host-side view of the nibble-packed storage format.

The format is the reference's (src/int4_pack.py:14-56): along the last axis,
even index -> low nibble, odd index -> high nibble; an odd last axis is
zero-padded. On the device the quantizer kernels write this format directly
and the decode kernels read it; these NumPy helpers exist for callers that
hold codes on the host (inspection, serialisation, tests).
"""

import numpy as np


def pack_int4(q: np.ndarray) -> np.ndarray:
    q = np.asarray(q)
    assert q.dtype == np.uint8, f"expected uint8, got {q.dtype}"
    assert q.max(initial=0) <= 15, "values must fit in 4 bits"
    if q.shape[-1] % 2 == 1:
        q = np.concatenate([q, np.zeros(q.shape[:-1] + (1,), np.uint8)], axis=-1)
    return (q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8)


def unpack_int4(packed: np.ndarray, last_dim: int) -> np.ndarray:
    packed = np.asarray(packed)
    assert packed.dtype == np.uint8
    out = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = packed & 0x0F
    out[..., 1::2] = packed >> 4
    return out[..., :last_dim]


def packed_nbytes(shape: tuple) -> int:
    n = (shape[-1] + 1) // 2
    for d in shape[:-1]:
        n *= d
    return n
