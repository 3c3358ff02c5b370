"""Input contract of the shared-stream attention entry point.

Same contract and error texts as the reference's
``normalize_attention_inputs`` (src/_validate.py:11-64): query is 3-D; the
four page lists have equal length; each key page is ``[rows, head_dim]``; each
value page has its key page's shape; each scale / zero-point is
``(head_dim,)``; every block length lies in ``[0, rows of that page]``.
Returns ``(query, block_lens as int32)``.
"""

import numpy as np


def normalize_attention_inputs(query, k_q_blocks, k_scales, k_zps, v_blocks, block_lens):
    query = np.asarray(query)
    if query.ndim != 3:
        raise ValueError(f"query must be [batch, heads, head_dim], got shape {query.shape}")
    dim = query.shape[2]
    n = len(k_q_blocks)
    if not (len(k_scales) == len(k_zps) == len(v_blocks) == n):
        raise ValueError(
            "k_q_blocks, k_scales, k_zps and v_blocks must have the same length, got "
            f"{n}, {len(k_scales)}, {len(k_zps)}, {len(v_blocks)}")
    rows = np.zeros(n, dtype=np.int64)
    for i in range(n):
        ks, vs = np.shape(k_q_blocks[i]), np.shape(v_blocks[i])
        if len(ks) != 2 or ks[1] != dim:
            raise ValueError(f"key page {i} must be [rows, {dim}], got shape {ks}")
        if vs != ks:
            raise ValueError(f"value page {i} has shape {vs}, expected {ks} to match its key page")
        if np.shape(k_scales[i]) != (dim,) or np.shape(k_zps[i]) != (dim,):
            raise ValueError(
                f"scale/zero-point for page {i} must have shape ({dim},), got "
                f"{np.shape(k_scales[i])} and {np.shape(k_zps[i])}")
        rows[i] = ks[0]
    if block_lens is None:
        lens = rows.copy()
    else:
        lens = np.asarray(block_lens).astype(np.int64).reshape(-1)
        if lens.shape[0] != n:
            raise ValueError(f"block_lens has {lens.shape[0]} entries for {n} pages")
        bad = np.flatnonzero((lens < 0) | (lens > rows))
        if bad.size:
            i = int(bad[0])
            raise ValueError(
                f"block_lens[{i}] = {int(lens[i])} is outside [0, {int(rows[i])}], the number of "
                "rows actually present in that page")
    return query, lens.astype(np.int32)
