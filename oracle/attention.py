"""Attention oracle: online-softmax decode over INT4 paged KV (test infrastructure only).

* ``online_softmax`` restates ``online_softmax_ref`` of the reference,
  ``src/flash_decode_ref.py:30-139``: per page, dequantize keys as
  ``kq*scale - zp*scale`` (:92), raw logits ``query @ k.T`` with no softmax
  scale (:97), online max / rescale / sum / weighted-value update (:106-126),
  empty pages skipped (:78-82), ``out = o / max(l, 1e-10)`` (:136-137). It uses
  the same NumPy primitives in the same order so that, on one machine, it
  reproduces the reference bit for bit.
* ``attention_f64`` restates the float64 arbiter of the reference's tests
  (``tests/test_pallas_flash_decode.py:53-78``): every live page concatenated,
  one softmax in float64.
* ``attention_exact_f32_keys`` is the same float64 evaluation, but with keys
  first dequantized in float32 exactly as the oracle does; it is what an
  implementation computes when its only rounding is the reference's key
  dequantization. The CUDA decode kernel is gated against it.
* ``paged_stream_pages`` / ``decode_paged`` drive the oracle over the paged
  layout of this framework: one call per (sequence, kv-head) stream, 16-token
  pages, per-(128-token group, head, channel) scale/zero-point taken from the
  group's first page, GQA query heads sharing their kv head.

Paged pool layout (also the CUDA kernels' layout):
  k_pool  uint8   [num_pages, H_kv, page, ceil(D/2)]   nibble-packed keys
  v_pool  float32 [num_pages, H_kv, page, D]
  sz_pool float32 [num_pages, H_kv, 2, D]              [scale; zero-point],
          stored at the physical page that holds the group's first token.
"""

import numpy as np

from .pack import unpack_int4

_F32 = np.float32


def online_softmax(query, pages, values, block_lens=None):
    """(out [B,H,D] f32, log_partition [B,H]) -- src/flash_decode_ref.py:30-139."""
    m, l, o = online_softmax_state(query, pages, values, block_lens)
    logz = np.log(np.maximum(l, 1e-10))
    return o / np.maximum(l, 1e-10)[:, :, np.newaxis], logz


def online_softmax_state(query, pages, values, block_lens=None):
    """The running (m, l, o) of src/flash_decode_ref.py:30-134 before the final
    normalization (:136-137): max logit, sum of e^(logit-m), unnormalized
    e^(logit-m)-weighted value sum, all float32."""
    q = np.asarray(query)
    if q.ndim != 3:
        raise AssertionError(f"Query must be 3D (batch, heads, dim), got {q.ndim}D")
    nb_, nh, d = q.shape
    n = len(pages)
    if len(values) != n:
        raise AssertionError("Number of blocks must match")
    if block_lens is None:
        block_lens = np.array([pages[i][0].shape[0] for i in range(n)])
    m = np.full((nb_, nh), -np.inf, dtype=_F32)
    l = np.zeros((nb_, nh), dtype=_F32)
    o = np.zeros((nb_, nh, d), dtype=_F32)
    for i in range(n):
        kq, s, z = pages[i]
        rows = int(block_lens[i])
        if rows == 0:
            continue
        v = values[i][:rows]
        k = kq[:rows].astype(_F32) * s[np.newaxis, :] - z[np.newaxis, :] * s[np.newaxis, :]
        logits = np.matmul(q, k.T)
        m_new = np.maximum(m, np.max(logits, axis=-1))
        rescale = np.exp(m - m_new)
        e = np.exp(logits - m_new[:, :, np.newaxis])
        l = l * rescale + np.sum(e, axis=-1)
        o = o * rescale[:, :, np.newaxis] + np.einsum('bhs,sd->bhd', e, v)
        m = m_new
    return m, l, o


def merge_partials(ms, ls, accs):
    """Combine partial softmax states of disjoint key ranges.

    Restates the cross-warp merge of the reference's CUDA kernel
    (csrc/flash_decode_int4.cu:199-220): M = max_p m_p; parts whose m is -inf
    are skipped; L = max(sum_p l_p e^(m_p - M), 1e-10); out = sum_p acc_p
    e^(m_p - M) / L -- here in float64. ms, ls: [P, ...]; accs: [P, ..., D].
    """
    ms = np.asarray(ms, np.float64)
    ls = np.asarray(ls, np.float64)
    accs = np.asarray(accs, np.float64)
    big = ms.max(axis=0)
    live = ms != -np.inf
    with np.errstate(invalid="ignore"):
        e = np.where(live, np.exp(np.where(live, ms - np.where(np.isfinite(big), big, 0.0), 0.0)), 0.0)
    den = np.maximum((ls * e).sum(axis=0), 1e-10)
    return (accs * e[..., None]).sum(axis=0) / den[..., None]


def _concat_live(pages, values, block_lens, key_f32):
    ks, vs = [], []
    for i, (kq, s, z) in enumerate(pages):
        rows = int(block_lens[i]) if block_lens is not None else kq.shape[0]
        if rows == 0:
            continue
        if key_f32:
            k = (kq[:rows].astype(_F32) * s[None, :] - z[None, :] * s[None, :]).astype(np.float64)
        else:
            s64 = s.astype(np.float64)
            z64 = z.astype(np.float64)
            k = kq[:rows].astype(np.float64) * s64 - z64 * s64
        ks.append(k)
        vs.append(np.asarray(values[i][:rows], dtype=np.float64))
    return ks, vs


def _softmax_f64(query, ks, vs):
    q64 = np.asarray(query, dtype=np.float64)
    if not ks:
        return np.zeros(q64.shape, np.float64)
    logits = q64 @ np.concatenate(ks).T
    vals = np.concatenate(vs)
    p = np.exp(logits - logits.max(axis=-1, keepdims=True))
    return (p @ vals) / p.sum(axis=-1, keepdims=True)


def attention_f64(query, pages, values, block_lens=None):
    """Float64 arbiter (tests/test_pallas_flash_decode.py:53-78 of the reference)."""
    ks, vs = _concat_live(pages, values, block_lens, key_f32=False)
    return _softmax_f64(query, ks, vs)


def attention_exact_f32_keys(query, pages, values, block_lens=None):
    """Float64 softmax over keys dequantized in float32 as the oracle does."""
    ks, vs = _concat_live(pages, values, block_lens, key_f32=True)
    return _softmax_f64(query, ks, vs)


def paged_stream_pages(k_pool, v_pool, sz_pool, block_table, seq_lens, b, h,
                       head_dim, page=16, group_pages=8):
    """Page list ``[(kq, scale, zp)], [v]`` of stream (sequence b, kv head h)."""
    n_tok = int(seq_lens[b])
    n_pages = (n_tok + page - 1) // page
    pages, vals = [], []
    for p in range(n_pages):
        phys = int(block_table[b, p])
        rows = min(page, n_tok - p * page)
        g_phys = int(block_table[b, (p // group_pages) * group_pages])
        kq = unpack_int4(k_pool[phys, h, :rows], head_dim)
        pages.append((kq, sz_pool[g_phys, h, 0], sz_pool[g_phys, h, 1]))
        vals.append(v_pool[phys, h, :rows])
    return pages, vals


def decode_paged_state(query, k_pool, v_pool, sz_pool, block_table, seq_lens,
                       page=16, group_pages=8):
    """Per-stream (m [B,H], l [B,H], acc [B,H,D]) of the float32 oracle over a
    paged cache (query heads == kv heads); empty streams are (-inf, 0, 0)."""
    q = np.asarray(query, dtype=_F32)
    nb_, h_, d = q.shape
    m = np.full((nb_, h_), -np.inf, _F32)
    l = np.zeros((nb_, h_), _F32)
    acc = np.zeros((nb_, h_, d), _F32)
    for b in range(nb_):
        for h in range(h_):
            pages, vals = paged_stream_pages(k_pool, v_pool, sz_pool, block_table, seq_lens,
                                             b, h, d, page, group_pages)
            if not pages:
                continue
            mm, ll, oo = online_softmax_state(q[b:b + 1, h:h + 1], pages, vals)
            m[b, h], l[b, h], acc[b, h] = mm[0, 0], ll[0, 0], oo[0, 0]
    return m, l, acc


def stream_f64(query, k_pages, v_pages, sz_pages, n_tok, page=16, group_pages=8):
    """Float64 arbiter for ONE stream whose pages are stored in order, vectorised.

    The same evaluation as ``attention_f64`` (tests/test_pallas_flash_decode.py:53-78
    of the reference): every valid row concatenated, keys dequantized in
    float64 as ``kq*s - zp*s``, one softmax. Pages: k_pages [P, page, D/2]
    packed codes, v_pages [P, page, D], sz_pages [P, 2, D] with the group's
    scale/zp stored at its first page (page index multiple of ``group_pages``).
    query [G, D] -> out [G, D] float64. Used where the per-page form is too
    slow (streams of 10^5 tokens); tests pin the two against each other.
    """
    q64 = np.asarray(query, np.float64)
    if n_tok == 0:
        return np.zeros(q64.shape, np.float64)
    d = q64.shape[-1]
    npg = (n_tok + page - 1) // page
    codes = unpack_int4(np.asarray(k_pages[:npg]), d).astype(np.float64)  # [P, page, D]
    grp = (np.arange(npg) // group_pages) * group_pages
    s64 = np.asarray(sz_pages, np.float64)[grp, 0][:, None, :]
    z64 = np.asarray(sz_pages, np.float64)[grp, 1][:, None, :]
    k = (codes * s64 - z64 * s64).reshape(npg * page, d)[:n_tok]
    v = np.asarray(v_pages[:npg], np.float64).reshape(npg * page, d)[:n_tok]
    logits = q64 @ k.T
    p = np.exp(logits - logits.max(axis=-1, keepdims=True))
    return (p @ v) / p.sum(axis=-1, keepdims=True)


_METHODS = {
    "oracle": lambda q, pg, v: online_softmax(q, pg, v)[0],
    "f64": attention_f64,
    "exact": attention_exact_f32_keys,
}


def decode_paged(query, k_pool, v_pool, sz_pool, block_table, seq_lens,
                 page=16, group_pages=8, method="oracle", streams=None):
    """Decode attention for every (sequence, kv head) stream of a paged cache.

    query [B, Hq, D]; Hq must be a multiple of H_kv and query heads
    ``h*G .. h*G+G-1`` (G = Hq / H_kv) read kv head ``h``. ``method`` picks the
    float32 oracle, the float64 arbiter or the exact-f32-keys evaluation.
    ``streams`` optionally restricts the work to a list of (b, h) pairs (the
    other outputs stay zero); the CPU baseline uses it to time a sample.
    """
    q = np.asarray(query, dtype=_F32)
    nb_, hq, d = q.shape
    hkv = k_pool.shape[1]
    if hq % hkv:
        raise ValueError("query heads must be a multiple of kv heads")
    g = hq // hkv
    fn = _METHODS[method]
    out = np.zeros((nb_, hq, d), np.float64 if method != "oracle" else _F32)
    todo = streams if streams is not None else [(b, h) for b in range(nb_) for h in range(hkv)]
    for b, h in todo:
        pages, vals = paged_stream_pages(k_pool, v_pool, sz_pool, block_table, seq_lens,
                                         b, h, d, page, group_pages)
        if not pages:
            continue
        out[b, h * g:(h + 1) * g] = fn(q[b:b + 1, h * g:(h + 1) * g], pages, vals)[0]
    return out
