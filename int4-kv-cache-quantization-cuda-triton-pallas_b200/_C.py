"""Torch-tensor binding over the C ABI -- the framework's ``_C`` module.

Mirrors the reference's pybind extension (csrc/bindings.cpp:26-132): the same
two entry points ``quantize_int4(kv)`` and ``flash_decode_int4(query, k_q,
k_scale, k_zp, value, block_lens)`` with the same argument meaning, the same
validation order and the same keywords in the ``RuntimeError`` messages
(``float32``, ``non-empty``, ``2D``, ``k_scale``, ``value``, ``block_lens``,
``int32``, ``head_dim`` ...). Outputs are allocated from the torch caching
allocator on the input's device; launches go on torch's current stream.

The paged entry points (``quantize_int4_grouped``, ``cache_write``,
``paged_decode``) are new: they serve the benchmark paged-cache configurations.

Nothing here computes on the CPU: a missing library raises.
"""

import torch

from . import _lib

MAX_HEAD_DIM = 256
PAGE_TOKENS = 16

#: value-pool dtypes of the paged path -> INT4KV_VALUES_* (include/int4kv_b200.h)
VALUE_KINDS = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t):
    return t.data_ptr() if t is not None else None


def _check_input(t, name):
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _same_device(ref, *ts):
    for t in ts:
        if t is not None and t.device != ref.device:
            raise RuntimeError("all tensors must be on the same CUDA device")


# --------------------------------------------------------------------------
# reference entry points
# --------------------------------------------------------------------------

def quantize_int4(kv):
    """Per-channel INT4 over all rows of kv[rows, C] -> [q u8 [rows, C], scale [C], zp [C]]."""
    lib = _lib.load()
    _check_input(kv, "kv")
    if kv.dim() != 2:
        raise RuntimeError("kv must be 2D [num_rows, num_channels]")
    if kv.dtype != torch.float32:
        raise RuntimeError("kv must be float32")
    rows, ch = kv.shape
    if rows <= 0 or ch <= 0:
        raise RuntimeError(f"kv must be non-empty, got [{rows}, {ch}]")
    if rows > 2**31 - 1 or ch > 2**31 - 1:
        raise RuntimeError("kv dimensions must fit in int32")
    with torch.cuda.device(kv.device):
        q = torch.empty((rows, ch), dtype=torch.uint8, device=kv.device)
        scale = torch.empty((ch,), dtype=torch.float32, device=kv.device)
        zp = torch.empty((ch,), dtype=torch.float32, device=kv.device)
        _lib.check(lib.cu_quantize_int4(_p(kv), rows, ch, _p(q), _p(scale), _p(zp), _stream(kv)),
                   "quantize_int4")
    return [q, scale, zp]


def flash_decode_int4(query, k_q, k_scale, k_zp, value, block_lens):
    """Shared-stream INT4 decode (reference csrc/bindings.cpp:56-127 contract)."""
    lib = _lib.load()
    for t, n in ((query, "query"), (k_q, "k_q"), (k_scale, "k_scale"), (k_zp, "k_zp"),
                 (value, "value"), (block_lens, "block_lens")):
        _check_input(t, n)
    if query.dim() != 3:
        raise RuntimeError("query must be 3D [batch, heads, head_dim]")
    if k_q.dim() != 3:
        raise RuntimeError("k_q must be 3D [num_blocks, block_size, head_dim]")
    if query.dtype != torch.float32:
        raise RuntimeError("query must be float32")
    if k_q.dtype != torch.uint8:
        raise RuntimeError("k_q must be uint8")
    if k_scale.dtype != torch.float32:
        raise RuntimeError("k_scale must be float32")
    if k_zp.dtype != torch.float32:
        raise RuntimeError("k_zp must be float32")
    if value.dtype != torch.float32:
        raise RuntimeError("value must be float32")
    if block_lens.dtype != torch.int32:
        raise RuntimeError("block_lens must be int32")
    hd = query.shape[2]
    nb, bs = k_q.shape[0], k_q.shape[1]
    if query.shape[0] <= 0 or query.shape[1] <= 0:
        raise RuntimeError("query must have at least one batch entry and one head")
    if not 1 <= hd <= MAX_HEAD_DIM:
        raise RuntimeError(f"head_dim must be in [1, {MAX_HEAD_DIM}], got {hd}")
    if k_q.shape[2] != hd:
        raise RuntimeError("k_q last dim must equal head_dim")
    if value.dim() != 3 or tuple(value.shape) != (nb, bs, hd):
        raise RuntimeError("value must be [num_blocks, block_size, head_dim] matching k_q")
    if k_scale.dim() != 2 or tuple(k_scale.shape) != (nb, hd):
        raise RuntimeError("k_scale must be [num_blocks, head_dim]")
    if k_zp.dim() != 2 or tuple(k_zp.shape) != (nb, hd):
        raise RuntimeError("k_zp must be [num_blocks, head_dim]")
    if block_lens.dim() != 1 or block_lens.shape[0] != nb:
        raise RuntimeError("block_lens must be [num_blocks]")
    _same_device(query, k_q, k_scale, k_zp, value, block_lens)
    b, h = query.shape[0], query.shape[1]
    with torch.cuda.device(query.device):
        out = torch.empty((b, h, hd), dtype=torch.float32, device=query.device)
        import ctypes
        need = ctypes.c_size_t(0)
        _lib.check(lib.int4kv_dense_decode_workspace_size(b, h, hd, nb, bs, ctypes.byref(need)),
                   "flash_decode_int4")
        ws = torch.empty((max(16, need.value),), dtype=torch.uint8, device=query.device)
        _lib.check(lib.int4kv_dense_decode(_p(query), _p(k_q), _p(k_scale), _p(k_zp), _p(value),
                                           _p(block_lens), b, h, hd, nb, bs, _p(out), _p(ws),
                                           ws.numel(), _stream(query)),
                   "flash_decode_int4")
    return out


# --------------------------------------------------------------------------
# paged-cache entry points
# --------------------------------------------------------------------------

def quantize_int4_grouped(kv, group_tokens=128):
    """kv[N, H, D] f32 -> (packed [N, H, D/2] u8, scale [G, H, D], zp [G, H, D])."""
    lib = _lib.load()
    _check_input(kv, "kv")
    if kv.dim() != 3:
        raise RuntimeError("kv must be 3D [num_tokens, num_heads, head_dim]")
    if kv.dtype != torch.float32:
        raise RuntimeError("kv must be float32")
    n, h, d = kv.shape
    if n <= 0 or h <= 0 or d <= 0:
        raise RuntimeError(f"kv must be non-empty, got {list(kv.shape)}")
    if d % 4:
        raise RuntimeError(f"head_dim must be a multiple of 4 for the packed layout, got {d}")
    if group_tokens <= 0:
        raise RuntimeError(f"group_tokens must be positive, got {group_tokens}")
    g = (n + group_tokens - 1) // group_tokens
    with torch.cuda.device(kv.device):
        packed = torch.empty((n, h, d // 2), dtype=torch.uint8, device=kv.device)
        scale = torch.empty((g, h, d), dtype=torch.float32, device=kv.device)
        zp = torch.empty((g, h, d), dtype=torch.float32, device=kv.device)
        _lib.check(lib.int4kv_quantize_grouped(_p(kv), n, h, d, group_tokens, _p(packed), _p(scale),
                                               _p(zp), _stream(kv)),
                   "quantize_int4_grouped")
    return packed, scale, zp


def _check_pools(k_pool, v_pool, sz_pool):
    _check_input(k_pool, "k_pool")
    _check_input(sz_pool, "sz_pool")
    if k_pool.dtype != torch.uint8 or k_pool.dim() != 4:
        raise RuntimeError("k_pool must be uint8 [num_pages, kv_heads, page, head_dim/2]")
    num_pages, hkv, page, half = k_pool.shape
    d = 2 * half
    if v_pool is not None:
        _check_input(v_pool, "v_pool")
        if v_pool.dtype not in VALUE_KINDS or tuple(v_pool.shape) != (num_pages, hkv, page, d):
            raise RuntimeError("v_pool must be float32, float16 or bfloat16 "
                               "[num_pages, kv_heads, page, head_dim] matching k_pool")
    if sz_pool.dtype != torch.float32 or tuple(sz_pool.shape) != (num_pages, hkv, 2, d):
        raise RuntimeError("sz_pool must be float32 [num_pages, kv_heads, 2, head_dim] matching k_pool")
    return num_pages, hkv, page, d


def _check_table(block_table, batch):
    _check_input(block_table, "block_table")
    if block_table.dtype != torch.int32:
        raise RuntimeError("block_table must be int32")
    if block_table.dim() != 2 or block_table.shape[0] != batch or block_table.shape[1] <= 0:
        raise RuntimeError(f"block_table must be [batch={batch}, max_pages>0]")
    return block_table.shape[1]


def cache_write(k, v, tok_offsets, block_table, k_pool, v_pool, sz_pool, max_rows_per_seq,
                start_pos=None, group_tokens=128, status=None):
    """Quantize k and scatter k/v rows of each sequence into the paged pools."""
    lib = _lib.load()
    num_pages, hkv, page, d = _check_pools(k_pool, v_pool, sz_pool)
    _check_input(k, "k")
    if k.dtype != torch.float32 or k.dim() != 3 or tuple(k.shape[1:]) != (hkv, d):
        raise RuntimeError(f"k must be float32 [tokens, {hkv}, {d}]")
    if v is not None:
        _check_input(v, "v")
        if v.dtype != torch.float32 or v.shape != k.shape:
            raise RuntimeError("v must be float32 with the shape of k")
    _check_input(tok_offsets, "tok_offsets")
    if tok_offsets.dtype != torch.int32 or tok_offsets.dim() != 1:
        raise RuntimeError("tok_offsets must be int32 [batch+1]")
    batch = tok_offsets.shape[0] - 1
    if batch <= 0:
        raise RuntimeError("tok_offsets must describe at least one sequence")
    max_pages = _check_table(block_table, batch)
    if start_pos is not None:
        _check_input(start_pos, "start_pos")
        if start_pos.dtype != torch.int32 or tuple(start_pos.shape) != (batch,):
            raise RuntimeError("start_pos must be int32 [batch]")
    if status is not None and (status.dtype != torch.int32 or status.numel() < 1):
        raise RuntimeError("status must be an int32 tensor")
    _same_device(k, v, tok_offsets, block_table, k_pool, v_pool, sz_pool, start_pos, status)
    vk = VALUE_KINDS[v_pool.dtype] if v_pool is not None else 0
    with torch.cuda.device(k.device):
        _lib.check(lib.int4kv_cache_write_ex(_p(k), _p(v), _p(tok_offsets), _p(start_pos), batch,
                                             int(max_rows_per_seq), hkv, d, group_tokens, page,
                                             _p(block_table), max_pages, num_pages, _p(k_pool),
                                             _p(v_pool), vk, _p(sz_pool), _p(status), _stream(k)),
                   "cache_write")


def block_decode(query, k_packed, k_scale, k_zp, value, block_lens, block_ids):
    """Shared-stream decode over listed blocks of a block cache, read in place
    (int4kv_block_decode). query [B, H, D] -> [B, H, D] float32."""
    import ctypes
    lib = _lib.load()
    for t, name in ((query, "query"), (k_packed, "k_packed"), (k_scale, "k_scale"),
                    (k_zp, "k_zp"), (value, "value"), (block_lens, "block_lens"),
                    (block_ids, "block_ids")):
        _check_input(t, name)
    if query.dtype != torch.float32 or query.dim() != 3:
        raise RuntimeError("query must be float32 [batch, heads, head_dim]")
    b, h, d = query.shape
    if d > MAX_HEAD_DIM:
        raise RuntimeError(f"head_dim {d} exceeds {MAX_HEAD_DIM}")
    if k_packed.dtype != torch.uint8 or k_packed.dim() != 3 or k_packed.shape[2] != (d + 1) // 2:
        raise RuntimeError("k_packed must be uint8 [blocks, block_size, ceil(head_dim/2)]")
    nblk, bs = k_packed.shape[:2]
    if value.dtype not in VALUE_KINDS or tuple(value.shape) != (nblk, bs, d):
        raise RuntimeError("value must be float32/float16/bfloat16 [blocks, block_size, head_dim]")
    for t, name in ((k_scale, "k_scale"), (k_zp, "k_zp")):
        if t.dtype != torch.float32 or tuple(t.shape) != (nblk, d):
            raise RuntimeError(f"{name} must be float32 [blocks, head_dim]")
    if block_lens.dtype != torch.int32 or tuple(block_lens.shape) != (nblk,):
        raise RuntimeError("block_lens must be int32 [blocks]")
    if block_ids.dtype != torch.int32 or block_ids.dim() != 1:
        raise RuntimeError("block_ids must be int32 [listed]")
    _same_device(query, k_packed, k_scale, k_zp, value, block_lens, block_ids)
    nl = block_ids.shape[0]
    with torch.cuda.device(query.device):
        out = torch.empty((b, h, d), dtype=torch.float32, device=query.device)
        need = ctypes.c_size_t(0)
        _lib.check(lib.int4kv_dense_decode_workspace_size(b, h, d, nl, bs, ctypes.byref(need)),
                   "dense_decode_workspace_size")
        ws = torch.empty((max(16, need.value),), dtype=torch.uint8, device=query.device)
        _lib.check(lib.int4kv_block_decode(_p(query), _p(k_packed), _p(k_scale), _p(k_zp),
                                           _p(value), VALUE_KINDS[value.dtype], _p(block_lens),
                                           _p(block_ids), nl, nblk, b, h, d, bs, _p(out), _p(ws),
                                           ws.numel(), _stream(query)),
                   "block_decode")
    return out


def cache_append(k_new, v_new, positions, stage_slots, k_stage, block_table, k_pool, v_pool,
                 sz_pool, group_tokens=128, status=None, rope=None, q=None, q_out=None):
    """Append one token per sequence (int4kv_cache_append): k_new / v_new [B, H, D].

    With ``rope = (cos, sin)`` (float32 [positions, D/2] each) the new keys are
    rotated at their positions before they are staged and quantized, and the
    query ``q`` [B, Hq, D] (if given) is rotated into ``q_out`` in the same
    launch (int4kv_cache_append_rope). Returns ``q_out`` (or None).
    """
    lib = _lib.load()
    num_pages, hkv, page, d = _check_pools(k_pool, v_pool, sz_pool)
    _check_input(k_new, "k_new")
    if k_new.dtype != torch.float32 or k_new.dim() != 3 or tuple(k_new.shape[1:]) != (hkv, d):
        raise RuntimeError(f"k_new must be float32 [batch, {hkv}, {d}]")
    b = k_new.shape[0]
    if v_new is not None:
        _check_input(v_new, "v_new")
        if v_new.dtype != torch.float32 or v_new.shape != k_new.shape:
            raise RuntimeError("v_new must be float32 with the shape of k_new")
    for t, name in ((positions, "positions"), (stage_slots, "stage_slots")):
        _check_input(t, name)
        if t.dtype != torch.int32 or tuple(t.shape) != (b,):
            raise RuntimeError(f"{name} must be int32 [batch]")
    _check_input(k_stage, "k_stage")
    if k_stage.dtype != torch.float32 or k_stage.dim() != 3 or \
            tuple(k_stage.shape[1:]) != (group_tokens, hkv * d):
        raise RuntimeError(f"k_stage must be float32 [slots, {group_tokens}, {hkv * d}]")
    max_pages = _check_table(block_table, b)
    cos = sin = None
    rope_n = 0
    if rope is not None:
        cos, sin = rope
        for t, name in ((cos, "rope cos"), (sin, "rope sin")):
            _check_input(t, name)
            if t.dtype != torch.float32 or t.dim() != 2 or t.shape[1] != d // 2:
                raise RuntimeError(f"{name} must be float32 [positions, {d // 2}]")
        if cos.shape != sin.shape:
            raise RuntimeError("rope cos and sin must have the same shape")
        rope_n = cos.shape[0]
    hq = 0
    if q is not None:
        _check_input(q, "q")
        if q.dtype != torch.float32 or q.dim() != 3 or q.shape[0] != b or q.shape[2] != d:
            raise RuntimeError(f"q must be float32 [{b}, heads, {d}]")
        hq = q.shape[1]
        if q_out is None:
            q_out = torch.empty_like(q)
        _check_input(q_out, "q_out")
        if q_out.dtype != torch.float32 or q_out.shape != q.shape:
            raise RuntimeError("q_out must be float32 with the shape of q")
    _same_device(k_new, v_new, positions, stage_slots, k_stage, block_table, k_pool, v_pool,
                 sz_pool, status, cos, sin, q, q_out)
    vk = VALUE_KINDS[v_pool.dtype] if v_pool is not None else 0
    with torch.cuda.device(k_new.device):
        _lib.check(lib.int4kv_cache_append_rope(
            _p(k_new), _p(v_new), _p(positions), _p(stage_slots), _p(k_stage), k_stage.shape[0],
            b, hkv, d, group_tokens, page, _p(block_table), max_pages, num_pages, _p(k_pool),
            _p(v_pool), vk, _p(sz_pool), _p(cos), _p(sin), rope_n, _p(q),
            _p(q_out) if q is not None else None, hq, _p(status), _stream(k_new)),
            "cache_append")
    return q_out if q is not None else None


def paged_decode_workspace_bytes(batch, q_heads, kv_heads, head_dim, device=None,
                                 value_dtype=torch.float32):
    import ctypes
    lib = _lib.load()
    need = ctypes.c_size_t(0)
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        _lib.check(lib.int4kv_paged_decode_workspace_size_ex(batch, q_heads, kv_heads, head_dim,
                                                             VALUE_KINDS[value_dtype],
                                                             ctypes.byref(need)),
                   "paged_decode_workspace_size")
    return need.value


def paged_decode(query, k_pool, v_pool, sz_pool, block_table, seq_lens, group_tokens=128,
                 out=None, workspace=None, status=None):
    """INT4 paged flash-decode: query[B, H, D] over per-(sequence, head) page streams."""
    lib = _lib.load()
    num_pages, hkv, page, d = _check_pools(k_pool, v_pool, sz_pool)
    if v_pool is None:
        raise RuntimeError("v_pool is required")
    _check_input(query, "query")
    if query.dtype != torch.float32 or query.dim() != 3:
        raise RuntimeError("query must be float32 [batch, heads, head_dim]")
    b, hq, qd = query.shape
    if qd != d:
        raise RuntimeError(f"query head_dim {qd} != pool head_dim {d}")
    if d not in (64, 128, 256):
        raise RuntimeError(f"paged decode supports head_dim in (64, 128, 256), got {d}")
    if page != PAGE_TOKENS:
        raise RuntimeError(f"paged decode needs {PAGE_TOKENS}-token pages, got {page}")
    if hq < hkv or hq % hkv:
        raise RuntimeError(f"query heads ({hq}) must be a multiple of kv heads ({hkv})")
    max_pages = _check_table(block_table, b)
    _check_input(seq_lens, "seq_lens")
    if seq_lens.dtype != torch.int32 or tuple(seq_lens.shape) != (b,):
        raise RuntimeError("seq_lens must be int32 [batch]")
    _same_device(query, k_pool, v_pool, sz_pool, block_table, seq_lens, out, workspace, status)
    with torch.cuda.device(query.device):
        if out is None:
            out = torch.empty((b, hq, d), dtype=torch.float32, device=query.device)
        elif out.dtype != torch.float32 or tuple(out.shape) != (b, hq, d) or not out.is_contiguous():
            raise RuntimeError("out must be contiguous float32 [batch, heads, head_dim]")
        need = paged_decode_workspace_bytes(b, hq, hkv, d, query.device, v_pool.dtype)
        if workspace is None:
            # zero-filled once; every completed launch leaves it zero-filled again
            workspace = torch.zeros((need,), dtype=torch.uint8, device=query.device)
        elif workspace.numel() * workspace.element_size() < need:
            raise RuntimeError(f"workspace needs {need} bytes")
        _lib.check(lib.int4kv_paged_decode_ex(_p(query), _p(k_pool), _p(v_pool),
                                              VALUE_KINDS[v_pool.dtype], _p(sz_pool),
                                              _p(block_table), _p(seq_lens), b, hq, hkv, d, page,
                                              group_tokens, max_pages, num_pages, _p(out),
                                              _p(workspace),
                                              workspace.numel() * workspace.element_size(),
                                              _p(status), _stream(query), None, None),
                   "paged_decode")
    return out


def paged_decode_partials(query, k_pool, v_pool, sz_pool, block_table, seq_lens,
                          group_tokens=128, out=None, workspace=None, status=None):
    """paged_decode writing per-stream partial records instead of outputs.

    Returns ``out``: uint8 [batch * heads * (16 + 4 * head_dim)], one record
    ``[m f64][l f64][acc f32 x head_dim]`` per (sequence, head) stream
    (``INT4KV_PARTIAL_RECORD_BYTES``), for a later ``merge_partials``.
    """
    lib = _lib.load()
    num_pages, hkv, page, d = _check_pools(k_pool, v_pool, sz_pool)
    if v_pool is None:
        raise RuntimeError("v_pool is required")
    _check_input(query, "query")
    if query.dtype != torch.float32 or query.dim() != 3:
        raise RuntimeError("query must be float32 [batch, heads, head_dim]")
    b, hq, qd = query.shape
    if qd != d or hq < hkv or hq % hkv:
        raise RuntimeError("query must be [batch, G * kv_heads, pool head_dim]")
    max_pages = _check_table(block_table, b)
    _check_input(seq_lens, "seq_lens")
    if seq_lens.dtype != torch.int32 or tuple(seq_lens.shape) != (b,):
        raise RuntimeError("seq_lens must be int32 [batch]")
    _same_device(query, k_pool, v_pool, sz_pool, block_table, seq_lens, out, workspace, status)
    nbytes = b * hq * (16 + 4 * d)
    with torch.cuda.device(query.device):
        if out is None:
            out = torch.empty((nbytes,), dtype=torch.uint8, device=query.device)
        elif out.dtype != torch.uint8 or out.numel() != nbytes or not out.is_contiguous():
            raise RuntimeError(f"partials must be contiguous uint8 [{nbytes}]")
        need = paged_decode_workspace_bytes(b, hq, hkv, d, query.device, v_pool.dtype)
        if workspace is None:
            workspace = torch.zeros((need,), dtype=torch.uint8, device=query.device)
        elif workspace.numel() * workspace.element_size() < need:
            raise RuntimeError(f"workspace needs {need} bytes")
        _lib.check(lib.int4kv_paged_decode_partials_ex(
            _p(query), _p(k_pool), _p(v_pool), VALUE_KINDS[v_pool.dtype], _p(sz_pool),
            _p(block_table), _p(seq_lens), b, hq, hkv, d, page, group_tokens, max_pages,
            num_pages, _p(out), _p(workspace), workspace.numel() * workspace.element_size(),
            _p(status), _stream(query)),
            "paged_decode_partials")
    return out


def merge_partials(partials, streams, head_dim, out=None):
    """Combine partial records [parts, streams * record] into float32 [streams, head_dim]."""
    lib = _lib.load()
    _check_input(partials, "partials")
    rec = 16 + 4 * head_dim
    if partials.dtype != torch.uint8 or partials.numel() % (streams * rec):
        raise RuntimeError(f"partials must be uint8 [parts, {streams} x {rec}]")
    parts = partials.numel() // (streams * rec)
    with torch.cuda.device(partials.device):
        if out is None:
            out = torch.empty((streams, head_dim), dtype=torch.float32, device=partials.device)
        elif out.dtype != torch.float32 or out.numel() != streams * head_dim or not out.is_contiguous():
            raise RuntimeError("out must be contiguous float32 [streams, head_dim]")
        _lib.check(lib.int4kv_merge_partials(_p(partials), parts, streams, head_dim, _p(out),
                                             _stream(partials)), "merge_partials")
    return out


# --------------------------------------------------------------------------
# fused peer exchange (sequence split over NVLink peer memory)
# --------------------------------------------------------------------------

def exchange_bytes(world, streams, head_dim):
    """Bytes of one rank's exchange buffer (int4kv_exchange_bytes)."""
    import ctypes
    lib = _lib.load()
    n = ctypes.c_size_t(0)
    _lib.check(lib.int4kv_exchange_bytes(world, streams, head_dim, ctypes.byref(n)), "exchange_bytes")
    return n.value


def exchange_alloc(device, nbytes):
    """A zero-filled device allocation of its own (IPC-shareable); returns its address."""
    import ctypes
    lib = _lib.load()
    ptr = ctypes.c_void_p(None)
    _lib.check(lib.int4kv_exchange_alloc(int(device), int(nbytes), ctypes.byref(ptr)), "exchange_alloc")
    return int(ptr.value)


def exchange_free(ptr):
    _lib.check(_lib.load().int4kv_exchange_free(ptr), "exchange_free")


def ipc_handle(ptr):
    """64 opaque bytes naming the allocation that starts at ``ptr``."""
    import ctypes
    buf = ctypes.create_string_buffer(64)
    _lib.check(_lib.load().int4kv_ipc_handle(ptr, buf), "ipc_handle")
    return bytes(buf.raw)


def ipc_open(handle):
    """Map a peer process's allocation on the current device; returns its address here."""
    import ctypes
    if not isinstance(handle, (bytes, bytearray)) or len(handle) != 64:
        raise RuntimeError("an IPC handle is 64 bytes")
    ptr = ctypes.c_void_p(None)
    _lib.check(_lib.load().int4kv_ipc_open(bytes(handle), ctypes.byref(ptr)), "ipc_open")
    return int(ptr.value)


def ipc_close(ptr):
    _lib.check(_lib.load().int4kv_ipc_close(ptr), "ipc_close")


def exchange_merge(partials, peer_bufs, rank, streams, head_dim, out, status=None):
    """Push this rank's partial records to every rank's exchange buffer, wait
    (bounded) for theirs and merge: out [streams, head_dim] float32 on every rank.

    ``peer_bufs`` = addresses of the ranks' exchange buffers as mapped on this
    GPU, in rank order (``exchange_alloc`` / ``ipc_open``).
    """
    import ctypes
    lib = _lib.load()
    _check_input(partials, "partials")
    _check_input(out, "out")
    _same_device(partials, out, status)
    rec = 16 + 4 * head_dim
    if partials.dtype != torch.uint8 or partials.numel() != streams * rec:
        raise RuntimeError(f"partials must be uint8 [{streams} x {rec}]")
    if out.dtype != torch.float32 or out.numel() != streams * head_dim:
        raise RuntimeError("out must be contiguous float32 [streams, head_dim]")
    if status is not None and (status.dtype != torch.int32 or status.numel() < 1):
        raise RuntimeError("status must be an int32 tensor")
    world = len(peer_bufs)
    arr = (ctypes.c_void_p * max(world, 1))(*[int(p) for p in peer_bufs])
    with torch.cuda.device(partials.device):
        _lib.check(lib.int4kv_exchange_merge(_p(partials), arr, world, rank, streams, head_dim,
                                             _p(out), _p(status), _stream(partials)),
                   "exchange_merge")
    return out


def rope(x, positions, cos, sin, out=None, status=None):
    """Rotary embedding of rows x [rows, heads, D] at positions [rows] (int4kv_rope)."""
    lib = _lib.load()
    _check_input(x, "x")
    if x.dtype != torch.float32 or x.dim() != 3:
        raise RuntimeError("x must be float32 [rows, heads, head_dim]")
    rows, h, d = x.shape
    _check_input(positions, "positions")
    if positions.dtype != torch.int32 or tuple(positions.shape) != (rows,):
        raise RuntimeError("positions must be int32 [rows]")
    for t, name in ((cos, "rope cos"), (sin, "rope sin")):
        _check_input(t, name)
        if t.dtype != torch.float32 or t.dim() != 2 or t.shape[1] != d // 2:
            raise RuntimeError(f"{name} must be float32 [positions, {d // 2}]")
    if out is None:
        out = torch.empty_like(x)
    _check_input(out, "out")
    _same_device(x, positions, cos, sin, out, status)
    with torch.cuda.device(x.device):
        _lib.check(lib.int4kv_rope(_p(x), _p(positions), rows, h, d, _p(cos), _p(sin),
                                   cos.shape[0], _p(out), _p(status), _stream(x)), "rope")
    return out


def paged_decode_split_bytes(batch, q_heads, head_dim):
    """Bytes of one rank's exchange buffer for the fused split decode."""
    import ctypes
    n = ctypes.c_size_t(0)
    _lib.check(_lib.load().int4kv_paged_decode_split_bytes(batch, q_heads, head_dim,
                                                           ctypes.byref(n)),
               "paged_decode_split_bytes")
    return n.value


def paged_decode_split(query, k_pool, v_pool, sz_pool, block_table, seq_lens, peer_bufs, rank,
                       group_tokens=128, out=None, workspace=None, status=None):
    """The sequence split in one launch (int4kv_paged_decode_split): this rank's
    token range decoded and merged with every rank's records through the peer
    exchange buffers ``peer_bufs`` (addresses in rank order, as mapped here).
    Returns the full attention output [batch, heads, head_dim] float32."""
    import ctypes
    lib = _lib.load()
    num_pages, hkv, page, d = _check_pools(k_pool, v_pool, sz_pool)
    if v_pool is None:
        raise RuntimeError("v_pool is required")
    _check_input(query, "query")
    if query.dtype != torch.float32 or query.dim() != 3:
        raise RuntimeError("query must be float32 [batch, heads, head_dim]")
    b, hq, qd = query.shape
    if qd != d or hq < hkv or hq % hkv:
        raise RuntimeError("query must be [batch, G * kv_heads, pool head_dim]")
    max_pages = _check_table(block_table, b)
    _check_input(seq_lens, "seq_lens")
    if seq_lens.dtype != torch.int32 or tuple(seq_lens.shape) != (b,):
        raise RuntimeError("seq_lens must be int32 [batch]")
    if status is not None and (status.dtype != torch.int32 or status.numel() < 1):
        raise RuntimeError("status must be an int32 tensor")
    _same_device(query, k_pool, v_pool, sz_pool, block_table, seq_lens, out, workspace, status)
    world = len(peer_bufs)
    arr = (ctypes.c_void_p * max(world, 1))(*[int(p) for p in peer_bufs])
    with torch.cuda.device(query.device):
        if out is None:
            out = torch.empty((b, hq, d), dtype=torch.float32, device=query.device)
        elif out.dtype != torch.float32 or tuple(out.shape) != (b, hq, d) or not out.is_contiguous():
            raise RuntimeError("out must be contiguous float32 [batch, heads, head_dim]")
        need = paged_decode_workspace_bytes(b, hq, hkv, d, query.device, v_pool.dtype)
        if workspace is None:
            workspace = torch.zeros((need,), dtype=torch.uint8, device=query.device)
        elif workspace.numel() * workspace.element_size() < need:
            raise RuntimeError(f"workspace needs {need} bytes")
        _lib.check(lib.int4kv_paged_decode_split(
            _p(query), _p(k_pool), _p(v_pool), VALUE_KINDS[v_pool.dtype], _p(sz_pool),
            _p(block_table), _p(seq_lens), b, hq, hkv, d, page, group_tokens, max_pages,
            num_pages, arr, world, rank, _p(out), _p(workspace),
            workspace.numel() * workspace.element_size(), _p(status), _stream(query)),
            "paged_decode_split")
    return out
