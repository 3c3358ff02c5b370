"""Operator surface: the reference's ``src/ops.py`` API, backed by sm_100a kernels.

Same entry points, argument meaning and return types as the reference
(src/ops.py:86-344): ``quantize_int4``, ``flash_decode``,
``prepare_quantize_int4_cuda``, ``prepare_flash_decode_cuda``,
``backend_status``, the backend tuples, ``CUDA_MAX_HEAD_DIM`` and the
``HAS_*`` flags. Plus the paged-cache operators the benchmark configurations
need: ``quantize_int4_grouped``, ``flash_decode_paged`` and their
``prepare_*`` forms.

Deliberate differences from the reference's dispatch:

* One backend: ``"cuda"`` (B200 kernels). There is no Triton, no Pallas and no
  CPU path in this framework. ``backend="triton"`` for attention raises the
  reference's own "no Triton attention kernel" error; every other name,
  ``"reference"`` included, raises "unknown backend". The NumPy reference is
  the test oracle, not a backend.
* No silent fallback: where the reference's auto-detect falls back to NumPy
  (non-2-D quantizer input, src/ops.py:155-161; head_dim > 256,
  src/ops.py:245-246; extension missing), this module raises.
"""

from typing import List, Optional, Tuple

import numpy as np

from ._prepared import PreparedCall
from ._validate import normalize_attention_inputs
from . import _lib

try:
    import torch
    HAS_TORCH = True
except ImportError:  # pragma: no cover - torch is a hard dependency in practice
    torch = None
    HAS_TORCH = False

HAS_JAX = False  # no JAX / Pallas path in this framework


def _cuda_ready() -> bool:
    return HAS_TORCH and _lib.available() and torch.cuda.is_available()


HAS_CUDA = _cuda_ready()
if HAS_TORCH:
    from . import _C
else:  # pragma: no cover
    _C = None

#: Backends implementing each op in this framework.
QUANTIZE_BACKENDS = ("cuda",)
ATTENTION_BACKENDS = ("cuda",)

#: The shared-stream attention kernel's head_dim limit (reference src/ops.py:166).
CUDA_MAX_HEAD_DIM = 256


def _validate_backend(backend: Optional[str], supported: tuple, op: str) -> None:
    """A named backend is delivered or refused -- never substituted (src/ops.py:90-108)."""
    if backend is None or backend in supported:
        return
    if backend == "triton" and op == "attention":
        raise ValueError(
            "no Triton attention kernel exists in this framework -- it has no Triton code at "
            "all. Use backend='cuda' (the B200 kernels).")
    raise ValueError(
        f"unknown backend {backend!r} for {op}; supported: {supported}. This framework runs "
        "only its sm_100a CUDA kernels; the NumPy reference is its test oracle, not a backend.")


def _require_cuda(use_cuda: Optional[bool]) -> None:
    if use_cuda is False:
        raise ValueError("use_cuda=False asks for a CPU path, which this framework does not have")
    if not HAS_CUDA:
        why = "libint4kv_b200.so is not built" if not _lib.available() else "no CUDA device is visible"
        raise RuntimeError(f"CUDA backend requested but unavailable: {why}. "
                           "Build with __graft_entry__.build() and run on a B200.")


def _cuda_sync(_out) -> None:
    torch.cuda.synchronize()


def _to_device_f32(a):
    if isinstance(a, torch.Tensor):
        return a.to(device="cuda", dtype=torch.float32).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


# --------------------------------------------------------------------------
# quantizer
# --------------------------------------------------------------------------

def quantize_int4(kv: np.ndarray, use_cuda: Optional[bool] = None,
                  backend: Optional[str] = None,
                  interpret: Optional[bool] = None) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per-channel asymmetric INT4 over all rows of kv[rows, channels].

    Returns (q uint8 [rows, channels] one code per byte, scale [channels],
    zp [channels]) as NumPy, bit-identical to the reference oracle.
    ``interpret`` is accepted for signature compatibility and ignored.
    """
    _validate_backend(backend, QUANTIZE_BACKENDS, "quantize")
    _require_cuda(use_cuda)
    if np.ndim(kv) != 2:
        raise ValueError(
            f"the CUDA quantizer takes a 2D [rows, channels] array, got shape {np.shape(kv)}. "
            "Use quantize_int4_grouped() for [tokens, heads, head_dim] keys.")
    return prepare_quantize_int4_cuda(kv)()


def prepare_quantize_int4_cuda(kv) -> PreparedCall:
    """Stage kv on the GPU once; run() is one kernel launch."""
    _require_cuda(None)
    kv_t = _to_device_f32(kv)
    return PreparedCall(run=lambda: _C.quantize_int4(kv_t), sync=_cuda_sync,
                        to_numpy=lambda out: tuple(t.cpu().numpy() for t in out))


def quantize_int4_grouped(kv, group_tokens: int = 128):
    """Keys [tokens, heads, head_dim] -> (packed [tokens, heads, head_dim/2] u8,
    scale [groups, heads, head_dim], zp [groups, heads, head_dim]) as NumPy.

    One scale/zero-point per (group of ``group_tokens`` tokens, head, channel),
    two codes per byte (even channel in the low nibble).
    """
    return prepare_quantize_int4_grouped(kv, group_tokens)()


def prepare_quantize_int4_grouped(kv, group_tokens: int = 128) -> PreparedCall:
    _require_cuda(None)
    kv_t = _to_device_f32(kv)
    return PreparedCall(run=lambda: _C.quantize_int4_grouped(kv_t, group_tokens), sync=_cuda_sync,
                        to_numpy=lambda out: tuple(t.cpu().numpy() for t in out))


# --------------------------------------------------------------------------
# shared-stream attention (the reference's flash_decode)
# --------------------------------------------------------------------------

def flash_decode(query: np.ndarray, k_q_blocks: List[np.ndarray], k_scales: List[np.ndarray],
                 k_zps: List[np.ndarray], v_blocks: List[np.ndarray],
                 block_lens: Optional[np.ndarray] = None, use_cuda: Optional[bool] = None,
                 backend: Optional[str] = None, interpret: Optional[bool] = None) -> np.ndarray:
    """Fused online-softmax attention over INT4 pages (reference src/ops.py:176-253).

    Every query in [batch, heads] attends over the SAME page stream (the
    reference's interface). Returns float32 [batch, heads, head_dim].
    """
    _validate_backend(backend, ATTENTION_BACKENDS, "attention")
    query, block_lens = normalize_attention_inputs(query, k_q_blocks, k_scales, k_zps, v_blocks,
                                                   block_lens)
    if len(k_q_blocks) == 0:
        # attention over an empty cache: no mass accumulated -> exact zeros
        return np.zeros(query.shape, dtype=np.float32)
    _require_cuda(use_cuda)
    if query.shape[2] > CUDA_MAX_HEAD_DIM:
        raise ValueError(
            f"the CUDA attention kernel supports head_dim <= {CUDA_MAX_HEAD_DIM}, got "
            f"{query.shape[2]}; this framework has no other attention backend")
    return prepare_flash_decode_cuda(query, k_q_blocks, k_scales, k_zps, v_blocks, block_lens)()


def prepare_flash_decode_cuda(query, k_q_blocks, k_scales, k_zps, v_blocks,
                              block_lens=None) -> PreparedCall:
    """Validate, pad pages to a dense [nb, rows, D] layout and stage on the GPU once."""
    _require_cuda(None)
    query, block_lens = normalize_attention_inputs(query, k_q_blocks, k_scales, k_zps, v_blocks,
                                                   block_lens)
    nb = len(k_q_blocks)
    dim = query.shape[2]
    if nb == 0:
        zeros = np.zeros(query.shape, dtype=np.float32)
        return PreparedCall(run=lambda: zeros)
    if dim > CUDA_MAX_HEAD_DIM:
        raise ValueError(f"the CUDA attention kernel supports head_dim <= {CUDA_MAX_HEAD_DIM}, "
                         f"got {dim}")
    rows = max(np.shape(b)[0] for b in k_q_blocks)
    kq = np.zeros((nb, rows, dim), np.uint8)
    vv = np.zeros((nb, rows, dim), np.float32)
    for i in range(nb):
        n = np.shape(k_q_blocks[i])[0]
        kq[i, :n] = k_q_blocks[i]
        vv[i, :n] = v_blocks[i]
    sc = np.ascontiguousarray(np.stack(k_scales), dtype=np.float32)
    zp = np.ascontiguousarray(np.stack(k_zps), dtype=np.float32)
    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda()
           for a in (query.astype(np.float32), kq, sc, zp, vv, block_lens.astype(np.int32))]
    return PreparedCall(run=lambda: _C.flash_decode_int4(*dev), sync=_cuda_sync,
                        to_numpy=lambda out: out.cpu().numpy())


# --------------------------------------------------------------------------
# paged attention (per-(sequence, kv-head) streams, benchmark configs 0/2/3/4)
# --------------------------------------------------------------------------

def prepare_flash_decode_paged(query, k_pool, v_pool, sz_pool, block_table, seq_lens,
                               group_tokens: int = 128) -> PreparedCall:
    """Stage a paged problem on the GPU once; run() is the decode + combine launch pair.

    Arrays may be NumPy (copied to the GPU) or CUDA tensors (used in place).
    Layout: see ``paged.PagedKVCache``.
    """
    _require_cuda(None)

    def dev(a, dtype):
        if isinstance(a, torch.Tensor):
            return a.to(device="cuda", dtype=dtype).contiguous()
        return torch.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype)

    q = dev(query, torch.float32)
    kp = dev(k_pool, torch.uint8)
    vp = dev(v_pool, torch.float32)
    sp = dev(sz_pool, torch.float32)
    bt = dev(block_table, torch.int32)
    sl = dev(seq_lens, torch.int32)
    out = torch.empty_like(q)
    ws = torch.zeros((_C.paged_decode_workspace_bytes(q.shape[0], q.shape[1], kp.shape[1],
                                                      q.shape[2], q.device),),
                     dtype=torch.uint8, device=q.device)
    return PreparedCall(
        run=lambda: _C.paged_decode(q, kp, vp, sp, bt, sl, group_tokens, out=out, workspace=ws),
        sync=_cuda_sync, to_numpy=lambda o: o.cpu().numpy())


def flash_decode_paged(query, k_pool, v_pool, sz_pool, block_table, seq_lens,
                       group_tokens: int = 128) -> np.ndarray:
    """INT4 paged decode attention; returns float32 [batch, heads, head_dim] as NumPy."""
    return prepare_flash_decode_paged(query, k_pool, v_pool, sz_pool, block_table, seq_lens,
                                      group_tokens)()


def backend_status() -> dict:
    """Backend availability, with the reference's keys (src/ops.py:316-344)."""
    return {
        'has_torch': HAS_TORCH,
        'has_cuda': HAS_CUDA,
        'has_triton': False,
        'has_jax': HAS_JAX,
        'jax_devices': [],
        'pallas_interpret_default': False,
        'active_backend': 'cuda' if HAS_CUDA else 'none',
        'available_backends': ['cuda'] if HAS_CUDA else [],
        'library': _lib.LIB_PATH if _lib.available() else None,
    }
