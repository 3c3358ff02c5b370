"""int4kv_paged_decode_static_scratch: the paged decode with its scratch in a
fixed device array, called through the C ABI, against int4kv_paged_decode
(caller-provided workspace) on the same inputs.

Named to be collected last, so it runs both after the rest of the suite and,
on its own, in a fresh process (the entry point's first call on the device does
its set-up there).
"""

import ctypes

import numpy as np
import pytest

from helpers import pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
W = pkg("workloads")
C = pkg("_C")

CUDA_ERROR_INVALID_VALUE = 1
STATIC_SCRATCH_BYTES = 8 << 20  # INT4KV_STATIC_SCRATCH_BYTES
TOL = 1e-6  # both paths run the same kernel; the bar is the decode's own f64-arbiter tolerance


def _lib():
    pkg("_build").build()
    return pkg("_lib").load()


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _problem(batch, heads, d, lens, seed, q_heads=None):
    shape = W.DecodeShape(batch, heads, d, lens, pool_pages=sum((n + 15) // 16 for n in lens) + 16,
                          q_heads=q_heads)
    prob = W.torch_build_cache(shape, seed=seed)
    cache = prob["cache"]
    bt, sl = cache.block_table(list(range(batch)))
    return shape, prob["query"], cache, bt, sl


def _args(shape, query, cache, bt, sl):
    return (_p(query), _p(cache.k_pool), _p(cache.v_pool), _p(cache.sz_pool), _p(bt), _p(sl),
            shape.batch, shape.query_heads, shape.heads, shape.head_dim, 16, shape.group_tokens,
            bt.shape[1], cache.num_pages)


def _workspace_bytes(shape):
    return C.paged_decode_workspace_bytes(shape.batch, shape.query_heads, shape.heads,
                                          shape.head_dim)


def _existing(lib, shape, query, cache, bt, sl):
    out = torch.full_like(query, float("nan"))
    ws_bytes = _workspace_bytes(shape)
    ws = torch.zeros((ws_bytes,), dtype=torch.uint8, device=query.device)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.int4kv_paged_decode(*_args(shape, query, cache, bt, sl), _p(out), _p(ws), ws_bytes,
                                 None, ctypes.c_void_p(stream))
    assert rc == 0, f"int4kv_paged_decode: cudaError {rc}"
    torch.cuda.synchronize()
    return out


def _static(lib, shape, query, cache, bt, sl):
    out = torch.full_like(query, float("nan"))
    status = torch.zeros((1,), dtype=torch.int32, device=query.device)
    need = ctypes.c_size_t(0)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.int4kv_paged_decode_static_scratch(*_args(shape, query, cache, bt, sl), _p(out),
                                                _p(status), ctypes.byref(need),
                                                ctypes.c_void_p(stream))
    assert rc == 0, f"int4kv_paged_decode_static_scratch: cudaError {rc}"
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    # a call that fits reports exactly the workspace the existing entry point asks for
    assert need.value == _workspace_bytes(shape)
    assert 0 < need.value <= STATIC_SCRATCH_BYTES
    return out


@pytest.mark.parametrize("batch,heads,d,lens,q_heads", [
    (8, 32, 128, [2048] * 8, None),               # config-0 shape
    (5, 4, 128, [300, 0, 4096, 17, 1], None),     # ragged, with an empty sequence
    (3, 8, 64, [129, 2000, 16], None),
    (4, 8, 128, [1500, 0, 2048, 77], 32),         # grouped-query: 32 query heads over 8 kv heads
])
def test_static_scratch_matches_existing_entry_point(batch, heads, d, lens, q_heads):
    lib = _lib()
    shape, query, cache, bt, sl = _problem(batch, heads, d, lens, seed=batch * 100 + d,
                                           q_heads=q_heads)
    ref = _existing(lib, shape, query, cache, bt, sl).cpu().numpy()
    first = _static(lib, shape, query, cache, bt, sl).cpu().numpy()
    second = _static(lib, shape, query, cache, bt, sl).cpu().numpy()  # two calls in a row
    assert np.isfinite(ref).all()
    np.testing.assert_allclose(first, ref, rtol=0, atol=TOL)
    np.testing.assert_allclose(second, ref, rtol=0, atol=TOL)
    for b, n in enumerate(lens):
        if n == 0:
            assert np.all(first[b] == 0) and np.all(second[b] == 0)


def test_static_scratch_rejects_launches_beyond_its_capacity():
    """8192 streams at head_dim 256 need more than the fixed scratch holds: the
    call is refused before any launch and reports the bytes it would need. The
    buffers are nonetheless a complete, valid problem (one 16-token page per
    sequence)."""
    lib = _lib()
    batch, heads, d = 256, 32, 256
    dev = torch.device("cuda")
    query = torch.zeros((batch, heads, d), device=dev)
    k_pool = torch.zeros((batch, heads, 16, d // 2), dtype=torch.uint8, device=dev)
    v_pool = torch.zeros((batch, heads, 16, d), device=dev)
    sz_pool = torch.zeros((batch, heads, 2, d), device=dev)
    bt = torch.arange(batch, dtype=torch.int32, device=dev).view(batch, 1)
    sl = torch.full((batch,), 16, dtype=torch.int32, device=dev)
    out = torch.full_like(query, 7.0)
    need = ctypes.c_size_t(0)
    rc = lib.int4kv_paged_decode_static_scratch(
        _p(query), _p(k_pool), _p(v_pool), _p(sz_pool), _p(bt), _p(sl), batch, heads, heads, d,
        16, 16, 1, batch, _p(out), None, ctypes.byref(need),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rc == CUDA_ERROR_INVALID_VALUE
    assert need.value > STATIC_SCRATCH_BYTES
    assert bool((out == 7.0).all()), "a refused call must not launch"
    # the refused call left the scratch usable: the next call that fits matches
    # the existing entry point
    shape, query, cache, bt, sl = _problem(3, 4, 128, [600, 33, 0], seed=5)
    ref = _existing(lib, shape, query, cache, bt, sl).cpu().numpy()
    got = _static(lib, shape, query, cache, bt, sl).cpu().numpy()
    np.testing.assert_allclose(got, ref, rtol=0, atol=TOL)
