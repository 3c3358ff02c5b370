"""The paged decode storing its output straight into mapped pinned host
memory (zero-copy), as the benchmark's end-to-end leg uses it: the output
pointer of int4kv_paged_decode_ex may be any address the device can store
to. Checked against the same decode into device memory, through the C ABI."""

import ctypes

import numpy as np
import pytest

from helpers import pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
rt = pytest.importorskip("cuda.bindings.runtime")
W = pkg("workloads")
C = pkg("_C")


def _decode(lib, shape, query, cache, bt, sl, out_ptr, ws, ws_bytes):
    stream = torch.cuda.current_stream().cuda_stream
    vk = C.VALUE_KINDS[cache.v_pool.dtype]
    rc = lib.int4kv_paged_decode_ex(
        query.data_ptr(), cache.k_pool.data_ptr(), cache.v_pool.data_ptr(), vk,
        cache.sz_pool.data_ptr(), bt.data_ptr(), sl.data_ptr(), shape.batch, shape.query_heads,
        shape.heads, shape.head_dim, 16, shape.group_tokens, bt.shape[1], cache.num_pages,
        ctypes.c_void_p(out_ptr), ws.data_ptr(), ws_bytes, None, ctypes.c_void_p(stream),
        None, None)
    assert rc == 0, f"int4kv_paged_decode_ex: cudaError {rc}"


@pytest.mark.parametrize("batch,heads,q_heads,lens,vdtype", [
    (8, 32, None, [2048] * 8, "float32"),                 # config 0's shape
    (5, 8, 32, [300, 0, 4096, 17, 1], "float32"),         # grouped queries, ragged, empty
    (3, 4, None, [129, 2000, 16], "float16"),
])
def test_decode_output_to_mapped_host_memory(batch, heads, q_heads, lens, vdtype):
    pkg("_build").build()
    lib = pkg("_lib").load()
    shape = W.DecodeShape(batch, heads, 128, lens, pool_pages=sum((n + 15) // 16 for n in lens) + 8,
                          q_heads=q_heads)
    prob = W.torch_build_cache(shape, seed=batch + heads, value_dtype=getattr(torch, vdtype))
    cache, query = prob["cache"], prob["query"]
    bt, sl = cache.block_table(list(range(batch)))
    ws_bytes = C.paged_decode_workspace_bytes(batch, shape.query_heads, heads, 128,
                                              value_dtype=cache.v_pool.dtype)
    ws = torch.zeros((ws_bytes,), dtype=torch.uint8, device="cuda")
    out = torch.full_like(query, float("nan"))
    nbytes = out.numel() * 4
    err, hptr = rt.cudaHostAlloc(nbytes, rt.cudaHostAllocMapped)
    assert err == rt.cudaError_t.cudaSuccess
    try:
        err, dptr = rt.cudaHostGetDevicePointer(hptr, 0)
        assert err == rt.cudaError_t.cudaSuccess
        host = np.frombuffer((ctypes.c_uint8 * nbytes).from_address(hptr), dtype=np.float32)
        host[:] = np.nan
        _decode(lib, shape, query, cache, bt, sl, out.data_ptr(), ws, ws_bytes)
        for _ in range(2):  # two calls in a row into the same mapped buffer
            _decode(lib, shape, query, cache, bt, sl, dptr, ws, ws_bytes)
            torch.cuda.synchronize()
            got = host.reshape(tuple(out.shape)).copy()
            ref = out.cpu().numpy()
            assert np.isfinite(got).all()
            np.testing.assert_allclose(got, ref, rtol=0, atol=1e-6)
            for b, n in enumerate(lens):
                if n == 0:
                    assert np.all(got[b] == 0)
    finally:
        rt.cudaFreeHost(hptr)


@pytest.mark.parametrize("nbytes", [16, 4112, 135200, 3 << 20])
def test_stage_inputs_from_mapped_host_memory(nbytes):
    """int4kv_stage_inputs copies mapped pinned host memory into device memory
    with SM loads; a second call after the host rewrote the buffer sees the
    new bytes (no stale copy cached on the device)."""
    pkg("_build").build()
    lib = pkg("_lib").load()
    err, hptr = rt.cudaHostAlloc(nbytes, rt.cudaHostAllocMapped)
    assert err == rt.cudaError_t.cudaSuccess
    try:
        err, dptr = rt.cudaHostGetDevicePointer(hptr, 0)
        assert err == rt.cudaError_t.cudaSuccess
        host = np.frombuffer((ctypes.c_uint8 * nbytes).from_address(hptr), dtype=np.uint8)
        dev = torch.zeros((nbytes,), dtype=torch.uint8, device="cuda")
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rng = np.random.default_rng(nbytes)
        for _ in range(2):
            host[:] = rng.integers(0, 256, nbytes, dtype=np.uint8)
            rc = lib.int4kv_stage_inputs(ctypes.c_void_p(dev.data_ptr()), ctypes.c_void_p(dptr),
                                         nbytes, stream)
            assert rc == 0, f"int4kv_stage_inputs: cudaError {rc}"
            torch.cuda.synchronize()
            assert np.array_equal(dev.cpu().numpy(), host)
    finally:
        rt.cudaFreeHost(hptr)


def test_stage_inputs_rejects_unaligned_arguments():
    pkg("_build").build()
    lib = pkg("_lib").load()
    err, hptr = rt.cudaHostAlloc(4096, rt.cudaHostAllocMapped)
    assert err == rt.cudaError_t.cudaSuccess
    try:
        err, dptr = rt.cudaHostGetDevicePointer(hptr, 0)
        assert err == rt.cudaError_t.cudaSuccess
        dev = torch.full((4096,), 7, dtype=torch.uint8, device="cuda")
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        d = dev.data_ptr()
        for dst, src, n in [(d, dptr, 40), (d + 8, dptr, 64), (d, dptr + 4, 64), (d, dptr, 0),
                            (0, dptr, 64), (d, 0, 64)]:
            rc = lib.int4kv_stage_inputs(ctypes.c_void_p(dst), ctypes.c_void_p(src), n, stream)
            assert rc == 1  # cudaErrorInvalidValue, nothing launched
        torch.cuda.synchronize()
        assert bool((dev == 7).all())
    finally:
        rt.cudaFreeHost(hptr)
