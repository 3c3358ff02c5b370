"""The C-ABI library builds, loads and exports every symbol include/*.h declares.

No compute runs here (no GPU needed): only the launchers' host-side argument
checks, which must refuse bad sizes with cudaErrorInvalidValue before any
CUDA call.
"""

import ctypes
import glob
import os
import re

import pytest

from helpers import pkg

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA_ERROR_INVALID_VALUE = 1


def header_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?\w+\s*\*?\s+(\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


@pytest.fixture(scope="module")
def lib():
    build = pkg("_build")
    build.build()
    return pkg("_lib").load()


def test_header_declares_the_reference_launchers():
    names = header_functions()
    assert {"cu_quantize_int4", "cu_flash_decode_int4"} <= names


def test_every_declared_symbol_is_exported(lib):
    names = header_functions()
    assert names, "no declarations parsed"
    for n in sorted(names):
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"
    assert set(pkg("_lib").EXPORTED) == names


def test_build_info(lib):
    assert "sm_100a" in pkg("_lib").build_info()


def test_reference_launchers_reject_bad_sizes(lib):
    n = None
    assert lib.cu_quantize_int4(n, 0, 4, n, n, n, n) == CUDA_ERROR_INVALID_VALUE
    assert lib.cu_quantize_int4(n, 4, -1, n, n, n, n) == CUDA_ERROR_INVALID_VALUE
    # head_dim beyond the kernel limit and non-positive sizes (reference :267-269)
    assert lib.cu_flash_decode_int4(n, n, n, n, n, n, 1, 1, 257, 1, 1, n, n) == CUDA_ERROR_INVALID_VALUE
    assert lib.cu_flash_decode_int4(n, n, n, n, n, n, 1, 1, 0, 1, 1, n, n) == CUDA_ERROR_INVALID_VALUE
    assert lib.cu_flash_decode_int4(n, n, n, n, n, n, 0, 1, 64, 1, 1, n, n) == CUDA_ERROR_INVALID_VALUE
    assert lib.cu_flash_decode_int4(n, n, n, n, n, n, 1, 1, 64, -1, 1, n, n) == CUDA_ERROR_INVALID_VALUE


def test_paged_launchers_reject_bad_sizes(lib):
    n = None
    # head_dim not a multiple of 4
    assert lib.int4kv_quantize_grouped(n, 8, 2, 6, 128, n, n, n, n) == CUDA_ERROR_INVALID_VALUE
    # group longer than 128 rows is not a paged-write group
    assert lib.int4kv_cache_write(n, n, n, n, 1, 16, 2, 64, 256, 16, n, 4, 4, n, n, n, n, n) \
        == CUDA_ERROR_INVALID_VALUE
    # page size other than 16, query heads not a multiple of kv heads
    assert lib.int4kv_paged_decode(n, n, n, n, n, n, 1, 2, 2, 128, 32, 128, 4, 4, n, n, 0, n, n) \
        == CUDA_ERROR_INVALID_VALUE
    assert lib.int4kv_paged_decode(n, n, n, n, n, n, 1, 3, 2, 128, 16, 128, 4, 4, n, n, 0, n, n) \
        == CUDA_ERROR_INVALID_VALUE
    size = ctypes.c_size_t(0)
    assert lib.int4kv_paged_decode_workspace_size(1, 2, 2, 96, ctypes.byref(size)) \
        == CUDA_ERROR_INVALID_VALUE
    # the allocation-free variant checks the same sizes before touching its scratch
    need = ctypes.c_size_t(12345)
    assert lib.int4kv_paged_decode_static_scratch(n, n, n, n, n, n, 1, 3, 2, 128, 16, 128, 4, 4,
                                                  n, n, ctypes.byref(need), n) \
        == CUDA_ERROR_INVALID_VALUE
    assert need.value == 12345
    assert lib.int4kv_dense_decode_workspace_size(1, 1, 300, 1, 1, ctypes.byref(size)) \
        == CUDA_ERROR_INVALID_VALUE


def test_exchange_layout_and_argument_checks(lib):
    par = pkg("parallel")
    for streams, d in [(1, 64), (20, 128), (64, 128), (9, 256), (4096, 128)]:
        size = ctypes.c_size_t(0)
        assert lib.int4kv_exchange_bytes(8, streams, d, ctypes.byref(size)) == 0
        assert size.value == par.exchange_layout(streams, d)["bytes"]
    size = ctypes.c_size_t(0)
    assert lib.int4kv_exchange_bytes(9, 8, 128, ctypes.byref(size)) == CUDA_ERROR_INVALID_VALUE
    assert lib.int4kv_exchange_bytes(2, 8, 96, ctypes.byref(size)) == CUDA_ERROR_INVALID_VALUE
    n = None
    bufs = (ctypes.c_void_p * 2)(4096, 8192)
    # rank outside the world, too many ranks, misaligned peer buffer
    assert lib.int4kv_exchange_merge(n, bufs, 2, 2, 8, 128, n, n, n) == CUDA_ERROR_INVALID_VALUE
    assert lib.int4kv_exchange_merge(n, bufs, 9, 0, 8, 128, n, n, n) == CUDA_ERROR_INVALID_VALUE
    odd = (ctypes.c_void_p * 2)(4096, 8200)
    assert lib.int4kv_exchange_merge(ctypes.c_void_p(4096), odd, 2, 0, 8, 128, ctypes.c_void_p(4096),
                                     n, n) == CUDA_ERROR_INVALID_VALUE
    assert lib.int4kv_ipc_open(n, n) == CUDA_ERROR_INVALID_VALUE


def test_rope_entry_points_reject_bad_arguments(lib):
    n = None
    p = ctypes.c_void_p(4096)
    # head_dim not a multiple of 8, empty table, overlapping in/out
    assert lib.int4kv_rope(p, p, 4, 2, 12, p, p, 8, ctypes.c_void_p(1 << 20), n, n) == CUDA_ERROR_INVALID_VALUE
    assert lib.int4kv_rope(p, p, 4, 2, 64, p, p, 0, ctypes.c_void_p(1 << 20), n, n) == CUDA_ERROR_INVALID_VALUE
    assert lib.int4kv_rope(p, p, 4, 2, 64, p, p, 8, ctypes.c_void_p(4096 + 256), n, n) == CUDA_ERROR_INVALID_VALUE
    assert lib.int4kv_rope(p, p, 0, 2, 64, p, p, 8, p, n, n) == 0  # nothing to do
    # a rope table without its partner, a query without an output
    assert lib.int4kv_cache_append_rope(p, n, p, p, p, 1, 1, 2, 64, 128, 16, p, 4, 4, p, n, 0, p,
                                        p, n, 8, n, n, 0, n, n) == CUDA_ERROR_INVALID_VALUE
    assert lib.int4kv_cache_append_rope(p, n, p, p, p, 1, 1, 2, 64, 128, 16, p, 4, 4, p, n, 0, p,
                                        p, p, 8, p, n, 2, n, n) == CUDA_ERROR_INVALID_VALUE


def test_split_decode_layout_and_argument_checks(lib):
    """int4kv_paged_decode_split_bytes matches the documented buffer layout
    (the offsets tests use to stand in for peers), and the split decode
    rejects a bad world / rank / peer buffer before touching the device."""
    par = pkg("parallel")
    for batch, heads, d in [(1, 32, 128), (1, 8, 64), (4, 6, 256), (2, 1, 128)]:
        size = ctypes.c_size_t(0)
        assert lib.int4kv_paged_decode_split_bytes(batch, heads, d, ctypes.byref(size)) == 0
        assert size.value == par.split_layout(batch * heads, d)["bytes"]
        assert par.split_layout(batch * heads, d)["off_recs"] % 128 == 0
    size = ctypes.c_size_t(0)
    assert lib.int4kv_paged_decode_split_bytes(1, 8, 96, ctypes.byref(size)) == CUDA_ERROR_INVALID_VALUE
    assert lib.int4kv_paged_decode_split_bytes(0, 8, 128, ctypes.byref(size)) == CUDA_ERROR_INVALID_VALUE
    p, n = ctypes.c_void_p(1 << 20), None

    def call(bufs, world, rank):
        return lib.int4kv_paged_decode_split(p, p, p, 0, p, p, p, 1, 8, 8, 128, 16, 128, 4, 4,
                                             bufs, world, rank, p, p, 1 << 20, n, n)

    two = (ctypes.c_void_p * 9)(*([1 << 20] * 9))
    assert call(two, 9, 0) == CUDA_ERROR_INVALID_VALUE      # more than 8 ranks
    assert call(two, 2, 2) == CUDA_ERROR_INVALID_VALUE      # rank outside the world
    assert call(two, 2, -1) == CUDA_ERROR_INVALID_VALUE
    assert call(two, 0, 0) == CUDA_ERROR_INVALID_VALUE      # no ranks
    assert call(n, 2, 0) == CUDA_ERROR_INVALID_VALUE        # no buffer list
    odd = (ctypes.c_void_p * 2)(1 << 20, (1 << 20) + 64)
    assert call(odd, 2, 0) == CUDA_ERROR_INVALID_VALUE      # a peer buffer not 128-byte aligned
    empty = (ctypes.c_void_p * 2)(1 << 20, 0)
    assert call(empty, 2, 1) == CUDA_ERROR_INVALID_VALUE    # a missing peer buffer


def test_benchmark_config_shapes():
    """The benchmark's decode configurations by name, including the grouped-
    query forms at config 0's and config 2's shapes."""
    W = pkg("workloads")
    s = W.config_shape("cfg0")
    assert (s.batch, s.heads, s.query_heads, s.head_dim, s.seq_lens[0]) == (8, 32, 32, 128, 2048)
    assert s.algorithmic_bytes() == 306450432
    g = W.config_shape("cfg0_gqa4")
    assert (g.heads, g.query_heads) == (8, 32)
    l = W.config_shape("cfg2_32768_gqa4")
    assert (l.batch, l.heads, l.query_heads, l.seq_lens[0]) == (8, 8, 32, 32768)
    assert l.pool_pages == 8 * 2048
    m = W.config_shape("cfg2_512")
    assert (m.heads, m.query_heads, m.seq_lens[0]) == (32, 32, 512)
    for bad in ("cfg2_512_gqa5", "cfg0_gqa3", "cfg9"):
        with pytest.raises(ValueError):
            W.config_shape(bad)


def test_benchmark_headline_timing_follows_the_l2_rule():
    """The bench times its headline step back to back (no flush) only where a
    step's inputs are more than twice the 126 MB L2, and says so in `config`;
    smaller configurations keep the L2 flush between steps."""
    import importlib
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if root not in sys.path:
        sys.path.insert(0, root)
    bench = importlib.import_module("bench")
    W = pkg("workloads")
    for name in ("cfg0", "cfg2_8192", "cfg4_long"):
        shape = W.config_shape(name)
        assert shape.algorithmic_bytes() > 2 * 126e6
        assert bench.workload_config(shape, name, 1)["l2"].startswith("not flushed")
    for name in ("cfg2_512", "cfg0_gqa4", "cfg0_gqa8"):
        shape = W.config_shape(name)
        assert shape.algorithmic_bytes() <= 2 * 126e6
        assert bench.workload_config(shape, name, 1)["l2"].startswith("flushed")
