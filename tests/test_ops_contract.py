"""Operator-surface contract that holds without a GPU.

Follows the reference's dispatch tests (tests/test_ops_dispatch.py:90-251):
malformed input raises the same ValueError texts, a named backend is
delivered or refused, the empty cache returns exact zeros. Differences from
the reference are deliberate: no Triton/Pallas/NumPy backends exist here, so
they are refused, and nothing falls back to a CPU path.
"""

import numpy as np
import pytest

import oracle
from helpers import pkg

ops = pkg("ops")


def _paged_problem(batch=2, heads=3, dim=32, n_blocks=3, rows=64, seed=0):
    rng = np.random.RandomState(seed)
    query = (rng.randn(batch, heads, dim) / np.sqrt(dim)).astype(np.float32)
    kq, ks, kz, vv = [], [], [], []
    for _ in range(n_blocks):
        k = rng.randn(rows, dim).astype(np.float32)
        v = rng.randn(rows, dim).astype(np.float32)
        q, s, z = oracle.quantize_int4(k)
        kq.append(q); ks.append(s); kz.append(z); vv.append(v)
    return query, kq, ks, kz, vv


class TestInputContract:
    def test_block_len_longer_than_page(self):
        q, kq, ks, kz, vv = _paged_problem()
        with pytest.raises(ValueError, match="outside"):
            ops.flash_decode(q, kq, ks, kz, vv, np.array([64, 65, 64]))

    def test_negative_block_len(self):
        q, kq, ks, kz, vv = _paged_problem()
        with pytest.raises(ValueError, match="outside"):
            ops.flash_decode(q, kq, ks, kz, vv, np.array([64, -1, 64]))

    def test_wrong_number_of_block_lens(self):
        q, kq, ks, kz, vv = _paged_problem()
        with pytest.raises(ValueError, match="entries"):
            ops.flash_decode(q, kq, ks, kz, vv, np.array([64, 64]))

    def test_mismatched_page_lists(self):
        q, kq, ks, kz, vv = _paged_problem()
        with pytest.raises(ValueError, match="same length"):
            ops.flash_decode(q, kq, ks, kz, vv[:-1])

    def test_value_page_shape(self):
        q, kq, ks, kz, vv = _paged_problem()
        vv[1] = vv[1][:-3]
        with pytest.raises(ValueError, match="value page 1"):
            ops.flash_decode(q, kq, ks, kz, vv)

    def test_key_page_head_dim(self):
        q, kq, ks, kz, vv = _paged_problem(dim=32)
        with pytest.raises(ValueError, match="key page"):
            ops.flash_decode(q[:, :, :16], kq, ks, kz, vv)

    def test_scale_shape(self):
        q, kq, ks, kz, vv = _paged_problem()
        ks[2] = ks[2][:-1]
        with pytest.raises(ValueError, match="scale/zero-point for page 2"):
            ops.flash_decode(q, kq, ks, kz, vv)

    def test_non_3d_query(self):
        q, kq, ks, kz, vv = _paged_problem()
        with pytest.raises(ValueError, match="query must be"):
            ops.flash_decode(q[0], kq, ks, kz, vv)

    def test_empty_cache_returns_exact_zeros(self):
        q, _, _, _, _ = _paged_problem()
        out = ops.flash_decode(q, [], [], [], [])
        assert out.shape == q.shape and out.dtype == np.float32
        np.testing.assert_array_equal(out, np.zeros_like(q))


class TestBackendSelection:
    def _args(self):
        q, kq, ks, kz, vv = _paged_problem(1, 2, 16, 1, 32)
        return (q, kq, ks, kz, vv, np.array([32], np.int32))

    def test_attention_rejects_triton(self):
        with pytest.raises(ValueError, match="no Triton attention kernel"):
            ops.flash_decode(*self._args(), backend="triton")

    @pytest.mark.parametrize("name", ["nonsense", "pallas", "reference"])
    def test_attention_rejects_other_backends(self, name):
        with pytest.raises(ValueError, match="unknown backend"):
            ops.flash_decode(*self._args(), backend=name)

    @pytest.mark.parametrize("name", ["nonsense", "triton", "pallas", "reference"])
    def test_quantize_rejects_other_backends(self, name):
        kv = np.random.RandomState(1).randn(32, 8).astype(np.float32)
        with pytest.raises(ValueError, match="unknown backend"):
            ops.quantize_int4(kv, backend=name)

    def test_declared_backends(self):
        assert ops.QUANTIZE_BACKENDS == ("cuda",)
        assert ops.ATTENTION_BACKENDS == ("cuda",)
        assert ops.CUDA_MAX_HEAD_DIM == 256

    def test_no_cpu_path(self):
        kv = np.random.RandomState(2).randn(16, 8).astype(np.float32)
        with pytest.raises(ValueError, match="CPU path"):
            ops.quantize_int4(kv, use_cuda=False)
        with pytest.raises(ValueError, match="CPU path"):
            ops.flash_decode(*self._args(), use_cuda=False)

    @pytest.mark.skipif(ops.HAS_CUDA, reason="needs a host without a usable GPU")
    def test_missing_gpu_raises_instead_of_falling_back(self):
        kv = np.random.RandomState(3).randn(16, 8).astype(np.float32)
        with pytest.raises(RuntimeError, match="CUDA backend requested"):
            ops.quantize_int4(kv)
        with pytest.raises(RuntimeError, match="CUDA backend requested"):
            ops.flash_decode(*self._args())

    def test_backend_status_keys(self):
        st = ops.backend_status()
        for k in ("has_torch", "has_cuda", "has_triton", "has_jax", "jax_devices",
                  "pallas_interpret_default", "active_backend", "available_backends"):
            assert k in st
        assert st["has_triton"] is False and st["has_jax"] is False
