"""The vLLM-style shim (INT4PagedKVCache), device-resident.

Follows the reference's tests/test_vllm_integration.py:13-101 and adds exact
parity: the shim's decode equals the oracle run over the same blocks (keys
quantized per block by the oracle, values rounded through fp16 as the
reference shim stores them).
"""

import numpy as np
import pytest

import oracle
from helpers import pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
V = pkg("vllm_integration")


def test_write_and_decode():
    rng = np.random.RandomState(0)
    cache = V.INT4PagedKVCache(num_blocks=16, block_size=128, head_dim=64)
    for b in range(4):
        cache.write_block(b, rng.randn(128, 64).astype(np.float32), rng.randn(128, 64).astype(np.float32))
    out = cache.decode_attention(rng.randn(2, 4, 64).astype(np.float32), block_table=[0, 1, 2, 3])
    assert out.shape == (2, 4, 64) and np.isfinite(out).all()


@pytest.mark.parametrize("head_dim,rows", [(64, 256), (32, 40), (30, 17), (128, 200)])
def test_decode_matches_oracle(head_dim, rows):
    rng = np.random.RandomState(head_dim)
    cache = V.INT4PagedKVCache(num_blocks=8, block_size=256, head_dim=head_dim)
    ks, vs = [], []
    for b in range(3):
        k = rng.randn(rows if b != 1 else rows // 2 + 1, head_dim).astype(np.float32)
        v = rng.randn(*k.shape).astype(np.float32)
        cache.write_block(b, k, v)
        ks.append(k); vs.append(v)
    q = (rng.randn(1, 2, head_dim) / np.sqrt(head_dim)).astype(np.float32)
    got = cache.decode_attention(q, block_table=[2, 0, 1])
    pages, vals = [], []
    for b in (2, 0, 1):
        qq, s, z = oracle.quantize_int4(ks[b])
        pages.append((qq, s, z))
        vals.append(vs[b].astype(np.float16).astype(np.float32))
    ref, _ = oracle.online_softmax(q, pages, vals)
    assert np.abs(got - ref).max() <= 1e-5


def test_packed_storage_is_real():
    rng = np.random.RandomState(7)
    cache = V.INT4PagedKVCache(num_blocks=4, block_size=128, head_dim=64)
    cache.write_block(0, rng.randn(128, 64).astype(np.float32), rng.randn(128, 64).astype(np.float32))
    assert cache.k_packed[0].nbytes == 128 * 64 // 2
    assert cache.k_packed[0].dtype == torch.uint8 and cache.k_packed[0].is_cuda


def test_free_block():
    cache = V.INT4PagedKVCache(num_blocks=4, block_size=64, head_dim=32)
    k = np.random.randn(64, 32).astype(np.float32)
    cache.write_block(0, k, k)
    cache.free_block(0)
    assert 0 not in cache.k_packed
    assert cache.memory_stats()['blocks'] == 0


def test_memory_compression_ratio():
    cache = V.INT4PagedKVCache(num_blocks=16, block_size=256, head_dim=128)
    for b in range(8):
        k = np.random.randn(256, 128).astype(np.float32)
        cache.write_block(b, k, k)
    assert cache.memory_stats()['ratio'] > 1.5


def test_int4_decode_close_to_fp32():
    rng = np.random.RandomState(1)
    d = 64
    cache = V.INT4PagedKVCache(num_blocks=8, block_size=256, head_dim=d)
    keys, values = [], []
    for b in range(3):
        k = rng.randn(256, d).astype(np.float32)
        v = rng.randn(256, d).astype(np.float32)
        cache.write_block(b, k, v)
        keys.append(k); values.append(v)
    q = (rng.randn(1, 2, d) / np.sqrt(d)).astype(np.float32)
    out = cache.decode_attention(q, block_table=[0, 1, 2])
    kk, vv = np.concatenate(keys), np.concatenate(values)
    lg = q[0] @ kk.T
    p = np.exp(lg - lg.max(-1, keepdims=True))
    fp32 = (p @ vv) / p.sum(-1, keepdims=True)
    assert np.abs(out[0] - fp32).mean() < 0.05


@pytest.mark.parametrize("head_dim,block_size", [(64, 256), (128, 128), (30, 48)])
def test_append_token_equals_write_block(head_dim, block_size):
    """A block filled token by token (each append re-quantizes the block's rows)
    stores exactly what write_block stores for the same rows, at every length."""
    rng = np.random.RandomState(head_dim + block_size)
    k = rng.randn(block_size, head_dim).astype(np.float32) * 2
    v = rng.randn(block_size, head_dim).astype(np.float32)
    inc = V.INT4PagedKVCache(num_blocks=4, block_size=block_size, head_dim=head_dim)
    ref = V.INT4PagedKVCache(num_blocks=4, block_size=block_size, head_dim=head_dim)
    for n in range(block_size):
        inc.append_token(2, k[n], v[n])
        if n in (0, 1, 16, block_size // 2, block_size - 1):
            ref.write_block(2, k[:n + 1], v[:n + 1])
            for name in ("k_packed", "k_scale", "k_zp", "v"):
                a = getattr(inc, name)[2].cpu().numpy()
                b = getattr(ref, name)[2].cpu().numpy()
                np.testing.assert_array_equal(a.view(np.uint8), b.view(np.uint8))
    q = rng.randn(2, 3, head_dim).astype(np.float32)
    np.testing.assert_array_equal(inc.decode_attention(q, [2]), ref.decode_attention(q, [2]))
    with pytest.raises(ValueError, match="full"):
        inc.append_token(2, k[0], v[0])


def test_decode_reads_blocks_in_listed_order_and_skips_nothing():
    """The in-place block decode over a permuted, repeated block list equals the
    oracle over the same list (blocks are read where they are stored)."""
    rng = np.random.RandomState(3)
    d = 64
    cache = V.INT4PagedKVCache(num_blocks=8, block_size=64, head_dim=d)
    blocks = {}
    for b in (5, 0, 3):
        k = rng.randn(64 if b != 3 else 20, d).astype(np.float32)
        v = rng.randn(*k.shape).astype(np.float32)
        cache.write_block(b, k, v)
        blocks[b] = (k, v)
    table = [3, 5, 0, 5]
    q = (rng.randn(2, 2, d) / 8).astype(np.float32)
    got = cache.decode_attention(q, table)
    pages, vals = [], []
    for b in table:
        k, v = blocks[b]
        qk, s, z = oracle.quantize_int4(k)
        pages.append((qk, s, z))
        vals.append(v.astype(np.float16).astype(np.float32))
    exact = oracle.attention_f64(q, pages, vals)
    assert np.abs(got - exact).max() <= 1e-6
