"""Paged decode with 16-bit value pools (float16 / bfloat16), through the C ABI.

The cache write rounds each value to nearest even as it stores it (checked
bit for bit against torch's own conversion); the decode widens the stored
values to float32 exactly, so the bar is the float64 arbiter evaluated on the
stored (16-bit) values: <= 1e-6, as for float32 values.
"""

import numpy as np
import pytest

import oracle
from helpers import pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
C = pkg("_C")
P = pkg("paged")
W = pkg("workloads")

EXACT_TOL = 1e-6
DTYPES = [torch.float16, torch.bfloat16]


def _problem(lens, heads, d, value_dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    cache = P.PagedKVCache(sum((n + 15) // 16 for n in lens) + 8, heads, d, device="cuda",
                           seed=seed, value_dtype=value_dtype)
    ks, vs = [], []
    for n in lens:
        sc = torch.rand((heads, d), generator=g, device="cuda") * 2.5 + 0.5
        off = torch.randn((heads, d), generator=g, device="cuda") * 2.0
        ks.append(torch.randn((n, heads, d), generator=g, device="cuda") * sc + off)
        vs.append(torch.randn((n, heads, d), generator=g, device="cuda"))
    cache.write_sequences(list(range(len(lens))), ks, vs)
    q = torch.randn((len(lens), heads, d), generator=g, device="cuda")
    return cache, ks, vs, q


def _host_pools(cache, ids):
    bt, sl = cache.block_table(ids)
    return (cache.k_pool.cpu().numpy(), cache.v_pool.float().cpu().numpy(),
            cache.sz_pool.cpu().numpy(), bt.cpu().numpy(), sl.cpu().numpy())


@pytest.mark.parametrize("value_dtype", DTYPES)
@pytest.mark.parametrize("d,lens", [(128, [2048, 300, 0, 17]), (64, [1000, 129]), (256, [400, 16])])
def test_values16_decode_matches_arbiter(value_dtype, d, lens):
    cache, ks, vs, q = _problem(lens, 4, d, value_dtype, seed=d + len(lens))
    ids = list(range(len(lens)))
    out = cache.decode(q, ids).cpu().numpy()
    kp, vp, sp, bt, sl = _host_pools(cache, ids)
    exact = oracle.decode_paged(q.cpu().numpy(), kp, vp, sp, bt, sl, method="f64")
    assert np.isfinite(out).all()
    assert np.abs(out - exact).max() <= EXACT_TOL
    for b, n in enumerate(lens):
        if n == 0:
            assert np.all(out[b] == 0)


@pytest.mark.parametrize("value_dtype", DTYPES)
def test_values16_stored_with_round_to_nearest_even(value_dtype):
    lens = [300, 45]
    cache, ks, vs, q = _problem(lens, 2, 128, value_dtype, seed=3)
    for b, (n, v) in enumerate(zip(lens, vs)):
        pages = cache.pages[b]
        got = torch.cat([cache.v_pool[p] for p in pages], dim=1)[:, :n]  # [heads, n, d]
        want = v.to(value_dtype).transpose(0, 1)
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("value_dtype", DTYPES)
def test_values16_keys_identical_to_float32_cache(value_dtype):
    """The key side (codes, scales, zero-points) does not depend on the value type."""
    lens = [777, 128]
    c16, ks, vs, q = _problem(lens, 2, 128, value_dtype, seed=11)
    c32, *_ = _problem(lens, 2, 128, torch.float32, seed=11)
    assert torch.equal(c16.k_pool, c32.k_pool)
    assert torch.equal(c16.sz_pool.view(torch.int32), c32.sz_pool.view(torch.int32))


def test_values16_full_anchor_config():
    """Config-0 shape with float16 values: every stream within 1e-6 of the arbiter
    on a sample, and the whole output finite."""
    shape = W.config_shape("cfg0")
    prob = W.torch_build_cache(shape, seed=5, value_dtype=torch.float16)
    cache, q = prob["cache"], prob["query"]
    ids = list(range(shape.batch))
    out = cache.decode(q, ids).cpu().numpy()
    assert np.isfinite(out).all()
    kp, vp, sp, bt, sl = _host_pools(cache, ids)
    rng = np.random.default_rng(0)
    streams = [(int(b), int(h)) for b, h in zip(rng.integers(0, shape.batch, 6),
                                               rng.integers(0, shape.heads, 6))]
    exact = oracle.decode_paged(q.cpu().numpy(), kp, vp, sp, bt, sl, method="f64", streams=streams)
    for b, h in streams:
        assert np.abs(out[b, h] - exact[b, h]).max() <= EXACT_TOL


@pytest.mark.parametrize("value_dtype", [torch.float16, torch.bfloat16])
def test_sequence_split_partials_with_16bit_values(value_dtype):
    """Partial records of two group-aligned token ranges over 16-bit value pools
    merge to the whole-sequence decode (the sequence split's per-GPU step)."""
    heads, d, L = 4, 128, 3000
    g = torch.Generator(device="cuda").manual_seed(21)
    k = torch.randn((L, heads, d), generator=g, device="cuda") * 2 + 0.5
    v = torch.randn((L, heads, d), generator=g, device="cuda")
    q = torch.randn((1, heads, d), generator=g, device="cuda")
    whole = P.PagedKVCache(L // 16 + 8, heads, d, device="cuda", seed=1, value_dtype=value_dtype)
    whole.write_sequences([0], [k], [v])
    want = whole.decode(q, [0])
    parts = []
    for t0, t1 in [(0, 1280), (1280, L)]:
        c = P.PagedKVCache(L // 16 + 8, heads, d, device="cuda", seed=2, value_dtype=value_dtype)
        c.write_sequences([0], [k[t0:t1]], [v[t0:t1]])
        bt, sl = c.block_table([0])
        parts.append(C.paged_decode_partials(q, c.k_pool, c.v_pool, c.sz_pool, bt, sl))
    merged = C.merge_partials(torch.stack(parts).contiguous(), heads, d)
    assert float((merged.view_as(want) - want).abs().max()) <= 2e-6
