"""Paged decode where the warp pairs' runs hold many stream boundaries.

Decodes without ring groups run as warp pairs: two warps share one stream-K run
from both ends, claim its middle pages through a shared-memory word, and merge
the stream that holds their meeting point through shared memory. These cases
put many short ragged streams (some empty, some of one token, some page
aligned) into the runs, so pairs finish streams alone, split a stream at the
meeting point, meet exactly on a stream boundary, hold a single page, or get
no page at all (fewer pages than pairs). The bar is the float64 arbiter
evaluated on the stored values (<= 1e-6) and exact zeros for empty sequences,
as for every other decode test.
"""

import numpy as np
import pytest

import oracle
from helpers import pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
P = pkg("paged")

EXACT_TOL = 1e-6


def _lens(kind, seed):
    rng = np.random.default_rng(seed)
    if kind == "fewer_pages_than_pairs":  # 16 sequences of 0..20 tokens
        lens = rng.integers(0, 21, 16)
    elif kind == "about_two_pages_per_pair":  # 64 sequences of 1..48 tokens
        lens = rng.integers(1, 49, 64)
    elif kind == "page_aligned":  # 32 sequences of 16 * (1..40) tokens
        lens = 16 * rng.integers(1, 41, 32)
    else:  # "many_short": 64 sequences of 1..300 tokens, a few empty
        lens = rng.integers(1, 301, 64)
        lens[::13] = 0
    return [int(n) for n in lens]


def _check(lens, heads, d, value_dtype, seed, q_heads=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    cache = P.PagedKVCache(sum((n + 15) // 16 for n in lens) + 8, heads, d, device="cuda",
                           seed=seed, value_dtype=value_dtype)
    ks, vs = [], []
    for n in lens:
        sc = torch.rand((heads, d), generator=g, device="cuda") * 2.5 + 0.5
        off = torch.randn((heads, d), generator=g, device="cuda") * 2.0
        ks.append(torch.randn((n, heads, d), generator=g, device="cuda") * sc + off)
        vs.append(torch.randn((n, heads, d), generator=g, device="cuda"))
    ids = list(range(len(lens)))
    cache.write_sequences(ids, ks, vs)
    q = torch.randn((len(lens), q_heads or heads, d), generator=g, device="cuda")
    out = cache.decode(q, ids).cpu().numpy()
    bt, sl = cache.block_table(ids)
    exact = oracle.decode_paged(q.cpu().numpy(), cache.k_pool.cpu().numpy(),
                                cache.v_pool.float().cpu().numpy(), cache.sz_pool.cpu().numpy(),
                                bt.cpu().numpy(), sl.cpu().numpy(), method="f64")
    assert np.isfinite(out).all()
    err = np.abs(out - exact).max(axis=(1, 2))
    assert err.max() <= EXACT_TOL, [(b, n, float(e)) for b, (n, e) in enumerate(zip(lens, err)) if e > EXACT_TOL]
    for b, n in enumerate(lens):
        if n == 0:
            assert np.all(out[b] == 0)


@pytest.mark.parametrize("kind", ["fewer_pages_than_pairs", "about_two_pages_per_pair",
                                  "page_aligned", "many_short"])
@pytest.mark.parametrize("d", [64, 128])
def test_pairs_ragged_float32(kind, d):
    _check(_lens(kind, seed=d), 8, d, torch.float32, seed=len(kind) + d)


@pytest.mark.parametrize("kind", ["fewer_pages_than_pairs", "about_two_pages_per_pair",
                                  "page_aligned", "many_short"])
@pytest.mark.parametrize("q_heads", [16, 32])
def test_pairs_ragged_grouped_queries(kind, q_heads):
    """Grouped queries over 8 kv heads: G = 2 runs two-head warps, G = 4
    four-head warps, both paired on runs, with the multi-head record merge."""
    _check(_lens(kind, seed=q_heads), 8, 128, torch.float32, seed=len(kind) + q_heads,
           q_heads=q_heads)


@pytest.mark.parametrize("kind", ["about_two_pages_per_pair", "many_short"])
def test_pairs_ragged_float16(kind):
    _check(_lens(kind, seed=5), 8, 128, torch.float16, seed=len(kind))


def test_pairs_repeat_launches_identical():
    """The claims decide which warp takes which middle page, launch by launch;
    the merges are in float64 and exact summation order differences stay far
    below the tolerance, so two launches agree to float32 rounding."""
    lens = _lens("many_short", seed=9)
    g = torch.Generator(device="cuda").manual_seed(9)
    cache = P.PagedKVCache(sum((n + 15) // 16 for n in lens) + 8, 8, 128, device="cuda", seed=9)
    ks = [torch.randn((n, 8, 128), generator=g, device="cuda") for n in lens]
    vs = [torch.randn((n, 8, 128), generator=g, device="cuda") for n in lens]
    ids = list(range(len(lens)))
    cache.write_sequences(ids, ks, vs)
    q = torch.randn((len(lens), 8, 128), generator=g, device="cuda")
    a = cache.decode(q, ids)
    b = cache.decode(q, ids)
    torch.cuda.synchronize()
    assert float((a - b).abs().max()) <= 1e-6


@pytest.mark.parametrize("kind", ["fewer_pages_than_pairs", "many_short"])
@pytest.mark.parametrize("vdtype", ["float16", "bfloat16"])
def test_pairs_ragged_grouped_queries_values16(kind, vdtype):
    _check(_lens(kind, seed=3), 8, 128, getattr(torch, vdtype), seed=len(kind) + 7, q_heads=32)
