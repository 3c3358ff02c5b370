"""Grouped-query attention in the paged decode: query head h of a sequence
attends to kv head h / G (G = query heads / kv heads), the mapping the oracle
(and vLLM's attention backends) use. Gate: float64 arbiter <= 1e-6, and each
query head equals an MHA decode of that head against its kv head.

The kernel serves gs = gcd(G, 4) query heads from each staged page (gs warps
sharing one ring), so the cases cover gs = 1 (G = 3), 2 (G = 2, 6) and 4
(G = 4, 8, 32), with ragged batches whose page runs are shared between ring
groups (the cross-group merge), 16-bit value pools and partial-record mode.
"""

import numpy as np
import pytest

import oracle
from helpers import pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
P = pkg("paged")
C = pkg("_C")

EXACT_TOL = 1e-6


def _cache(lens, hkv, d, seed, value_dtype=torch.float32):
    g = torch.Generator(device="cuda").manual_seed(seed)
    cache = P.PagedKVCache(sum((n + 15) // 16 for n in lens) + 8, hkv, d, device="cuda", seed=seed,
                           value_dtype=value_dtype)
    ks = [torch.randn((n, hkv, d), generator=g, device="cuda") * 2 + 0.5 for n in lens]
    vs = [torch.randn((n, hkv, d), generator=g, device="cuda") for n in lens]
    cache.write_sequences(list(range(len(lens))), ks, vs)
    return cache, g


RAGGED = [2048, 300, 0, 17, 1, 5000, 129, 16, 0, 2047, 777, 64, 3000, 15, 128, 4100]


@pytest.mark.parametrize("group,lens,d,vdt", [
    (4, [2048, 300, 0, 17], 128, torch.float32), (8, [1000, 129], 64, torch.float32),
    (2, [4096], 128, torch.float32), (32, [700, 1], 128, torch.float32),
    (3, [1500, 33, 0], 128, torch.float32), (6, [900, 2048], 64, torch.float32),
    (4, RAGGED, 128, torch.float32), (2, RAGGED, 128, torch.bfloat16),
    (4, [600, 3000], 256, torch.float32), (4, RAGGED[:8], 128, torch.float16)])
def test_gqa_matches_arbiter(group, lens, d, vdt):
    hkv = 2 if group >= 6 else 4
    cache, g = _cache(lens, hkv, d, seed=group + d, value_dtype=vdt)
    q = torch.randn((len(lens), hkv * group, d), generator=g, device="cuda")
    ids = list(range(len(lens)))
    out = cache.decode(q, ids).cpu().numpy()
    bt, sl = cache.block_table(ids)
    exact = oracle.decode_paged(q.cpu().numpy(), cache.k_pool.cpu().numpy(),
                                cache.v_pool.float().cpu().numpy(), cache.sz_pool.cpu().numpy(),
                                bt.cpu().numpy(), sl.cpu().numpy(), method="f64")
    assert np.isfinite(out).all()
    assert np.abs(out - exact).max() <= EXACT_TOL
    for b, n in enumerate(lens):
        if n == 0:
            assert np.all(out[b] == 0)


def test_gqa_head_equals_mha_of_its_kv_head():
    """Query head h of a GQA decode gives the same output as an MHA decode whose
    query h' = h // G of every kv head is that query."""
    group, hkv, d = 4, 2, 128
    cache, g = _cache([1500, 64], hkv, d, seed=5, value_dtype=torch.float16)
    q = torch.randn((2, hkv * group, d), generator=g, device="cuda")
    gqa = cache.decode(q, [0, 1])
    for j in range(group):
        mha = cache.decode(q[:, j::group].contiguous(), [0, 1])  # heads j, G+j -> kv 0, 1
        assert torch.allclose(gqa[:, j::group], mha, rtol=0, atol=EXACT_TOL)


def test_gqa_rejects_ratio_that_is_not_a_multiple():
    cache, g = _cache([32], 4, 64, seed=1)
    with pytest.raises(RuntimeError, match="multiple"):
        cache.decode(torch.randn((1, 6, 64), device="cuda"), [0])


def test_gqa_partial_records_merge_to_the_output():
    """Partial mode with GQA: two token ranges of each sequence decoded into
    records and merged equal the whole decode (records are per query head)."""
    group, hkv, d = 4, 4, 128
    lens = [2048, 1024]
    g = torch.Generator(device="cuda").manual_seed(11)
    ks = [torch.randn((n, hkv, d), generator=g, device="cuda") * 2 + 0.5 for n in lens]
    vs = [torch.randn((n, hkv, d), generator=g, device="cuda") for n in lens]
    q = torch.randn((len(lens), hkv * group, d), generator=g, device="cuda")
    whole = P.PagedKVCache(400, hkv, d, device="cuda", seed=1)
    whole.write_sequences([0, 1], ks, vs)
    want = whole.decode(q, [0, 1])
    parts = []
    for lo, hi in [(0, 0.5), (0.5, 1.0)]:
        c = P.PagedKVCache(400, hkv, d, device="cuda", seed=2)
        c.write_sequences([0, 1], [k[int(lo * n):int(hi * n)] for k, n in zip(ks, lens)],
                          [v[int(lo * n):int(hi * n)] for v, n in zip(vs, lens)])
        bt, sl = c.block_table([0, 1])
        parts.append(C.paged_decode_partials(q, c.k_pool, c.v_pool, c.sz_pool, bt, sl))
    merged = C.merge_partials(torch.stack(parts).contiguous(), len(lens) * hkv * group, d)
    assert float((merged.view_as(want) - want).abs().max()) <= 2e-6
