"""Grouped-query attention in the paged decode: query head h of a sequence
attends to kv head h / G (G = query heads / kv heads), the mapping the oracle
(and vLLM's attention backends) use. Gate: float64 arbiter <= 1e-6, and each
query head equals an MHA decode of that head against its kv head.
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


@pytest.mark.parametrize("group,lens,d", [(4, [2048, 300, 0, 17], 128), (8, [1000, 129], 64),
                                          (2, [4096], 128), (32, [700, 1], 128)])
def test_gqa_matches_arbiter(group, lens, d):
    hkv = 2 if group == 32 else 4
    cache, g = _cache(lens, hkv, d, seed=group + d)
    q = torch.randn((len(lens), hkv * group, d), generator=g, device="cuda")
    ids = list(range(len(lens)))
    out = cache.decode(q, ids).cpu().numpy()
    bt, sl = cache.block_table(ids)
    exact = oracle.decode_paged(q.cpu().numpy(), cache.k_pool.cpu().numpy(),
                                cache.v_pool.cpu().numpy(), cache.sz_pool.cpu().numpy(),
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
