"""Edge cases of the paged path beyond the benchmark shapes.

* quantization groups of 64 and 32 tokens (the reference sweeps 64-token
  groups: README "use 64-token groups (+0.238%)"), oracle-built pools and a
  GPU-written cache, against the float64 arbiter;
* the largest batch the decode takes (4096 sequences: the per-CTA length
  prefix fills its shared-memory table), ragged and partly empty;
* malformed lengths (negative, longer than the block-table row) are clamped
  and reported in the status word, never read past the row.
"""

import numpy as np
import pytest

import oracle
from helpers import oracle_build_pools, pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
C = pkg("_C")
P = pkg("paged")
W = pkg("workloads")
ops = pkg("ops")

TOL = 1e-6
BAD_LENGTH = 2


@pytest.mark.parametrize("group,d,lens", [(64, 128, [700, 64, 0, 65, 1]), (32, 64, [333, 32, 31]),
                                          (16, 128, [100, 17])])
def test_small_groups_match_arbiter(group, d, lens):
    prob = W.np_paged_problem(len(lens), 3, d, lens,
                              pool_pages=sum((n + 15) // 16 for n in lens) + 5, seed=group + d,
                              group=group)
    pools = oracle_build_pools(prob)
    got = ops.flash_decode_paged(prob["query"], *pools, prob["block_table"], prob["seq_lens"],
                                 group)
    exact = oracle.decode_paged(prob["query"], *pools, prob["block_table"], prob["seq_lens"],
                                group_pages=group // 16, method="f64")
    assert np.isfinite(got).all()
    assert np.abs(got - exact).max() <= TOL


@pytest.mark.parametrize("group", [64, 32])
def test_small_groups_gpu_written_cache(group):
    """The GPU writer with short groups gives the oracle's codes and parameters,
    and the decode over it matches the arbiter."""
    heads, d, lens = 2, 128, [300, 40]
    g = torch.Generator(device="cuda").manual_seed(group)
    ks = [torch.randn((n, heads, d), generator=g, device="cuda") * 2 + 1 for n in lens]
    vs = [torch.randn((n, heads, d), generator=g, device="cuda") for n in lens]
    cache = P.PagedKVCache(64, heads, d, group_tokens=group, device="cuda", seed=3)
    cache.write_sequences([0, 1], ks, vs)
    q = torch.randn((2, heads, d), generator=g, device="cuda")
    out = cache.decode(q, [0, 1]).cpu().numpy()
    bt, sl = cache.block_table([0, 1])
    exact = oracle.decode_paged(q.cpu().numpy(), cache.k_pool.cpu().numpy(),
                                cache.v_pool.cpu().numpy(), cache.sz_pool.cpu().numpy(),
                                bt.cpu().numpy(), sl.cpu().numpy(), group_pages=group // 16,
                                method="f64")
    assert np.abs(out - exact).max() <= TOL
    # codes / scales are the oracle's grouped quantizer with the same group
    for s, k in enumerate(ks):
        n = lens[s]
        pages = cache.pages[s]
        codes = torch.cat([cache.k_pool[p] for p in pages], dim=1)[:, :n].transpose(0, 1).cpu().numpy()
        q_, sc, zp = oracle.quantize_grouped(k.cpu().numpy(), group)
        np.testing.assert_array_equal(codes, oracle.pack_int4(q_))
        gp = group // 16
        got_sc = np.stack([cache.sz_pool[pages[i * gp], :, 0].cpu().numpy()
                           for i in range(sc.shape[0])])
        np.testing.assert_array_equal(got_sc.view(np.uint32), sc.view(np.uint32))


def test_largest_batch():
    batch, heads, d = 4096, 2, 64
    rng = np.random.default_rng(5)
    lens = rng.integers(0, 41, batch).tolist()
    lens[0], lens[-1] = 0, 40
    prob = W.np_paged_problem(batch, heads, d, lens,
                              pool_pages=sum((n + 15) // 16 for n in lens) + 16, seed=5)
    pools = oracle_build_pools(prob)
    got = ops.flash_decode_paged(prob["query"], *pools, prob["block_table"], prob["seq_lens"])
    sample = [(int(b), int(h)) for b, h in zip(rng.integers(0, batch, 64), rng.integers(0, heads, 64))]
    exact = oracle.decode_paged(prob["query"], *pools, prob["block_table"], prob["seq_lens"],
                                method="f64", streams=sample)
    assert np.isfinite(got).all()
    assert max(float(np.abs(got[b, h] - exact[b, h]).max()) for b, h in sample) <= TOL
    empty = np.asarray(lens) == 0
    assert np.all(got[empty] == 0)


def test_lengths_beyond_the_row_are_clamped_and_reported():
    lens = [40, 20]
    prob = W.np_paged_problem(2, 2, 128, lens, pool_pages=8, seed=9)
    k_pool, v_pool, sz_pool = oracle_build_pools(prob)
    dev = "cuda"
    bt = torch.from_numpy(prob["block_table"]).to(dev)  # [2, 3] pages
    t = lambda a: torch.from_numpy(a).to(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    bad = torch.tensor([40 + 1000, -5], dtype=torch.int32, device=dev)
    out = C.paged_decode(t(prob["query"]), t(k_pool), t(v_pool), t(sz_pool), bt, bad,
                         status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & BAD_LENGTH
    o = out.cpu().numpy()
    assert np.isfinite(o).all()
    assert np.all(o[1] == 0)  # a negative length decodes as empty
    # the long one is clamped to its row: the decode of the row's 48 slots
    cap = bt.shape[1] * 16
    exact = oracle.decode_paged(prob["query"], k_pool, v_pool, sz_pool, prob["block_table"],
                                np.array([cap, 0], np.int32), method="f64")
    assert np.abs(o[0] - exact[0]).max() <= TOL
