"""GPU parity of the multi-GPU building blocks, on one B200.

* partial mode of the paged decode (``int4kv_paged_decode_partials``) and the
  merge kernel (``int4kv_merge_partials``): a sequence split into the split
  plan's ranges, each range decoded into partial records, merged -- against
  the whole-sequence decode and the float64 arbiter;
* batch x head shards (``plan_batch_heads``) decoded shard by shard and
  reassembled, against the whole-batch decode.

The ranges / shards run as independent launches on one GPU (no kernel waits
on another); the NCCL exchange itself is covered by the gloo tests on CPU and
by ``tests/dist_sequence_split.py`` under torchrun on several GPUs.
"""

import numpy as np
import pytest

import oracle
from helpers import pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
C = pkg("_C")
P = pkg("paged")
par = pkg("parallel")

TOL = 1e-6  # vs the float64 arbiter, as for the one-GPU decode


def _seq(L, heads, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    sc = torch.rand((heads, d), generator=g, device="cuda") * 2.5 + 0.5
    off = torch.randn((heads, d), generator=g, device="cuda") * 2.0
    k = torch.randn((L, heads, d), generator=g, device="cuda") * sc + off
    v = torch.randn((L, heads, d), generator=g, device="cuda")
    q = torch.randn((1, heads, d), generator=g, device="cuda")
    return q, k, v


def _cache(k, v, heads, d, seed):
    n = k.shape[0]
    cache = P.PagedKVCache((n + 15) // 16 + 8, heads, d, device="cuda", seed=seed)
    cache.write_sequences([0], [k], [v])
    return cache


def _host(cache, ids):
    bt, sl = cache.block_table(ids)
    return (cache.k_pool.cpu().numpy(), cache.v_pool.cpu().numpy(), cache.sz_pool.cpu().numpy(),
            bt.cpu().numpy(), sl.cpu().numpy())


@pytest.mark.parametrize("L,heads,d,world", [(5000, 8, 128, 3), (131072 // 8, 4, 128, 8),
                                             (1000, 4, 64, 2), (300, 2, 256, 4),
                                             (200, 4, 128, 8)])
def test_sequence_split_partials_merge(L, heads, d, world):
    q, k, v = _seq(L, heads, d, seed=L + d)
    full = _cache(k, v, heads, d, seed=1)
    want = full.decode(q, [0])
    ranges = par.plan_sequence_split(L, world)
    recs = []
    for r, (t0, t1) in enumerate(ranges):
        cache = P.PagedKVCache((t1 - t0 + 15) // 16 + 8, heads, d, device="cuda", seed=10 + r)
        cache.write_sequences([0], [k[t0:t1]], [v[t0:t1]])
        bt, sl = cache.block_table([0])
        recs.append(C.paged_decode_partials(q, cache.k_pool, cache.v_pool, cache.sz_pool, bt, sl))
    gathered = torch.stack(recs)  # [world, heads * record], as the all-gather lays it out
    got = C.merge_partials(gathered, heads, d).view(1, heads, d)
    torch.cuda.synchronize()
    arb = oracle.decode_paged(q.cpu().numpy(), *_host(full, [0]), method="f64")
    g = got.cpu().numpy()
    assert np.isfinite(g).all()
    assert np.abs(g - arb).max() <= TOL
    assert np.abs(g - want.cpu().numpy()).max() <= 2 * TOL
    # the host restatement of the merge gives the same result from the same records
    rec = gathered.cpu().numpy().reshape(world, heads, 16 + 4 * d)
    m = rec[..., :8].copy().view(np.float64)[..., 0]
    lsum = rec[..., 8:16].copy().view(np.float64)[..., 0]
    acc = rec[..., 16:].copy().view(np.float32)
    host = oracle.merge_partials(m, lsum, acc)
    assert np.abs(host - g[0]).max() <= TOL


def test_partial_records_of_a_batch():
    """Normalizing each record by its l gives the plain decode; an empty
    sequence gives the empty record (-inf, 0, 0)."""
    heads, d = 4, 128
    lens = [700, 0, 16, 2100]
    cache = P.PagedKVCache(sum((n + 15) // 16 for n in lens) + 8, heads, d, device="cuda", seed=3)
    g = torch.Generator(device="cuda").manual_seed(5)
    for b, n in enumerate(lens):
        cache.write_sequences([b], [torch.randn((n, heads, d), generator=g, device="cuda") * 2],
                              [torch.randn((n, heads, d), generator=g, device="cuda")])
    q = torch.randn((len(lens), heads, d), generator=g, device="cuda")
    bt, sl = cache.block_table(list(range(len(lens))))
    parts = C.paged_decode_partials(q, cache.k_pool, cache.v_pool, cache.sz_pool, bt, sl)
    want = cache.decode(q, list(range(len(lens)))).cpu().numpy()
    rec = parts.cpu().numpy().reshape(len(lens), heads, 16 + 4 * d)
    m = rec[..., :8].copy().view(np.float64)[..., 0]
    lsum = rec[..., 8:16].copy().view(np.float64)[..., 0]
    acc = rec[..., 16:].copy().view(np.float32)
    assert np.all(m[1] == -np.inf) and np.all(lsum[1] == 0) and np.all(acc[1] == 0)
    live = [0, 2, 3]
    got = acc[live] / lsum[live][..., None]
    assert np.abs(got - want[live]).max() <= TOL
    # single-part merge through the kernel reproduces the decode (empty -> zeros)
    merged = C.merge_partials(parts.view(1, -1), len(lens) * heads, d).view(len(lens), heads, d)
    mg = merged.cpu().numpy()
    assert np.abs(mg - want).max() <= TOL and np.all(mg[1] == 0)


def test_batch_head_shards_reassemble():
    heads, d = 8, 128
    lens = [3000, 17, 0, 900, 4096, 128]
    world = 4
    g = torch.Generator(device="cuda").manual_seed(9)
    ks = [torch.randn((n, heads, d), generator=g, device="cuda") * 1.5 for n in lens]
    vs = [torch.randn((n, heads, d), generator=g, device="cuda") for n in lens]
    q = torch.randn((len(lens), heads, d), generator=g, device="cuda")
    full = P.PagedKVCache(sum((n + 15) // 16 for n in lens) + 8, heads, d, device="cuda", seed=2)
    full.write_sequences(list(range(len(lens))), ks, vs)
    want = full.decode(q, list(range(len(lens)))).cpu().numpy()
    got = np.full_like(want, np.nan)
    for shard in par.plan_batch_heads(lens, heads, world):
        if not shard.units:
            continue
        w = shard.width
        local = P.PagedKVCache(sum((lens[b] + 15) // 16 for b, _ in shard.units) + 8, w, d,
                               device="cuda", seed=20 + shard.rank)
        local.write_sequences(list(range(len(shard.units))),
                              [ks[b][:, h0:h0 + w] for b, h0 in shard.units],
                              [vs[b][:, h0:h0 + w] for b, h0 in shard.units])
        lq = torch.stack([q[b, h0:h0 + w] for b, h0 in shard.units]).contiguous()
        out = local.decode(lq, list(range(len(shard.units)))).cpu().numpy()
        for i, (b, h0) in enumerate(shard.units):
            got[b, h0:h0 + w] = out[i]
    assert np.isfinite(got).all()
    assert np.abs(got - want).max() <= 2 * TOL


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 or more GPUs")
@pytest.mark.parametrize("exchange", ["nccl", "p2p", "fused"])
def test_sequence_split_across_gpus(exchange):
    import os
    import subprocess
    import sys
    n = min(torch.cuda.device_count(), 8)
    script = os.path.join(os.path.dirname(os.path.abspath(__file__)), "dist_sequence_split.py")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "300", sys.executable, "-m",
                        "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
                        "--master-addr", "127.0.0.1", "--master-port", str(29531 + ["nccl", "p2p", "fused"].index(exchange)), script,
                        "32768", "8", exchange], capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
