"""Token-by-token appends (int4kv_cache_append) against bulk writes and the oracle.

After every decode-step append, a sequence's open 128-token group is
quantized again over its valid rows -- the reference's rule for a partial
group (min / max over the rows it holds). So after any number of appends the
pools must equal a bulk write of the same tokens bit for bit, and the codes /
scales / zero-points must equal the oracle's grouped quantizer on the whole
key sequence.
"""

import numpy as np
import pytest

import oracle
from helpers import pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
P = pkg("paged")


def _logical(cache, s, group=128):
    """(codes [n, H, D/2], scale/zp [G, H, D], values [n, H, D]) of sequence s in token order."""
    n = cache.lens[s]
    pages = cache.pages[s]
    k = torch.cat([cache.k_pool[p] for p in pages], dim=1)[:, :n].transpose(0, 1)
    v = torch.cat([cache.v_pool[p] for p in pages], dim=1)[:, :n].transpose(0, 1)
    gp = group // 16
    sz = torch.stack([cache.sz_pool[pages[g * gp]] for g in range((n + group - 1) // group)])
    return k.cpu(), sz[:, :, 0].cpu(), sz[:, :, 1].cpu(), v.cpu()


def _tokens(n, heads, d, g):
    sc = torch.rand((heads, d), generator=g, device="cuda") * 2.5 + 0.5
    off = torch.randn((heads, d), generator=g, device="cuda") * 2.0
    return (torch.randn((n, heads, d), generator=g, device="cuda") * sc + off,
            torch.randn((n, heads, d), generator=g, device="cuda"))


@pytest.mark.parametrize("value_dtype", [torch.float32, torch.float16])
def test_appends_equal_bulk_write_and_oracle(value_dtype):
    heads, d = 4, 128
    prefill = [300, 0, 128, 17]
    steps = 150
    g = torch.Generator(device="cuda").manual_seed(1)
    full = [_tokens(n + steps, heads, d, g) for n in prefill]
    inc = P.PagedKVCache(256, heads, d, device="cuda", seed=3, value_dtype=value_dtype,
                         max_open_sequences=2)  # forces the staging pool to grow
    inc.write_sequences(list(range(4)), [k[:n] for (k, _), n in zip(full, prefill)],
                        [v[:n] for (_, v), n in zip(full, prefill)])
    for t in range(steps):
        inc.append(list(range(4)), torch.stack([k[n + t] for (k, _), n in zip(full, prefill)]),
                   torch.stack([v[n + t] for (_, v), n in zip(full, prefill)]))
    bulk = P.PagedKVCache(256, heads, d, device="cuda", seed=9, value_dtype=value_dtype)
    bulk.write_sequences(list(range(4)), [k for k, _ in full], [v for _, v in full])
    for s, (k, _) in enumerate(full):
        a, b = _logical(inc, s), _logical(bulk, s)
        assert torch.equal(a[0], b[0])
        assert torch.equal(a[1].view(torch.int32), b[1].view(torch.int32))
        assert torch.equal(a[2].view(torch.int32), b[2].view(torch.int32))
        assert torch.equal(a[3], b[3])
        q, sc, zp = oracle.quantize_grouped(k.cpu().numpy(), 128)
        np.testing.assert_array_equal(a[0].numpy(), oracle.pack_int4(q))
        np.testing.assert_array_equal(a[1].numpy().view(np.uint32), sc.view(np.uint32))
        np.testing.assert_array_equal(a[2].numpy().view(np.uint32), zp.view(np.uint32))
    # same logical cache -> the decode gives the same bits
    qv = torch.randn((4, heads, d), generator=g, device="cuda")
    assert torch.equal(inc.decode(qv, list(range(4))), bulk.decode(qv, list(range(4))))


def test_append_to_new_sequences_only():
    heads, d = 2, 64
    g = torch.Generator(device="cuda").manual_seed(2)
    cache = P.PagedKVCache(32, heads, d, device="cuda", seed=1)
    ks, vs = _tokens(40, heads, d, g)
    for t in range(40):
        cache.append([7], ks[t:t + 1], vs[t:t + 1])
    assert cache.lens[7] == 40 and len(cache.pages[7]) == 3
    q, sc, zp = oracle.quantize_grouped(ks.cpu().numpy(), 128)
    k, s, z, v = _logical(cache, 7)
    np.testing.assert_array_equal(k.numpy(), oracle.pack_int4(q))
    np.testing.assert_array_equal(s.numpy().view(np.uint32), sc.view(np.uint32))
    assert torch.equal(v, vs.cpu())
