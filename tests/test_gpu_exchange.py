"""GPU checks of the fused peer exchange (``int4kv_exchange_merge``) on one B200.

The kernel pushes this rank's partial records into every rank's exchange
buffer, raises its per-chunk flags there, waits for the other ranks' flags in
its own buffer and merges. On one GPU the other ranks are stood in for by
writes from the host side (torch ops on the same stream, before the launch):
their records and flags are already in the buffer when the kernel starts, so
no kernel ever waits on another launch. The result must equal
``int4kv_merge_partials`` over the same records bit for bit (same float64
arithmetic in the same rank order), and the kernel's own pushes must land in
the stand-in peers' buffers at the documented offsets.

A flag that nothing sets exercises the bounded wait: the kernel gives up after
2 s, reports INT4KV_STATUS_PEER_TIMEOUT and writes NaN, and the context stays
usable. The multi-process path runs in ``tests/dist_sequence_split.py`` on
several GPUs.
"""

import numpy as np
import pytest

from helpers import pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
C = pkg("_C")
par = pkg("parallel")

PEER_TIMEOUT = 8


def _records(world, streams, d, seed):
    """[world, streams * record] uint8: m f64 (some -inf), l f64 > 0, acc f32."""
    rng = np.random.default_rng(seed)
    rec = par.partial_record_bytes(d)
    out = np.zeros((world, streams, rec), dtype=np.uint8)
    for r in range(world):
        for s in range(streams):
            empty = (r + s) % 5 == 3
            m = -np.inf if empty else rng.normal() * 4.0
            l = 0.0 if empty else rng.uniform(0.5, 300.0)
            acc = np.zeros(d, np.float32) if empty else rng.normal(size=d).astype(np.float32) * l
            out[r, s, 0:8] = np.frombuffer(np.float64(m).tobytes(), np.uint8)
            out[r, s, 8:16] = np.frombuffer(np.float64(l).tobytes(), np.uint8)
            out[r, s, 16:] = np.frombuffer(acc.tobytes(), np.uint8)
    return torch.from_numpy(out.reshape(world, -1)).cuda()


class _Buffers:
    def __init__(self, world, streams, d):
        self.lay = par.exchange_layout(streams, d)
        n = C.exchange_bytes(world, streams, d)
        assert n == self.lay["bytes"]
        self.ptrs = [C.exchange_alloc(torch.cuda.current_device(), n) for _ in range(world)]
        self.views = [par.device_bytes(p, n, "cuda") for p in self.ptrs]

    def recs(self, buf, parity, src, streams):
        lay = self.lay
        o = lay["off_recs"] + (parity * par.EXCHANGE_MAX_RANKS + src) * streams * lay["record"]
        return self.views[buf][o:o + streams * lay["record"]]

    def flags(self, buf, parity, src):
        lay = self.lay
        o = lay["off_flag"] + (parity * par.EXCHANGE_MAX_RANKS + src) * lay["chunks"] * 4
        return self.views[buf][o:o + lay["chunks"] * 4].view(torch.int32)

    def steps(self, buf):
        return self.views[buf][:self.lay["chunks"] * 4].view(torch.int32)

    def free(self):
        torch.cuda.synchronize()
        for p in self.ptrs:
            C.exchange_free(p)


@pytest.mark.parametrize("world,streams,d", [(1, 32, 128), (2, 20, 64), (4, 20, 128),
                                             (8, 9, 256), (3, 64, 128)])
def test_exchange_matches_merge(world, streams, d):
    bufs = _Buffers(world, streams, d)
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    out = torch.empty((streams, d), dtype=torch.float32, device="cuda")
    try:
        for step in (1, 2, 3):
            parity = step & 1
            parts = _records(world, streams, d, seed=100 * world + step)
            # the other ranks' pushes and flags, as they would arrive over NVLink
            for src in range(1, world):
                bufs.recs(0, parity, src, streams).copy_(parts[src])
                bufs.flags(0, parity, src).fill_(step)
            C.exchange_merge(parts[0].contiguous(), bufs.ptrs, 0, streams, d, out, status)
            want = C.merge_partials(parts.contiguous(), streams, d)
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            assert torch.equal(out, want), float((out - want).abs().max())
            # this rank's own pushes landed in every rank's buffer, flags raised
            for dst in range(world):
                assert torch.equal(bufs.recs(dst, parity, 0, streams), parts[0])
                assert bool((bufs.flags(dst, parity, 0) == step).all())
            assert bool((bufs.steps(0) == step).all())
    finally:
        bufs.free()


def test_exchange_peer_timeout_is_reported():
    world, streams, d = 2, 16, 128
    bufs = _Buffers(world, streams, d)
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    out = torch.zeros((streams, d), dtype=torch.float32, device="cuda")
    try:
        parts = _records(world, streams, d, seed=7)
        # rank 1 never arrives: its flags in rank 0's buffer stay 0
        C.exchange_merge(parts[0].contiguous(), bufs.ptrs, 0, streams, d, out, status)
        torch.cuda.synchronize()
        assert int(status.item()) & PEER_TIMEOUT
        assert bool(torch.isnan(out).all())
        # the context is still usable
        want = C.merge_partials(parts.contiguous(), streams, d)
        torch.cuda.synchronize()
        assert bool(torch.isfinite(want).all())
    finally:
        bufs.free()


def test_peer_exchange_single_rank_decoder():
    """SequenceSplitDecoder(exchange='p2p') at world 1 equals the plain decode."""
    P = pkg("paged")
    heads, d, L = 8, 128, 3000
    g = torch.Generator(device="cuda").manual_seed(5)
    k = torch.randn((L, heads, d), generator=g, device="cuda") * 2.0 + 0.5
    v = torch.randn((L, heads, d), generator=g, device="cuda")
    q = torch.randn((1, heads, d), generator=g, device="cuda")
    cache = P.PagedKVCache((L + 15) // 16 + 4, heads, d, device="cuda", seed=1)
    cache.write_sequences([0], [k], [v])
    dec = par.SequenceSplitDecoder(cache, 0, 1, exchange="p2p")
    try:
        got = dec.decode(q).clone()
        want = cache.decode(q, [0])
        torch.cuda.synchronize()
        assert dec.peer_status() == 0
        assert float((got - want).abs().max()) <= 2e-6
    finally:
        dec.close()


# ---------------------------------------------------------------------------
# the fused split decode: decode + exchange + merge in one launch
# ---------------------------------------------------------------------------

def _split_caches(L, heads, d, world, seed):
    P = pkg("paged")
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn((L, heads, d), generator=g, device="cuda") * 2.0 + 0.5
    v = torch.randn((L, heads, d), generator=g, device="cuda")
    caches = []
    for t0, t1 in par.plan_sequence_split(L, world):
        c = P.PagedKVCache((t1 - t0 + 15) // 16 + 4, heads, d, device="cuda", seed=t0)
        c.write_sequences([0], [k[t0:t1]], [v[t0:t1]])
        caches.append(c)
    whole = P.PagedKVCache((L + 15) // 16 + 4, heads, d, device="cuda", seed=1)
    whole.write_sequences([0], [k], [v])
    return caches, whole, g


@pytest.mark.parametrize("world,our,L,heads,d", [(2, 0, 3000, 8, 128), (4, 2, 2000, 4, 64),
                                                 (8, 7, 700, 4, 128), (3, 1, 5000, 2, 256)])
def test_fused_split_equals_merge(world, our, L, heads, d):
    """Rank `our` runs the fused kernel on its token range; the other ranks'
    records and flags are written into its buffer beforehand. Output = the
    merge of all ranks' partial records, bit for bit (and the whole-sequence
    decode to rounding); its own records land in every rank's buffer. With
    (8, 7, 700) rank 7's range is empty, so only the empty-stream path runs."""
    caches, whole, g = _split_caches(L, heads, d, world, seed=world + d)
    lay = par.split_layout(heads, d)
    n = C.paged_decode_split_bytes(1, heads, d)
    assert n == lay["bytes"]
    ptrs = [C.exchange_alloc(torch.cuda.current_device(), n) for _ in range(world)]
    views = [par.device_bytes(p, n, "cuda") for p in ptrs]
    rec = lay["record"]

    def recs(buf, parity, src):
        o = lay["off_recs"] + (parity * par.EXCHANGE_MAX_RANKS + src) * heads * rec
        return views[buf][o:o + heads * rec]

    def flags(buf, parity, src):
        o = lay["off_flag"] + (parity * par.EXCHANGE_MAX_RANKS + src) * heads * 4
        return views[buf][o:o + heads * 4].view(torch.int32)

    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    try:
        for step in (1, 2, 3):
            parity = step & 1
            q = torch.randn((1, heads, d), generator=g, device="cuda")
            parts = []
            for c in caches:
                bt, sl = c.block_table([0])
                parts.append(C.paged_decode_partials(q, c.k_pool, c.v_pool, c.sz_pool, bt, sl))
            for r in range(world):  # the others' pushes, as they would arrive over NVLink
                if r != our:
                    recs(our, parity, r).copy_(parts[r])
                    flags(our, parity, r).fill_(step)
            me = caches[our]
            bt, sl = me.block_table([0])
            # buffer order: rank r's buffer at index r (ours is `our`)
            out = C.paged_decode_split(q, me.k_pool, me.v_pool, me.sz_pool, bt, sl, ptrs, our,
                                       status=status)
            want = C.merge_partials(torch.stack(parts).contiguous(), heads, d).view(1, heads, d)
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            assert torch.equal(out, want), float((out - want).abs().max())
            assert float((out - whole.decode(q, [0])).abs().max()) <= 2e-6
            for dst in range(world):  # our record and flag reached every rank's buffer
                assert torch.equal(recs(dst, parity, our), parts[our])
                assert bool((flags(dst, parity, our) == step).all())
    finally:
        torch.cuda.synchronize()
        for p in ptrs:
            C.exchange_free(p)


def test_fused_split_peer_timeout_is_reported():
    caches, _, g = _split_caches(1000, 4, 128, 2, seed=3)
    n = C.paged_decode_split_bytes(1, 4, 128)
    ptrs = [C.exchange_alloc(torch.cuda.current_device(), n) for _ in range(2)]
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    try:
        me = caches[0]
        bt, sl = me.block_table([0])
        q = torch.randn((1, 4, 128), generator=g, device="cuda")
        out = C.paged_decode_split(q, me.k_pool, me.v_pool, me.sz_pool, bt, sl, ptrs, 0,
                                   status=status)  # rank 1 never arrives
        torch.cuda.synchronize()
        assert int(status.item()) & PEER_TIMEOUT
        assert bool(torch.isnan(out).all())
        assert bool(torch.isfinite(me.decode(q, [0])).all())  # the context is still usable
    finally:
        torch.cuda.synchronize()
        for p in ptrs:
            C.exchange_free(p)
