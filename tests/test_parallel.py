"""Multi-GPU host logic on CPU: shard planning, the sequence-split exchange on
gloo ranks (world size 2), and host-side failure detection.

The GPU kernels are replaced here by the oracle's partial softmax state
(checker side); what is under test is the product's planning, record
exchange and liveness logic, and the merge arithmetic the merge kernel
implements (restated in the oracle from the reference's warp merge).
"""

import multiprocessing as mp
import os
import socket
import time

import numpy as np
import pytest

import oracle
from helpers import oracle_build_pools, pkg

par = pkg("parallel")
W = pkg("workloads")


# ---------------- planning ----------------

@pytest.mark.parametrize("lens,heads,world", [
    ([2048] * 8, 32, 1), ([2048] * 8, 32, 2), ([2048] * 8, 32, 8), ([4096] * 256, 32, 8),
    ([100, 5000, 0, 16384, 7, 300, 12000], 32, 4), ([131072], 32, 8), ([3000, 10], 32, 8),
    ([5, 6, 7], 32, 8), ([16384] * 3, 8, 5), ([], 32, 4), ([0, 0], 4, 2),
])
def test_plan_batch_heads_covers_every_stream_once(lens, heads, world):
    shards = par.plan_batch_heads(lens, heads, world)
    assert [s.rank for s in shards] == list(range(world))
    seen = {}
    for s in shards:
        assert heads % s.width == 0 if s.units else True
        for b, h0 in s.units:
            for h in range(h0, h0 + s.width):
                assert (b, h) not in seen, f"stream {(b, h)} on ranks {seen[(b, h)]} and {s.rank}"
                seen[(b, h)] = s.rank
    assert set(seen) == {(b, h) for b in range(len(lens)) for h in range(heads)}
    # greedy longest-first: no rank exceeds the lightest by more than one unit's cost
    loads = [s.bytes for s in shards]
    if lens:
        unit_max = max(par.stream_bytes(n, 128) for n in lens) * shards[0].width
        assert max(loads) - min(loads) <= unit_max
    # whole sequences whenever there are at least as many as ranks
    if len(lens) >= world:
        assert all(s.width == heads for s in shards)


def test_plan_batch_heads_weak_scaling_is_even():
    """cfg0 per GPU x N: 8N equal sequences on N ranks -> 8 whole sequences each."""
    for n in (1, 2, 4, 8):
        shards = par.plan_batch_heads([2048] * (8 * n), 32, n)
        assert all(len(s.units) == 8 and s.width == 32 for s in shards)
        assert len({s.bytes for s in shards}) == 1


@pytest.mark.parametrize("L,world", [(131072, 2), (131072, 8), (1000, 3), (128, 4), (0, 2),
                                     (130, 2), (16384 + 5, 7)])
def test_plan_sequence_split_group_aligned(L, world):
    ranges = par.plan_sequence_split(L, world)
    assert len(ranges) == world
    assert ranges[0][0] == 0 and ranges[-1][1] == L
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    for t0, t1 in ranges:
        assert t0 <= t1 and t0 % 128 == 0
        assert t1 == L or t1 % 128 == 0
    groups = [-(-(t1 - t0) // 128) for t0, t1 in ranges]
    assert max(groups) - min(groups) <= 1 and sum(groups) == -(-L // 128)


def test_plan_rejects_bad_arguments():
    with pytest.raises(ValueError):
        par.plan_batch_heads([10], 0, 2)
    with pytest.raises(ValueError):
        par.plan_batch_heads([-1], 4, 2)
    with pytest.raises(ValueError):
        par.plan_sequence_split(100, 0)
    with pytest.raises(ValueError):
        par.plan_sequence_split(100, 2, group_tokens=20)


def test_split_decoder_and_exchange_reject_bad_modes():
    """Checked on the host before any device work: the exchange mode names
    and the exchange's rank limit."""
    class _Cache:  # what the constructor reads before it allocates
        head_dim, heads, device = 128, 8, "cpu"
    with pytest.raises(ValueError, match="exchange must be"):
        par.SequenceSplitDecoder(_Cache(), 0, 2, exchange="allgather")
    with pytest.raises(ValueError, match="1..8 ranks"):
        par.PeerExchange(0, 9, 8, 128, "cpu")
    lay = par.split_layout(8, 128)
    assert lay["off_flag"] % 128 == 0 and lay["off_recs"] % 128 == 0
    assert lay["bytes"] == lay["off_recs"] + 2 * par.EXCHANGE_MAX_RANKS * 8 * lay["record"]


# ---------------- merge arithmetic (oracle restatement) ----------------

def _split_problem(L, heads=4, d=64, world=3, seed=0):
    """One sequence of L tokens, and the same sequence cut into the split plan's
    ranges, each range laid out as its own paged problem (as each rank holds it)."""
    rng = np.random.default_rng(seed)
    keys = W.np_anchor_keys(rng, L, heads, d)
    vals = rng.standard_normal((L, heads, d)).astype(np.float32)
    query = rng.standard_normal((1, heads, d)).astype(np.float32)

    def pools(k, v, seed2):
        n = k.shape[0]
        prob = {"query": query, "keys": [k], "values": [v], "pool_pages": (n + 15) // 16 + 3,
                "group": 128, "seq_lens": np.array([n], np.int32)}
        prob["block_table"] = W.np_block_table(np.random.default_rng(seed2), [n],
                                               prob["pool_pages"])
        kp, vp, sp = oracle_build_pools(prob)
        return kp, vp, sp, prob["block_table"], prob["seq_lens"]

    full = pools(keys, vals, 1)
    parts = [pools(keys[t0:t1], vals[t0:t1], 10 + r)
             for r, (t0, t1) in enumerate(par.plan_sequence_split(L, world))]
    return query, full, parts


def test_oracle_merge_of_split_equals_full_decode():
    query, full, parts = _split_problem(1000, world=3)
    ref = oracle.decode_paged(query, *full, method="f64")
    states = [oracle.decode_paged_state(query, *p) for p in parts]
    merged = oracle.merge_partials([s[0] for s in states], [s[1] for s in states],
                                   [s[2] for s in states])
    # float32 states of disjoint ranges, merged in float64, vs one float64 softmax
    assert np.abs(merged - ref).max() <= 2e-5
    assert np.abs(merged - oracle.decode_paged(query, *full)).max() <= 2e-5


def test_oracle_merge_skips_empty_parts():
    m = np.array([[-np.inf], [1.0], [-np.inf]])
    l = np.array([[0.0], [2.0], [0.0]])
    acc = np.array([[[0.0, 0.0]], [[4.0, 6.0]], [[0.0, 0.0]]])
    np.testing.assert_array_equal(oracle.merge_partials(m, l, acc), [[2.0, 3.0]])
    # all parts empty -> zeros (the reference's 0 / max(0, 1e-10))
    np.testing.assert_array_equal(oracle.merge_partials(m[[0]], l[[0]], acc[[0]]), [[0.0, 0.0]])


# ---------------- gloo ranks ----------------

def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _pack(m, l, acc):
    """Records in the C ABI's layout: [m f64][l f64][acc f32 x D] per stream."""
    n, d = m.size, acc.shape[-1]
    rec = np.zeros((n, 16 + 4 * d), np.uint8)
    rec[:, 0:8] = m.reshape(n).astype(np.float64).view(np.uint8).reshape(n, 8)
    rec[:, 8:16] = l.reshape(n).astype(np.float64).view(np.uint8).reshape(n, 8)
    rec[:, 16:] = acc.reshape(n, d).astype(np.float32).view(np.uint8).reshape(n, 4 * d)
    return rec.reshape(-1)


def _unpack(buf, n, d):
    rec = np.asarray(buf, np.uint8).reshape(-1, n, 16 + 4 * d)
    m = rec[..., 0:8].copy().view(np.float64)[..., 0]
    l = rec[..., 8:16].copy().view(np.float64)[..., 0]
    acc = rec[..., 16:].copy().view(np.float32)
    return m, l, acc


def _leave(q, code):
    q.close()
    q.join_thread()  # flush queued reports before the hard exit
    os._exit(code)


def _rank_main(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch
    import torch.distributed as dist
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=20))
        store = dist.distributed_c10d._get_default_store()
        mon = par.PeerMonitor(store, rank, world, timeout=2.0, prefix=f"t-{mode}")
        if mode == "exchange":
            query, full, parts = _split_problem(777, heads=4, d=64, world=world, seed=3)
            m, l, acc = oracle.decode_paged_state(query, *parts[rank])
            mon.check()
            got = par.exchange_partials(torch.from_numpy(_pack(m, l, acc)), world)
            gm, gl, gacc = _unpack(got.numpy(), 4, 64)
            merged = oracle.merge_partials(gm, gl, gacc)
            ref = oracle.decode_paged(query, *full, method="f64")[0]
            q.put((rank, "ok", float(np.abs(merged - ref).max()), gm.shape))
        elif mode == "dead_peer":
            if rank == 1:
                q.put((rank, "exited", 0.0, None))
                _leave(q, 0)  # leaves between steps, before the collective step
            t0 = time.monotonic()
            try:
                mon.check()
                q.put((rank, "no error", 0.0, None))
            except par.PeerFailure as e:
                q.put((rank, "PeerFailure", time.monotonic() - t0, str(e)))
        elif mode == "raising_peer":
            if rank == 1:
                try:
                    raise RuntimeError("injected failure on rank 1")
                except RuntimeError:
                    q.put((rank, "raised", 0.0, None))
                    _leave(q, 1)
            try:
                mon.check()
                q.put((rank, "no error", 0.0, None))
            except par.PeerFailure as e:
                q.put((rank, "PeerFailure", 0.0, str(e)))
        q.put((rank, "done", 0.0, None))
    except Exception as e:  # report, never hang the parent
        q.put((rank, "error", 0.0, repr(e)))
    _leave(q, 0)  # skip process-group teardown (a dead peer would stall it)


def _run_ranks(mode, world=2, limit=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    msgs, deadline = [], time.monotonic() + limit
    for p in procs:
        p.join(max(0.1, deadline - time.monotonic()))
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    while True:
        try:
            msgs.append(q.get(timeout=1.0))
        except Exception:
            return msgs


def test_gloo_sequence_split_exchange():
    msgs = _run_ranks("exchange")
    oks = [m for m in msgs if m[1] == "ok"]
    assert len(oks) == 2, msgs
    for _, _, err, shape in oks:
        assert shape == (2, 4)
        assert err <= 2e-5


def test_gloo_dead_peer_detected_before_collective():
    msgs = _run_ranks("dead_peer")
    fails = [m for m in msgs if m[0] == 0 and m[1] == "PeerFailure"]
    assert fails, msgs
    _, _, waited, text = fails[0]
    assert "1" in text and waited < 10.0


def test_gloo_raising_peer_detected():
    msgs = _run_ranks("raising_peer")
    assert any(m[0] == 1 and m[1] == "raised" for m in msgs), msgs
    assert any(m[0] == 0 and m[1] == "PeerFailure" for m in msgs), msgs
