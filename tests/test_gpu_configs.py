"""Full-size parity of the paged decode on every decode configuration of the
benchmark definition, with the cache written by the GPU quantizer.

* config 0 (8 x 32 x d128 x 2048): ALL 256 streams against the reference's
  fp32 path (``online_softmax_ref``, src/flash_decode_ref.py:30-139, restated
  as ``oracle.online_softmax``) and the float64 arbiter
  (tests/test_pallas_flash_decode.py:53-78 of the reference, restated as
  ``oracle.attention_f64``; evaluated here by its vectorised one-stream form
  ``oracle.stream_f64``, pinned to it in tests/test_oracle_golden.py);
* config 2 at 512 / 8192 / 32768 tokens, config 3 (64 ragged sequences in a
  2^20-token pool, d64 and d128, an empty sequence and partial last pages),
  config 4's per-GPU layer (32 x 4096) and its long sequence (1 x 131072) on
  one GPU: a seeded sample of at least 32 streams each, empty sequences
  always included.

Gates per stream:

* ``max |gpu - f64 arbiter| <= 1e-6`` (the kernel's own accuracy);
* ``max |gpu - fp32 oracle| <= 1e-5`` (the benchmark's gate), except where
  the fp32 oracle is itself farther than that from the float64 value: at this
  distribution (unscaled logits of magnitude ~100) a few streams per batch
  have ``|oracle - f64|`` of 1.1e-5 to 2e-5, and no accurate kernel can be
  within 1e-5 of the oracle there. Those streams must satisfy
  ``|gpu - oracle| <= |oracle - f64| + 1e-6`` instead, and the test lists them.

Streams are copied off the device one (sequence, kv head) at a time, so the
host never holds a whole pool (config 3 at d128 is 21 GB of pools).
"""

import numpy as np
import pytest

import oracle
from helpers import pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
W = pkg("workloads")

REF_TOL = 1e-5
EXACT_TOL = 1e-6


def stream_on_host(cache, bt_row, n_tok, h):
    """Pools of one (sequence, kv head) stream as a one-sequence, one-head paged
    problem on the host: (k_pool, v_pool, sz_pool, block_table, seq_lens)."""
    npg = (n_tok + 15) // 16
    pages = torch.as_tensor(np.asarray(bt_row[:npg], np.int64), device=cache.k_pool.device)
    kp = cache.k_pool[pages, h][:, None].cpu().numpy()
    vp = cache.v_pool[pages, h][:, None].float().cpu().numpy()
    sp = cache.sz_pool[pages, h][:, None].cpu().numpy()
    bt = np.arange(npg, dtype=np.int32)[None]
    return kp, vp, sp, bt, np.array([n_tok], np.int32)


def check_streams(out, query, cache, bt, sl, streams, group_q=1):
    """Gate each (sequence, kv head) stream of ``out`` (device) against the fp32
    oracle and the float64 arbiter; returns the measured maxima and the streams
    where the fp32 oracle is itself more than REF_TOL from float64."""
    o = out.cpu().numpy()
    q = query.cpu().numpy()
    bt_h, sl_h = bt.cpu().numpy(), sl.cpu().numpy()
    G = group_q
    worst_f64 = worst_ref = 0.0
    oracle_off = []
    for b, h in streams:
        got = o[b:b + 1, h * G:(h + 1) * G]
        n = int(sl_h[b])
        if n == 0:
            assert np.all(got == 0), f"empty sequence {b} must give exact zeros"
            continue
        kp, vp, sp, bt1, sl1 = stream_on_host(cache, bt_h[b], n, h)
        q1 = q[b:b + 1, h * G:(h + 1) * G]
        ref = oracle.decode_paged(q1, kp, vp, sp, bt1, sl1)
        f64 = oracle.stream_f64(q1[0], kp[:, 0], vp[:, 0], sp[:, 0], n)[None]
        e_f64 = float(np.abs(got - f64).max())
        e_ref = float(np.abs(got - ref).max())
        o_f64 = float(np.abs(ref - f64).max())
        assert np.isfinite(got).all()
        assert e_f64 <= EXACT_TOL, (b, h, e_f64)
        if o_f64 > REF_TOL:
            oracle_off.append((b, h, o_f64, e_ref))
            assert e_ref <= o_f64 + EXACT_TOL, (b, h, e_ref, o_f64)
        else:
            assert e_ref <= REF_TOL, (b, h, e_ref, o_f64)
        worst_f64 = max(worst_f64, e_f64)
        worst_ref = max(worst_ref, e_ref)
    return {"max_abs_vs_f64": worst_f64, "max_abs_vs_oracle": worst_ref, "oracle_off": oracle_off}


def _sample(shape, k, seed):
    rng = np.random.default_rng(seed)
    pairs = {(int(b), int(h)) for b, h in zip(rng.integers(0, shape.batch, 4 * k),
                                              rng.integers(0, shape.heads, 4 * k))}
    pairs = sorted(pairs)[:k] if len(pairs) > k else sorted(pairs)
    # every empty sequence, and the longest one, are always checked
    for b, n in enumerate(shape.seq_lens):
        if n == 0 or n == max(shape.seq_lens):
            pairs.append((b, int(rng.integers(0, shape.heads))))
    return sorted(set(pairs))


def _run(name, seed):
    shape = W.config_shape(name)
    prob = W.torch_build_cache(shape, seed=seed)
    cache, query = prob["cache"], prob["query"]
    ids = list(range(shape.batch))
    bt, sl = cache.block_table(ids)
    out = cache.decode(query, ids)
    torch.cuda.synchronize()
    return shape, cache, query, bt, sl, out


def _release():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def test_config0_all_streams():
    shape, cache, query, bt, sl, out = _run("cfg0", seed=0)
    assert torch.isfinite(out).all()
    streams = [(b, h) for b in range(shape.batch) for h in range(shape.heads)]
    r = check_streams(out, query, cache, bt, sl, streams)
    # the exceptions are the oracle's own error, a small minority of the streams
    assert len(r["oracle_off"]) <= len(streams) // 16, r["oracle_off"]
    del cache, out
    _release()


@pytest.mark.parametrize("name", ["cfg2_512", "cfg2_8192", "cfg2_32768", "cfg3_d64", "cfg3_d128",
                                  "cfg4_layer", "cfg4_long"])
def test_benchmark_config_full_size(name):
    shape, cache, query, bt, sl, out = _run(name, seed=11)
    assert torch.isfinite(out).all()
    zero = [b for b, n in enumerate(shape.seq_lens) if n == 0]
    if zero:
        assert bool((out[zero] == 0).all())
    k = 32 if shape.batch * shape.heads >= 32 else shape.batch * shape.heads
    streams = _sample(shape, k, seed=len(name))
    if name == "cfg4_long":  # one sequence: 32 streams are all of its heads
        streams = [(0, h) for h in range(shape.heads)]
    assert len(streams) >= 32
    check_streams(out, query, cache, bt, sl, streams)
    del cache, out
    _release()


@pytest.mark.parametrize("name", ["cfg0_gqa2", "cfg0_gqa4", "cfg0_gqa8", "cfg0_gqa32"])
def test_grouped_query_full_size(name):
    """Config 0's shape with 32 query heads over 16 / 8 / 4 / 1 kv heads: every
    (sequence, kv head) stream, all of its query heads, against the fp32 oracle
    and the float64 arbiter. Covers the warps serving two (G = 2) and four
    (G = 4, 8, 32) query heads each, paired on one run, with the multi-head
    record merge."""
    shape, cache, query, bt, sl, out = _run(name, seed=21)
    assert torch.isfinite(out).all()
    G = shape.query_heads // shape.heads
    streams = [(b, h) for b in range(shape.batch) for h in range(shape.heads)]
    r = check_streams(out, query, cache, bt, sl, streams, group_q=G)
    assert len(r["oracle_off"]) <= max(2, len(streams) * G // 16), r["oracle_off"]
    del cache, out
    _release()


@pytest.mark.parametrize("vdtype", ["float16", "bfloat16"])
def test_config0_values16_full_size(vdtype):
    """Config 0 with the value pool stored as float16 / bfloat16 (rounded to
    nearest even by the cache writer; the oracle reads the stored values
    widened to float32): a seeded sample of 64 streams."""
    shape = W.config_shape("cfg0")
    shape.value_bytes = 2
    prob = W.torch_build_cache(shape, seed=31, value_dtype=getattr(torch, vdtype))
    cache, query = prob["cache"], prob["query"]
    ids = list(range(shape.batch))
    bt, sl = cache.block_table(ids)
    out = cache.decode(query, ids)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    check_streams(out, query, cache, bt, sl, _sample(shape, 64, seed=5))
    del cache, out
    _release()
