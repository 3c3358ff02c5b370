"""The fused decode step: RoPE -> quantize-on-append -> paged decode.

Checked against the oracle on the same seeded inputs:
* the rotated query and key are bit-exact with the RoPE oracle (which is
  pinned against transformers' apply_rotary_pos_emb, tests/test_rope_oracle.py);
* after prefill + appends, the pools equal the oracle's grouped quantizer on
  the whole rotated key sequence, bit for bit;
* the step's attention output is within 1e-6 of the float64 arbiter;
* ``LayerStack`` (all layers, device-side lengths) equals per-layer
  ``PagedKVCache.decode_step`` bit for bit, eagerly and replayed as a CUDA graph.
"""

import numpy as np
import pytest

import oracle
from helpers import pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
P = pkg("paged")
C = pkg("_C")
R = pkg("rope")
S = pkg("stepper")

TOL = 1e-6


def _tokens(n, heads, d, g):
    sc = torch.rand((heads, d), generator=g, device="cuda") * 2.5 + 0.5
    off = torch.randn((heads, d), generator=g, device="cuda") * 2.0
    return (torch.randn((n, heads, d), generator=g, device="cuda") * sc + off,
            torch.randn((n, heads, d), generator=g, device="cuda"))


def _logical(cache, s, group=128):
    n = cache.lens[s]
    pages = cache.pages[s]
    k = torch.cat([cache.k_pool[p] for p in pages], dim=1)[:, :n].transpose(0, 1)
    gp = group // 16
    sz = torch.stack([cache.sz_pool[pages[g * gp]] for g in range((n + group - 1) // group)])
    return k.cpu().numpy(), sz[:, :, 0].cpu().numpy(), sz[:, :, 1].cpu().numpy()


def test_rope_kernel_is_bit_exact():
    g = torch.Generator(device="cuda").manual_seed(3)
    for d in (64, 128, 256):
        cos, sin = R.rope_table(6000, d)
        x = torch.randn((37, 3, d), generator=g, device="cuda") * 4
        pos = torch.randint(0, 6000, (37,), generator=g, device="cuda", dtype=torch.int32)
        got = C.rope(x, pos, cos, sin).cpu().numpy()
        want = oracle.apply_rope(x.cpu().numpy(), pos.cpu().numpy(), cos.cpu().numpy(),
                                 sin.cpu().numpy())
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_rope_kernel_rejects_overlap_and_flags_bad_positions():
    cos, sin = R.rope_table(10, 64)
    x = torch.randn((4, 2, 64), device="cuda")
    with pytest.raises(RuntimeError):
        C.rope(x, torch.zeros(4, dtype=torch.int32, device="cuda"), cos, sin, out=x)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = C.rope(x, torch.tensor([0, 9, 10, -1], dtype=torch.int32, device="cuda"), cos, sin,
                 status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 2
    o = out.cpu().numpy()
    assert np.isfinite(o[:2]).all() and np.isnan(o[2:]).all()


@pytest.mark.parametrize("value_dtype", [torch.float32, torch.float16])
def test_decode_step_matches_oracle(value_dtype):
    heads, hq, d = 2, 4, 128
    prefill = [130, 16, 0, 255]
    steps = 20
    g = torch.Generator(device="cuda").manual_seed(7)
    full = [_tokens(n + steps, heads, d, g) for n in prefill]
    cos, sin = R.rope_table(1024, d)
    cache = P.PagedKVCache(128, heads, d, device="cuda", seed=5, value_dtype=value_dtype)
    ids = list(range(len(prefill)))
    cache.write_sequences(ids, [k[:n] for (k, _), n in zip(full, prefill)],
                          [v[:n] for (_, v), n in zip(full, prefill)], rope=(cos, sin))
    cos_h, sin_h = cos.cpu().numpy(), sin.cpu().numpy()
    for t in range(steps):
        q = torch.randn((len(ids), hq, d), generator=g, device="cuda")
        kt = torch.stack([k[n + t] for (k, _), n in zip(full, prefill)])
        vt = torch.stack([v[n + t] for (_, v), n in zip(full, prefill)])
        pos = np.array([n + t for n in prefill])
        out = cache.decode_step(ids, q, kt, vt, rope=(cos, sin))
        if t in (0, steps - 1):
            q_rot = oracle.apply_rope(q.cpu().numpy(), pos, cos_h, sin_h)
            bt, sl = cache.block_table(ids)
            exact = oracle.decode_paged(q_rot, cache.k_pool.cpu().numpy(),
                                        cache.v_pool.float().cpu().numpy(),
                                        cache.sz_pool.cpu().numpy(), bt.cpu().numpy(),
                                        sl.cpu().numpy(), method="f64")
            assert np.abs(out.cpu().numpy() - exact).max() <= TOL
    # the cache holds the oracle's quantization of the whole rotated key sequence
    for s, (k, _) in enumerate(full):
        n = prefill[s] + steps
        krot = oracle.apply_rope(k.cpu().numpy(), np.arange(n), cos_h, sin_h)
        codes, sc, zp = oracle.quantize_grouped(krot, 128)
        a = _logical(cache, s)
        np.testing.assert_array_equal(a[0], oracle.pack_int4(codes))
        np.testing.assert_array_equal(a[1].view(np.uint32), sc.view(np.uint32))
        np.testing.assert_array_equal(a[2].view(np.uint32), zp.view(np.uint32))


def _stack_and_reference(layers, seqs, heads, hq, d, prefill, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    data = [_tokens(n, heads, d, g) for n in prefill]
    stack = S.LayerStack(layers, seqs, heads, d, max_tokens=512, num_q_heads=hq, seed=seed)
    stack.prefill([k for k, _ in data], [v for _, v in data])
    refs = []
    for _ in range(layers):
        c = P.PagedKVCache(seqs * 33, heads, d, device="cuda", seed=seed + 1)
        c.write_sequences(list(range(seqs)), [k for k, _ in data], [v for _, v in data],
                          rope=stack.rope)
        refs.append(c)
    return stack, refs, g


def test_layer_stack_equals_per_layer_steps():
    layers, seqs, heads, hq, d = 3, 3, 2, 4, 128
    stack, refs, g = _stack_and_reference(layers, seqs, heads, hq, d, [129, 0, 300], seed=11)
    for _ in range(6):
        q = torch.randn((layers, seqs, hq, d), generator=g, device="cuda")
        k = torch.randn((layers, seqs, heads, d), generator=g, device="cuda")
        v = torch.randn((layers, seqs, heads, d), generator=g, device="cuda")
        out = stack.step(q, k, v).clone()
        for l in range(layers):
            want = refs[l].decode_step(list(range(seqs)), q[l], k[l], v[l], rope=stack.rope)
            assert torch.equal(out[l], want)
    assert stack.lens.tolist() == [135, 6, 306]


def test_layer_stack_graph_replay_equals_eager():
    layers, seqs, heads, hq, d = 2, 4, 2, 2, 64
    eager, _, g = _stack_and_reference(layers, seqs, heads, hq, d, [16, 17, 0, 127], seed=21)
    graphed, _, _ = _stack_and_reference(layers, seqs, heads, hq, d, [16, 17, 0, 127], seed=21)
    q = torch.zeros((seqs, hq, d), device="cuda")
    k = torch.zeros((seqs, heads, d), device="cuda")
    v = torch.zeros((seqs, heads, d), device="cuda")
    graphed.capture(q, k, v)
    for _ in range(5):
        qi = torch.randn((seqs, hq, d), generator=g, device="cuda")
        ki = torch.randn((seqs, heads, d), generator=g, device="cuda")
        vi = torch.randn((seqs, heads, d), generator=g, device="cuda")
        want = eager.step(qi, ki, vi).clone()
        q.copy_(qi), k.copy_(ki), v.copy_(vi)
        got = graphed.replay()
        assert torch.equal(got, want)
    assert graphed.lens.tolist() == eager.lens.tolist() == [21, 22, 5, 132]
    graphed.release()
