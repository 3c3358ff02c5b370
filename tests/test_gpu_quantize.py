"""GPU parity of the INT4 quantizers against the oracle (bit-exact).

Bar: codes, scales and zero-points identical to the reference's NumPy oracle
(bit for bit -- `view(uint32)` equality), on the golden vectors, on the
reference's own test shapes, and on benchmark config 1 sizes. At the largest
sizes the whole output is checked through size-independent properties
(per-group scale recomputed with exact device min/max, round-trip error
bound) plus exact comparison of a seeded sample of groups.
"""

import numpy as np
import pytest

import oracle
from helpers import golden, oracle_build_pools, pkg

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
C = pkg("_C")
ops = pkg("ops")
W = pkg("workloads")

QUANT = golden("golden_quant")


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def assert_same(got, ref):
    q, s, z = got
    qr, sr, zr = ref
    np.testing.assert_array_equal(q, qr)
    np.testing.assert_array_equal(bits(s), bits(sr))
    np.testing.assert_array_equal(bits(z), bits(zr))


# ---------------- the reference's quantizer contract (one group = all rows) ----------------

@pytest.mark.parametrize("name", sorted(k for k in QUANT if not k.startswith("grouped")))
def test_legacy_quantizer_golden(name):
    c = QUANT[name]
    kv = c["kv"].reshape(-1, c["kv"].shape[-1])
    assert_same(ops.quantize_int4(kv), (c["q"].reshape(kv.shape), c["scale"], c["zp"]))


@pytest.mark.parametrize("shape", [(1, 1), (1, 64), (255, 3), (256, 3), (257, 3), (1030, 8),
                                   (4096, 128), (32768, 128), (5000, 37), (7, 4097), (3, 300),
                                   (2049, 129), (100003, 3), (9, 512), (65536, 256)])
def test_legacy_quantizer_shapes(shape):
    kv = np.random.RandomState(shape[0]).randn(*shape).astype(np.float32)
    assert_same(ops.quantize_int4(kv, backend="cuda"), oracle.quantize_int4(kv))


def test_legacy_quantizer_twice_in_a_row_and_misaligned_rows():
    """The scale / zp outputs double as the running min / max keys during a
    call: a second call on the same outputs, and a call on an input whose rows
    start 4 bytes off a 16-byte boundary (the scalar-load path), both still
    match the oracle bit for bit."""
    kv = np.random.RandomState(3).randn(3001, 128).astype(np.float32) * 3 + 1
    t = torch.from_numpy(kv).cuda()
    first = C.quantize_int4(t)
    second = C.quantize_int4(t)
    ref = oracle.quantize_int4(kv)
    for got in (first, second):
        assert_same([x.cpu().numpy() for x in got], ref)
    buf = torch.empty((kv.size + 1,), dtype=torch.float32, device="cuda")
    view = buf[1:].view(kv.shape)  # 4-byte offset: not 16-byte aligned
    view.copy_(t)
    assert_same([x.cpu().numpy() for x in C.quantize_int4(view)], ref)


def test_legacy_quantizer_anchor_distribution():
    kv = W.np_anchor_keys(np.random.default_rng(5), 2048, 4, 128).reshape(2048, 512)
    assert_same(ops.quantize_int4(kv), oracle.quantize_int4(kv))


def test_binding_rejects_bad_quantizer_input():
    with pytest.raises(RuntimeError, match="float32"):
        C.quantize_int4(torch.zeros(4, 4, dtype=torch.float64, device="cuda"))
    with pytest.raises(RuntimeError, match="non-empty"):
        C.quantize_int4(torch.zeros(0, 4, device="cuda"))
    with pytest.raises(RuntimeError, match="2D"):
        C.quantize_int4(torch.zeros(4, device="cuda"))
    with pytest.raises(RuntimeError, match="CUDA"):
        C.quantize_int4(torch.zeros(4, 4))


# ---------------- grouped, packed (benchmark config 1) ----------------

@pytest.mark.parametrize("name", sorted(k for k in QUANT if k.startswith("grouped")))
def test_grouped_golden(name):
    c = QUANT[name]
    packed, s, z = ops.quantize_int4_grouped(c["kv"], 128)
    assert_same((packed, s, z), (oracle.pack_int4(c["q"]), c["scale"], c["zp"]))


@pytest.mark.parametrize("n,h,d,group", [(1, 1, 4, 128), (129, 2, 64, 128), (300, 3, 128, 128),
                                         (4096, 32, 128, 128), (1000, 8, 64, 16),
                                         (777, 4, 128, 200), (256, 2, 256, 64),
                                         (500, 3, 64, 128), (4000, 1, 64, 32)])
def test_grouped_matches_oracle(n, h, d, group):
    """Every kernel form: 128-channel TMA slabs (C % 128 == 0), 64-channel
    slabs (C = 192, 64), the register kernel (C = 4) and the two-pass kernel
    (groups > 128); full and short last groups."""
    kv = W.np_anchor_keys(np.random.default_rng(n + d), n, h, d)
    q, s, z = oracle.quantize_grouped(kv, group)
    assert_same(ops.quantize_int4_grouped(kv, group), (oracle.pack_int4(q), s, z))


def test_grouped_half_even_ties():
    """Exact .5 ties round to even on the device, as np.round does."""
    col = np.array([0.0, 15.0, 0.5, 1.5, 2.5, 3.5, 4.5, 13.5, 14.5] + [7.0] * 7, np.float32)
    kv = np.tile(col[:, None, None], (1, 1, 4))
    packed, s, _ = ops.quantize_int4_grouped(kv, 128)
    codes = oracle.unpack_int4(packed, 4)[:, 0, 0]
    assert codes[:9].tolist() == [0, 15, 0, 2, 2, 4, 4, 14, 14]


def torch_quantize_grouped(kv, group):
    """The oracle's grouped quantizer (oracle.quantize_grouped, restating
    src/quantize_int4_ref.py:51-75 per 128-token group and head) written with
    torch operations on the device, for full groups: exact min/max, IEEE
    float32 subtraction and tensor / tensor division (no reciprocal), round half
    to even (torch.round), clamp, then the nibble packing of src/int4_pack.py
    (even channel -> low nibble). Returns (packed, scale, zp)."""
    n, h, d = kv.shape
    blk = kv.view(n // group, group, h, d)
    lo, hi = blk.amin(dim=1, keepdim=True), blk.amax(dim=1, keepdim=True)
    scale = torch.clamp(hi - lo, min=1e-8) / torch.full_like(lo, 15.0)
    zp = -lo / scale
    codes = torch.clamp(torch.round((blk - lo) / scale), 0, 15).to(torch.uint8).view(n, h, d)
    packed = codes[..., 0::2] | (codes[..., 1::2] << 4)
    return packed, scale.view(n // group, h, d), zp.view(n // group, h, d)


@pytest.mark.parametrize("n_tokens", [2048, 8192, 32768, 131072])
def test_grouped_baseline_sizes(n_tokens):
    """benchmark config 1: [N, 32, 128], 128-token groups. Every code, scale and
    zero-point of the whole output is compared bit for bit with the torch
    restatement of the oracle, which is itself checked bit for bit against the
    oracle on a seeded sample of (group, head) slices."""
    h, d, group = 32, 128, 128
    g = torch.Generator(device="cuda").manual_seed(n_tokens)
    sc = torch.rand((h, d), generator=g, device="cuda") * 2.5 + 0.5
    off = torch.randn((h, d), generator=g, device="cuda") * 2.0
    kv = torch.randn((n_tokens, h, d), generator=g, device="cuda") * sc + off
    packed, scale, zp = C.quantize_int4_grouped(kv, group)
    torch.cuda.synchronize()
    G = n_tokens // group
    blk = kv.view(G, group, h, d)
    lo, hi = blk.amin(dim=1), blk.amax(dim=1)
    # tensor / tensor is IEEE division (tensor / python-scalar multiplies by a reciprocal)
    exp_scale = torch.clamp(hi - lo, min=1e-8) / torch.full_like(lo, 15.0)
    assert torch.equal(scale.view(torch.int32), exp_scale.view(torch.int32))
    assert torch.equal(zp.view(torch.int32), (-lo / exp_scale).view(torch.int32))
    # round trip: |k - dequant(k)| <= scale/2 (+1 ulp slack of the float32 dequant)
    codes = torch.stack([packed & 15, packed >> 4], dim=-1).view(n_tokens, h, d).float()
    deq = (codes.view(G, group, h, d) * scale[:, None] - zp[:, None] * scale[:, None])
    err = (deq - blk).abs()
    assert bool((err <= scale[:, None] * 0.5001 + 1e-6).all())
    # every byte of the output against the torch restatement of the oracle
    t_packed, t_scale, t_zp = torch_quantize_grouped(kv, group)
    assert torch.equal(packed, t_packed), int((packed != t_packed).sum())
    assert torch.equal(scale.view(torch.int32), t_scale.view(torch.int32))
    assert torch.equal(zp.view(torch.int32), t_zp.view(torch.int32))
    # the restatement (and so the GPU output) against the oracle itself on a
    # seeded sample of (group, head) slices
    rng = np.random.default_rng(n_tokens)
    kv_h = kv.cpu().numpy()
    pk_h, sc_h, zp_h = t_packed.cpu().numpy(), t_scale.cpu().numpy(), t_zp.cpu().numpy()
    for gi, hi_ in zip(rng.integers(0, G, 16), rng.integers(0, h, 16)):
        q_r, s_r, z_r = oracle.quantize_int4(kv_h[gi * group:(gi + 1) * group, hi_, :])
        np.testing.assert_array_equal(pk_h[gi * group:(gi + 1) * group, hi_], oracle.pack_int4(q_r))
        np.testing.assert_array_equal(bits(sc_h[gi, hi_]), bits(s_r))
        np.testing.assert_array_equal(bits(zp_h[gi, hi_]), bits(z_r))


# ---------------- paged cache write (quantize + scatter) ----------------

@pytest.mark.parametrize("d,lens", [(128, [300, 517, 0, 16, 1]), (64, [256, 141]), (256, [130, 7])])
def test_cache_write_matches_oracle_pools(d, lens):
    P = W
    prob = P.np_paged_problem(len(lens), 4, d, lens, pool_pages=sum((n + 15) // 16 for n in lens) + 7,
                              seed=d)
    k_ref, v_ref, sz_ref = oracle_build_pools(prob)
    dev = torch.device("cuda")
    kp = torch.zeros(k_ref.shape, dtype=torch.uint8, device=dev)
    vp = torch.zeros(v_ref.shape, dtype=torch.float32, device=dev)
    sp = torch.zeros(sz_ref.shape, dtype=torch.float32, device=dev)
    k = torch.from_numpy(np.concatenate(prob["keys"])).to(dev)
    v = torch.from_numpy(np.concatenate(prob["values"])).to(dev)
    offs = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
    bt = torch.from_numpy(prob["block_table"]).to(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    C.cache_write(k, v, offs, bt, kp, vp, sp, max_rows_per_seq=max(lens), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    np.testing.assert_array_equal(kp.cpu().numpy(), k_ref)
    np.testing.assert_array_equal(vp.cpu().numpy(), v_ref)
    np.testing.assert_array_equal(bits(sp.cpu().numpy()), bits(sz_ref))


def test_cache_write_flags_bad_block_table():
    dev = torch.device("cuda")
    kp = torch.zeros((4, 2, 16, 32), dtype=torch.uint8, device=dev)
    vp = torch.zeros((4, 2, 16, 64), dtype=torch.float32, device=dev)
    sp = torch.zeros((4, 2, 2, 64), dtype=torch.float32, device=dev)
    k = torch.randn((32, 2, 64), device=dev)
    offs = torch.tensor([0, 32], dtype=torch.int32, device=dev)
    bt = torch.tensor([[1, 99]], dtype=torch.int32, device=dev)  # page 99 does not exist
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    C.cache_write(k, k, offs, bt, kp, vp, sp, max_rows_per_seq=32, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 1  # INT4KV_STATUS_BAD_PAGE
    assert bool((kp[1] != 0).any())  # the valid page was still written
