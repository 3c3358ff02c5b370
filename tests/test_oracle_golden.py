"""The CPU oracle is pinned to the reference's own outputs (golden vectors).

tests/golden/*.npz were produced by tests/golden/make_golden.py from the
reference's NumPy implementation. Quantizer and packing: bit-exact. Attention:
the reference's float32 online softmax through NumPy/BLAS; the restatement
uses the same primitives in the same order, so it matches to the last bit on
one machine and to 1e-6 wherever BLAS orders sums differently.
"""

import numpy as np
import pytest

import oracle
from helpers import attn_case_lists, golden

QUANT = golden("golden_quant")
PACK = golden("golden_pack")
ATTN = golden("golden_attn")

ATTN_TOL = 1e-6


@pytest.mark.parametrize("name", sorted(k for k in QUANT if not k.startswith("grouped")))
def test_quantizer_bit_exact(name):
    c = QUANT[name]
    q, s, z = oracle.quantize_int4(c["kv"])
    np.testing.assert_array_equal(q, c["q"])
    np.testing.assert_array_equal(s.view(np.uint32), c["scale"].view(np.uint32))
    np.testing.assert_array_equal(z.view(np.uint32), c["zp"].view(np.uint32))


@pytest.mark.parametrize("name", sorted(k for k in QUANT if k.startswith("grouped")))
def test_grouped_quantizer_bit_exact(name):
    c = QUANT[name]
    q, s, z = oracle.quantize_grouped(c["kv"], 128)
    np.testing.assert_array_equal(q, c["q"])
    np.testing.assert_array_equal(s.view(np.uint32), c["scale"].view(np.uint32))
    np.testing.assert_array_equal(z.view(np.uint32), c["zp"].view(np.uint32))


def test_known_answer_scales():
    """tests/test_quantization.py:46-66 of the reference: scale = (11-1)/15."""
    q, s, z = oracle.quantize_int4(QUANT["kat_scales"]["kv"])
    np.testing.assert_allclose(s, [10 / 15, 10 / 15], rtol=1e-6)


def test_round_half_even_ties():
    """Bins at exact .5 ties follow round-half-even (np.round), not half-up."""
    q, s, _ = oracle.quantize_int4(QUANT["half_even_ties"]["kv"])
    assert s[0] == np.float32(1.0)
    assert q[:, 0].tolist() == [0, 15, 0, 2, 2, 4, 4, 14, 14]


@pytest.mark.parametrize("name", sorted(PACK))
def test_pack_exact(name):
    c = PACK[name]
    p = oracle.pack_int4(c["q"])
    np.testing.assert_array_equal(p, c["packed"])
    np.testing.assert_array_equal(oracle.unpack_int4(p, c["q"].shape[-1]), c["unpacked"])


def test_pack_rejects_out_of_range():
    with pytest.raises(AssertionError):
        oracle.pack_int4(np.array([[16]], np.uint8))


@pytest.mark.parametrize("name", sorted(k for k in ATTN if not k.startswith("paged")))
def test_online_softmax_matches_reference(name):
    query, kq, s, z, v, lens = attn_case_lists(ATTN[name])
    out, _ = oracle.online_softmax(query, list(zip(kq, s, z)), v, lens)
    assert np.abs(out - ATTN[name]["out"]).max() <= ATTN_TOL


@pytest.mark.parametrize("name", sorted(k for k in ATTN if k.startswith("paged")))
def test_paged_driver_matches_reference(name):
    c = ATTN[name]
    out = oracle.decode_paged(c["query"], c["k_pool"], c["v_pool"], c["sz_pool"],
                              c["block_table"], c["seq_lens"])
    assert np.abs(out - c["out"]).max() <= ATTN_TOL


def test_all_empty_is_exact_zeros():
    query, kq, s, z, v, lens = attn_case_lists(ATTN["all_empty"])
    out, _ = oracle.online_softmax(query, list(zip(kq, s, z)), v, lens)
    np.testing.assert_array_equal(out, np.zeros_like(out))


def test_arbiters_agree_with_oracle_on_small_cases():
    """The float64 arbiter and the exact-f32-keys evaluation sit within the
    float32 noise floor of the oracle on the reference's test distribution."""
    query, kq, s, z, v, lens = attn_case_lists(ATTN["ragged_64_0_17"])
    pages = list(zip(kq, s, z))
    ref, _ = oracle.online_softmax(query, pages, v, lens)
    f64 = oracle.attention_f64(query, pages, v, lens)
    ex = oracle.attention_exact_f32_keys(query, pages, v, lens)
    assert np.abs(ref - f64).max() < 1e-5
    assert np.abs(ref - ex).max() < 1e-5


@pytest.mark.parametrize("n_tok,gq", [(1, 1), (16, 2), (130, 1), (2048, 4), (3001, 1)])
def test_stream_f64_equals_per_page_arbiter(n_tok, gq):
    """The vectorised one-stream float64 arbiter evaluates the same mathematics
    as the per-page ``attention_f64`` (partial pages and groups included)."""
    from helpers import oracle_build_pools, pkg
    W = pkg("workloads")
    prob = W.np_paged_problem(1, 1, 128, [n_tok], pool_pages=(n_tok + 15) // 16 + 3, seed=n_tok)
    prob["query"] = np.repeat(prob["query"], gq, axis=1) * np.linspace(0.5, 1.5, gq)[None, :, None]
    prob["query"] = prob["query"].astype(np.float32)
    k_pool, v_pool, sz_pool = oracle_build_pools(prob)
    bt, sl = prob["block_table"], prob["seq_lens"]
    per_page = oracle.decode_paged(prob["query"], k_pool, v_pool, sz_pool, bt, sl, method="f64")
    pages = bt[0, :(n_tok + 15) // 16]
    vec = oracle.stream_f64(prob["query"][0], k_pool[pages, 0], v_pool[pages, 0],
                            sz_pool[pages, 0], n_tok)
    np.testing.assert_allclose(vec, per_page[0], rtol=0, atol=1e-12)
