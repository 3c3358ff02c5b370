"""The RoPE oracle against the reference model path's own rotation.

The reference quantizes post-RoPE keys of a Hugging Face Llama
(scripts/validate_llama.py:23-31), whose rotation is transformers'
``apply_rotary_pos_emb`` (rotate-half form). Pinned bit for bit on seeded
inputs, for several head dims and positions; no GPU.
"""

import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")


def _hf():
    try:
        from transformers.models.llama import modeling_llama as m
    except Exception as e:  # pragma: no cover - transformers is in this image
        pytest.skip(f"transformers unavailable: {e}")
    return m


@pytest.mark.parametrize("d,rows,heads", [(64, 7, 3), (128, 5, 4), (256, 3, 2)])
def test_oracle_rope_matches_transformers(d, rows, heads):
    m = _hf()
    rng = np.random.default_rng(d)
    cos, sin = oracle.rope_table_f32(5000, d)
    x = (rng.standard_normal((rows, heads, d)) * 3).astype(np.float32)
    pos = rng.integers(0, 5000, rows)
    pos[0] = 0
    pos[-1] = 4999
    ours = oracle.apply_rope(x, pos, cos, sin)
    # transformers: q [batch, heads, seq, D], cos/sin [batch, seq, D] (duplicated halves)
    q = torch.from_numpy(x).permute(1, 0, 2).unsqueeze(0)          # [1, heads, rows, D]
    cf = torch.from_numpy(np.concatenate([cos, cos], 1)[pos])[None]  # [1, rows, D]
    sf = torch.from_numpy(np.concatenate([sin, sin], 1)[pos])[None]
    q_e, k_e = m.apply_rotary_pos_emb(q, q.clone(), cf, sf)
    hf = q_e[0].permute(1, 0, 2).numpy()
    assert hf.dtype == np.float32
    assert np.array_equal(ours.view(np.uint32), hf.view(np.uint32))
    assert np.array_equal(k_e[0].permute(1, 0, 2).numpy().view(np.uint32), ours.view(np.uint32))


def test_position_zero_is_identity():
    cos, sin = oracle.rope_table_f32(4, 128)
    x = np.random.default_rng(1).standard_normal((2, 2, 128)).astype(np.float32)
    assert np.array_equal(oracle.apply_rope(x, [0, 0], cos, sin), x)


def test_product_table_equals_the_oracle_table():
    """The package's table builder (host side, a parameter like a weight) and
    the checker's give the same float32 values."""
    from helpers import pkg
    rope = pkg("rope")
    c, s = rope.rope_table(300, 128, device="cpu")
    oc, os_ = oracle.rope_table_f32(300, 128)
    assert np.array_equal(c.numpy(), oc) and np.array_equal(s.numpy(), os_)
