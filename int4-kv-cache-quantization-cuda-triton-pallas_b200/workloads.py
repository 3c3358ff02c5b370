"""Seeded synthetic inputs with the benchmark configurations' shapes and distributions.

The reference measures on synthetic data too (benchmarks/bench_three_backend.py:113-129);
these generators produce the anchor distribution of the benchmark configs:

* query ~ N(0, 1)
* keys ~ N(0, 1) * scale_c + offset_c per (sequence, head, channel), with
  offset_c ~ N(0, 2) and scale_c ~ U(0.5, 3) (post-RoPE outlier channels)
* values ~ N(0, 1), float32, unquantized
* 16-token pages placed by a seeded random permutation of the page pool.

NumPy generators (``np_*``) serve small CPU-checked cases; torch generators
(``torch_*``) build the full-size problems directly in HBM.
"""

from dataclasses import dataclass
from typing import List, Optional

import numpy as np

PAGE_TOKENS = 16


def np_anchor_keys(rng, n, h, d):
    sc = rng.uniform(0.5, 3.0, (h, d)).astype(np.float32)
    off = (rng.standard_normal((h, d)) * 2.0).astype(np.float32)
    return (rng.standard_normal((n, h, d)).astype(np.float32) * sc + off).astype(np.float32)


def np_block_table(rng, lens, pool_pages, page=PAGE_TOKENS):
    """Seeded scatter of each sequence's pages over a pool; returns int32 [B, max_pages]."""
    need = [(n + page - 1) // page for n in lens]
    if sum(need) > pool_pages:
        raise ValueError(f"pool of {pool_pages} pages is too small for {sum(need)} pages")
    perm = rng.permutation(pool_pages)[: sum(need)]
    bt = np.zeros((len(lens), max(1, max(need))), np.int32)
    pos = 0
    for b, k in enumerate(need):
        bt[b, :k] = perm[pos:pos + k]
        pos += k
    return bt


@dataclass
class DecodeShape:
    batch: int
    heads: int
    head_dim: int
    seq_lens: List[int]
    pool_pages: int
    group_tokens: int = 128
    value_bytes: int = 4  # 4 float32, 2 float16 / bfloat16 value pool
    q_heads: Optional[int] = None  # query heads (GQA: a multiple of `heads`); None = heads

    @property
    def query_heads(self):
        return self.q_heads if self.q_heads is not None else self.heads

    @property
    def pages(self):
        return sum((n + PAGE_TOKENS - 1) // PAGE_TOKENS for n in self.seq_lens)

    def algorithmic_bytes(self):
        """Bytes a decode step must move: valid-token K (packed) + V + per-group scale/zp
        + query + output + block-table entries. K/V/scale bytes count per kv head
        (``heads``), query/output per query head."""
        d = self.head_dim
        total = 0
        for n in self.seq_lens:
            groups = (n + self.group_tokens - 1) // self.group_tokens
            pages = (n + PAGE_TOKENS - 1) // PAGE_TOKENS
            total += self.heads * (n * d // 2 + self.value_bytes * n * d + 8 * d * groups) + 4 * pages
        total += 2 * 4 * self.batch * self.query_heads * d
        return total


def config_shape(name: str, seed: int = 0) -> DecodeShape:
    """The decode configurations of the benchmark definition (per GPU)."""
    if name == "cfg0":
        return DecodeShape(8, 32, 128, [2048] * 8, pool_pages=8 * 128)
    if name.startswith("cfg0_gqa"):  # config 0's 32 query heads over 32 / G kv heads
        G = int(name[len("cfg0_gqa"):])
        if G <= 0 or 32 % G:
            raise ValueError(f"unknown config {name}")
        return DecodeShape(8, 32 // G, 128, [2048] * 8, pool_pages=8 * 128, q_heads=32)
    if name.startswith("cfg2_"):  # cfg2_<L>, or cfg2_<L>_gqa<G>: 32 query heads over 32 / G
        parts = name.split("_")
        L = int(parts[1])
        G = int(parts[2][len("gqa"):]) if len(parts) > 2 and parts[2].startswith("gqa") else 1
        if G <= 0 or 32 % G:
            raise ValueError(f"unknown config {name}")
        return DecodeShape(8, 32 // G, 128, [L] * 8, pool_pages=8 * ((L + 15) // 16),
                           q_heads=32 if G > 1 else None)
    if name.startswith("cfg3_d"):
        d = int(name[len("cfg3_d"):])
        rng = np.random.default_rng(seed)
        lens = rng.integers(0, 16385, 64).tolist()
        lens[0] = 0  # always include an empty sequence
        lens[1] = 16384 if d == 128 else lens[1]
        return DecodeShape(64, 32, d, lens, pool_pages=(1 << 20) // PAGE_TOKENS)
    if name == "cfg4_layer":
        return DecodeShape(32, 32, 128, [4096] * 32, pool_pages=32 * 256)
    if name == "cfg4_long":
        return DecodeShape(1, 32, 128, [131072], pool_pages=131072 // 16)
    raise ValueError(f"unknown config {name}")


def torch_build_cache(shape: DecodeShape, seed: int = 0, device="cuda", value_dtype=None):
    """Build a full-size paged problem in HBM with the GPU quantizer.

    Returns dict(query, cache) where cache is a ``paged.PagedKVCache`` holding
    every sequence (ids 0..B-1). Keys/values are generated one sequence at a
    time so the fp32 staging never exceeds one sequence.
    """
    import torch
    from .paged import PagedKVCache

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    cache = PagedKVCache(shape.pool_pages, shape.heads, shape.head_dim, shape.group_tokens,
                         device=device, seed=seed,
                         value_dtype=value_dtype if value_dtype is not None else torch.float32)
    h, d = shape.heads, shape.head_dim
    for b, n in enumerate(shape.seq_lens):
        if n == 0:
            cache.write_sequences([b], [torch.zeros((0, h, d), device=device)])
            continue
        sc = torch.rand((h, d), generator=g, device=device) * 2.5 + 0.5
        off = torch.randn((h, d), generator=g, device=device) * 2.0
        k = torch.randn((n, h, d), generator=g, device=device) * sc + off
        v = torch.randn((n, h, d), generator=g, device=device)
        cache.write_sequences([b], [k], [v])
        del k, v
    query = torch.randn((shape.batch, shape.query_heads, d), generator=g, device=device)
    return {"query": query, "cache": cache}


def np_paged_problem(batch, heads, head_dim, seq_lens, pool_pages, seed=0, group=128):
    """Small paged problem on the host: raw keys/values per sequence, query, block table."""
    rng = np.random.default_rng(seed)
    query = rng.standard_normal((batch, heads, head_dim)).astype(np.float32)
    bt = np_block_table(rng, seq_lens, pool_pages)
    keys, vals = [], []
    for n in seq_lens:
        keys.append(np_anchor_keys(rng, n, heads, head_dim))
        vals.append(rng.standard_normal((n, heads, head_dim)).astype(np.float32))
    return {"query": query, "block_table": bt, "seq_lens": np.asarray(seq_lens, np.int32),
            "keys": keys, "values": vals, "pool_pages": pool_pages, "group": group}
