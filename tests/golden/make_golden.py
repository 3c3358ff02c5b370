"""Generate the golden vectors that pin the CPU oracle to the reference.

Run once, in a container where the reference repository is importable:

    python tests/golden/make_golden.py --reference <path to the reference checkout>

It imports the reference's own NumPy implementation (``src.quantize_int4_ref``,
``src.flash_decode_ref``, ``src.int4_pack``) and records its outputs on seeded
inputs into ``tests/golden/*.npz``. The tests never run this script and never
read the reference; they only load the ``.npz`` files.

Cases follow the reference's own tests: the known-answer scale test
(tests/test_quantization.py:46-66), uniform / tiny-range / large-negative /
mixed-magnitude inputs (:89-103, :174-201), the dispatch parity shapes
(tests/test_ops_dispatch.py:60-69, :330-338), packing extremes
(tests/test_int4_pack.py:33-35), ragged / empty-page attention
(tests/test_ops_dispatch.py:245-251, tests/test_pallas_flash_decode.py:119-148),
head_dim and page-row boundaries (tests/test_ops_dispatch.py:263-291), plus
the benchmark anchor distribution on the paged layout (16-token pages,
128-token groups, seeded block table).
"""

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def anchor_keys(rng, n, h, d):
    """Outlier-channel keys: N(0,1) * U(0.5,3) + N(0,2) per (head, channel)."""
    sc = rng.uniform(0.5, 3.0, (h, d)).astype(np.float32)
    off = (rng.standard_normal((h, d)) * 2.0).astype(np.float32)
    return (rng.standard_normal((n, h, d)).astype(np.float32) * sc + off).astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from src.quantize_int4_ref import quantize_int4_ref
    from src.flash_decode_ref import online_softmax_ref
    from src.int4_pack import pack_int4, unpack_int4

    # ---------------- quantizer ----------------
    quant = {}

    def add_q(name, kv):
        q, s, z = quantize_int4_ref(kv, per_channel=True)
        quant[f"{name}/kv"] = kv
        quant[f"{name}/q"] = q
        quant[f"{name}/scale"] = s
        quant[f"{name}/zp"] = z

    add_q("kat_scales", np.array([[[1.0, 2.0], [3.0, 4.0], [5.0, 6.0]],
                                  [[7.0, 8.0], [9.0, 10.0], [11.0, 12.0]]], np.float32))
    add_q("uniform", np.full((2, 4, 16), 5.0, np.float32))
    add_q("tiny_range", np.array([1.0000, 1.0001, 1.0002], np.float32)[:, None])
    add_q("large_negative", np.array([-1000.0, -100.0, -10.0, 0.0], np.float32)[:, None])
    add_q("mixed_magnitude", np.array([1e-6, 1e-3, 1.0, 1e3, 1e6], np.float32)[:, None])
    # exact .5 ties: min 0, max 15 -> scale 1 -> bins are round-half-even of x
    ties = np.array([0.0, 15.0, 0.5, 1.5, 2.5, 3.5, 4.5, 13.5, 14.5], np.float32)
    add_q("half_even_ties", np.stack([ties, ties * 2.0], axis=1))
    add_q("dispatch_256x64", np.random.RandomState(1).randn(256, 64).astype(np.float32))
    add_q("parity_512x32", np.random.RandomState(3).randn(512, 32).astype(np.float32))
    for shape in [(1, 1), (1, 64), (255, 3), (256, 3), (257, 3), (1030, 8), (1024, 32)]:
        add_q(f"shape_{shape[0]}x{shape[1]}",
              np.random.RandomState(shape[0]).randn(*shape).astype(np.float32))
    add_q("randn_3d", np.random.RandomState(42).randn(4, 8, 64).astype(np.float32))

    # grouped (benchmark config 1 layout): one reference call per (group, head)
    for name, (n, h, d, seed) in {"grouped_300x4x64": (300, 4, 64, 7),
                                  "grouped_256x1x128": (256, 1, 128, 8),
                                  "grouped_77x3x32": (77, 3, 32, 9)}.items():
        kv = anchor_keys(np.random.default_rng(seed), n, h, d)
        g = (n + 127) // 128
        q = np.zeros((n, h, d), np.uint8)
        sc = np.zeros((g, h, d), np.float32)
        zp = np.zeros((g, h, d), np.float32)
        for gi in range(g):
            for hi in range(h):
                qq, ss, zz = quantize_int4_ref(kv[gi * 128:(gi + 1) * 128, hi, :], per_channel=True)
                q[gi * 128:gi * 128 + qq.shape[0], hi] = qq
                sc[gi, hi] = ss
                zp[gi, hi] = zz
        quant[f"{name}/kv"] = kv
        quant[f"{name}/q"] = q
        quant[f"{name}/scale"] = sc
        quant[f"{name}/zp"] = zp
    np.savez_compressed(os.path.join(HERE, "golden_quant.npz"), **quant)

    # ---------------- packing ----------------
    pack = {}
    for name, q in {"extremes": np.array([[0, 15, 15, 0, 7, 8]], np.uint8),
                    "even_256x64": np.random.RandomState(0).randint(0, 16, (256, 64), dtype=np.uint8),
                    "odd_10x7": np.random.RandomState(1).randint(0, 16, (10, 7), dtype=np.uint8),
                    "three_d": np.random.RandomState(2).randint(0, 16, (4, 128, 32), dtype=np.uint8)}.items():
        p = pack_int4(q)
        pack[f"{name}/q"] = q
        pack[f"{name}/packed"] = p
        pack[f"{name}/unpacked"] = unpack_int4(p, q.shape[-1])
    np.savez_compressed(os.path.join(HERE, "golden_pack.npz"), **pack)

    # ---------------- attention: page-list form (legacy shared stream) ----------------
    attn = {}

    def paged_problem(batch, heads, dim, n_blocks, rows, seed, scale_query=True):
        rng = np.random.RandomState(seed)
        query = rng.randn(batch, heads, dim)
        if scale_query:
            query = query / np.sqrt(dim)
        query = query.astype(np.float32)
        kq, ks, kz, vv = [], [], [], []
        for _ in range(n_blocks):
            k = rng.randn(rows, dim).astype(np.float32)
            v = rng.randn(rows, dim).astype(np.float32)
            q_, s_, z_ = quantize_int4_ref(k, per_channel=True)
            kq.append(q_); ks.append(s_); kz.append(z_); vv.append(v)
        return query, kq, ks, kz, vv

    def add_a(name, query, kq, ks, kz, vv, lens):
        lens = np.asarray(lens, np.int32)
        out, _ = online_softmax_ref(query, list(zip(kq, ks, kz)), vv, lens)
        attn[f"{name}/query"] = query
        attn[f"{name}/n_blocks"] = np.int32(len(kq))
        for i in range(len(kq)):
            attn[f"{name}/kq{i}"] = kq[i]
            attn[f"{name}/s{i}"] = ks[i]
            attn[f"{name}/z{i}"] = kz[i]
            attn[f"{name}/v{i}"] = vv[i]
        attn[f"{name}/lens"] = lens
        attn[f"{name}/out"] = out

    add_a("ragged_64_0_17", *paged_problem(2, 3, 32, 3, 64, 0), [64, 0, 17])
    add_a("full_pages", *paged_problem(2, 4, 64, 4, 96, 4, scale_query=False), [96] * 4)
    add_a("first_page_empty", *paged_problem(1, 2, 64, 3, 64, 6, scale_query=False), [0, 64, 64])
    add_a("all_empty", *paged_problem(1, 2, 64, 3, 64, 5, scale_query=False), [0, 0, 0])
    add_a("empty_middle", *paged_problem(2, 4, 64, 4, 128, 4, scale_query=False), [128, 0, 64, 128])
    for dim in [1, 2, 31, 33, 127, 129, 255, 256]:
        add_a(f"head_dim_{dim}", *paged_problem(2, 3, dim, 3, 40, dim), [40, 17, 40])
    for rows in [1, 3, 5, 129]:
        add_a(f"page_rows_{rows}", *paged_problem(2, 3, 64, 3, rows, rows), [rows] * 3)

    # ---------------- attention: paged per-(sequence, head) streams, anchor distribution ----------------
    def paged_anchor(name, batch, heads, dim, lens, pool_pages, seed, page=16, group=128):
        rng = np.random.default_rng(seed)
        gp = group // page
        maxp = max(1, max((l + page - 1) // page for l in lens))
        query = rng.standard_normal((batch, heads, dim)).astype(np.float32)
        k_pool = np.zeros((pool_pages, heads, page, (dim + 1) // 2), np.uint8)
        v_pool = np.zeros((pool_pages, heads, page, dim), np.float32)
        sz_pool = np.zeros((pool_pages, heads, 2, dim), np.float32)
        perm = rng.permutation(pool_pages)
        bt = np.zeros((batch, maxp), np.int32)
        cursor = 0
        out = np.zeros((batch, heads, dim), np.float32)
        for b, n in enumerate(lens):
            np_b = (n + page - 1) // page
            bt[b, :np_b] = perm[cursor:cursor + np_b]
            cursor += np_b
            if n == 0:
                continue
            keys = anchor_keys(rng, n, heads, dim)
            vals = rng.standard_normal((n, heads, dim)).astype(np.float32)
            for h in range(heads):
                pages, vpages = [], []
                for g in range((n + group - 1) // group):
                    qg, sg, zg = quantize_int4_ref(keys[g * group:(g + 1) * group, h, :], per_channel=True)
                    gphys = bt[b, g * gp]
                    sz_pool[gphys, h, 0] = sg
                    sz_pool[gphys, h, 1] = zg
                    packed = pack_int4(qg)
                    for pi in range((qg.shape[0] + page - 1) // page):
                        p = g * gp + pi
                        rows = min(page, n - p * page)
                        phys = bt[b, p]
                        k_pool[phys, h, :rows] = packed[pi * page:pi * page + rows]
                        v_pool[phys, h, :rows] = vals[p * page:p * page + rows, h]
                        pages.append((unpack_int4(k_pool[phys, h, :rows], dim), sg, zg))
                        vpages.append(v_pool[phys, h, :rows])
                o, _ = online_softmax_ref(query[b:b + 1, h:h + 1], pages, vpages)
                out[b, h] = o[0, 0]
        attn[f"{name}/query"] = query
        attn[f"{name}/k_pool"] = k_pool
        attn[f"{name}/v_pool"] = v_pool
        attn[f"{name}/sz_pool"] = sz_pool
        attn[f"{name}/block_table"] = bt
        attn[f"{name}/seq_lens"] = np.asarray(lens, np.int32)
        attn[f"{name}/out"] = out

    paged_anchor("paged_anchor_d128", 3, 2, 128, [300, 517, 0], 56, 11)
    paged_anchor("paged_anchor_d64", 2, 2, 64, [256, 141], 28, 12)
    np.savez_compressed(os.path.join(HERE, "golden_attn.npz"), **attn)
    for f in ("golden_quant.npz", "golden_pack.npz", "golden_attn.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
