"""Test helpers: package import, golden fixtures, oracle-side pool building."""

import importlib
import os

import numpy as np

PKG_NAME = "int4-kv-cache-quantization-cuda-triton-pallas_b200"
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def pkg(mod=None):
    return importlib.import_module(PKG_NAME + ("." + mod if mod else ""))


def golden(name):
    """Load tests/golden/<name>.npz as {case: {field: array}}."""
    data = np.load(os.path.join(GOLDEN, name + ".npz"))
    cases = {}
    for key in data.files:
        case, field = key.split("/", 1)
        cases.setdefault(case, {})[field] = data[key]
    return cases


def attn_case_lists(c):
    n = int(c["n_blocks"])
    kq = [c[f"kq{i}"] for i in range(n)]
    s = [c[f"s{i}"] for i in range(n)]
    z = [c[f"z{i}"] for i in range(n)]
    v = [c[f"v{i}"] for i in range(n)]
    return c["query"], kq, s, z, v, c["lens"]


def oracle_build_pools(problem, page=16):
    """Quantize + pack + scatter a host paged problem with the ORACLE (the checker side)."""
    import oracle
    heads = problem["query"].shape[1]
    d = problem["query"].shape[2]
    pool = problem["pool_pages"]
    group = problem["group"]
    gp = group // page
    bt = problem["block_table"]
    k_pool = np.zeros((pool, heads, page, d // 2), np.uint8)
    v_pool = np.zeros((pool, heads, page, d), np.float32)
    sz_pool = np.zeros((pool, heads, 2, d), np.float32)
    for b, (k, v) in enumerate(zip(problem["keys"], problem["values"])):
        n = k.shape[0]
        if n == 0:
            continue
        q, s, z = oracle.quantize_grouped(k, group)
        packed = oracle.pack_int4(q)
        for p in range((n + page - 1) // page):
            rows = min(page, n - p * page)
            phys = bt[b, p]
            k_pool[phys, :, :rows] = packed[p * page:p * page + rows].transpose(1, 0, 2)
            v_pool[phys, :, :rows] = v[p * page:p * page + rows].transpose(1, 0, 2)
        for g in range(s.shape[0]):
            slot = bt[b, g * gp]
            sz_pool[slot, :, 0] = s[g]
            sz_pool[slot, :, 1] = z[g]
    return k_pool, v_pool, sz_pool
