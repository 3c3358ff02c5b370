"""Sequence split across GPUs, one process per GPU (run under torchrun).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 tests/dist_sequence_split.py \
        [L] [heads] [nccl|p2p|fused]

Every rank generates the same seeded sequence, keeps its group-aligned token
range in a paged cache on its own GPU, decodes it into partial records, and
``SequenceSplitDecoder`` exchanges the records -- one NCCL all-gather, the
peer-memory exchange kernel (``p2p``), or inside the decode kernel itself
(``fused``) -- and merges them. Each rank checks the merged output against a whole-sequence
decode on its own GPU; exit status 0 means every rank matched.
"""

import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import importlib  # noqa: E402

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

PKG = "int4-kv-cache-quantization-cuda-triton-pallas_b200"


def main():
    L = int(sys.argv[1]) if len(sys.argv) > 1 else 131072
    heads = int(sys.argv[2]) if len(sys.argv) > 2 else 32
    exchange = sys.argv[3] if len(sys.argv) > 3 else "nccl"
    d = 128
    rank, world, local = (int(os.environ[k]) for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    P = importlib.import_module(PKG + ".paged")
    par = importlib.import_module(PKG + ".parallel")
    g = torch.Generator(device="cuda").manual_seed(1234)
    sc = torch.rand((heads, d), generator=g, device="cuda") * 2.5 + 0.5
    off = torch.randn((heads, d), generator=g, device="cuda") * 2.0
    k = torch.randn((L, heads, d), generator=g, device="cuda") * sc + off
    v = torch.randn((L, heads, d), generator=g, device="cuda")
    q = torch.randn((1, heads, d), generator=g, device="cuda")
    t0, t1 = par.plan_sequence_split(L, world)[rank]
    cache = P.PagedKVCache((t1 - t0 + 15) // 16 + 8, heads, d, device="cuda", seed=rank)
    cache.write_sequences([0], [k[t0:t1]], [v[t0:t1]])
    store = dist.distributed_c10d._get_default_store()
    dec = par.SequenceSplitDecoder(cache, rank, world,
                                   monitor=par.PeerMonitor(store, rank, world, timeout=30.0),
                                   exchange=exchange)
    out = dec.decode(q)
    full = P.PagedKVCache((L + 15) // 16 + 8, heads, d, device="cuda", seed=99)
    full.write_sequences([0], [k], [v])
    want = full.decode(q, [0])
    err = float((out - want).abs().max())
    # the same step as a CUDA graph, replayed on a new query written into its input buffer
    dec.capture(q)
    q.copy_(torch.randn((1, heads, d), generator=g, device="cuda"))
    got = dec.replay().clone()
    gerr = float((got - full.decode(q, [0])).abs().max())
    # a second eager step after the replays (the exchange's step counters advance)
    q.copy_(torch.randn((1, heads, d), generator=g, device="cuda"))
    serr = float((dec.decode(q) - full.decode(q, [0])).abs().max())
    status = dec.peer_status()
    dec.close()
    torch.cuda.synchronize()
    good_rank = max(err, gerr, serr) <= 2e-6 and bool(torch.isfinite(out).all()) and status == 0
    ok = torch.tensor([1.0 if good_rank else 0.0], device="cuda")
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    print(f"rank {rank} ({exchange}): range [{t0}, {t1}) max|split - whole| = {err:.3e}, "
          f"graph replay {gerr:.3e}, next step {serr:.3e}, status {status}", flush=True)
    good = bool(ok.item() == 1.0)
    dist.destroy_process_group()
    sys.exit(0 if good else 1)


if __name__ == "__main__":
    main()
