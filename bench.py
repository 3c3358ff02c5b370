#!/usr/bin/env python
"""Benchmark: fused INT4 paged flash-decode attention on B200 (+ quantizer GB/s).

One step = one decode-attention pass of benchmark config 0 per GPU
(8 sequences x 32 heads x d128 x 2048 tokens, 16-token pages in a seeded
random block table, INT4 keys with per-(128-token group, head, channel)
scale/zp, fp32 values), inputs resident in HBM. With N GPUs every rank owns
its own config-0 batch (batch x heads sharded, no collective): weak scaling.

Prints ONE JSON line (rank 0). `value` = algorithmic HBM bytes of all ranks
per step / step time (max over ranks), in GB/s. The step time is K steps back
to back between one pair of CUDA events after a barrier and a synchronize,
with no L2 flush where a step's inputs exceed twice the 126 MB L2 (config 0:
306.5 MB); otherwise the L2 is flushed before every step and each step is
timed with its own events. The flushed, per-launch figures are reported
beside the headline under `flushed`.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's own CPU implementation of the path
(the NumPy oracle restated in oracle/, all host cores) on the same workload.
"""

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PKG = "int4-kv-cache-quantization-cuda-triton-pallas_b200"
METRIC = "INT4 paged decode-attn µs & HBM GB/s (frac of ~8 TB/s); quantizer GB/s"
FALLBACK_HBM_GBS = 6650.0
L2_FLUSH_BYTES = 256 << 20


class MappedHostBuffer:
    """Pinned host memory mapped into the device's address space
    (cudaHostAlloc with cudaHostAllocMapped): kernels store to `device_ptr`,
    the host reads the same bytes through `array()`."""

    def __init__(self, nbytes):
        import ctypes
        from cuda.bindings import runtime as rt
        self._rt, self._ctypes, self.nbytes = rt, ctypes, nbytes
        err, self.host_ptr = rt.cudaHostAlloc(nbytes, rt.cudaHostAllocMapped)
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"cudaHostAlloc failed: {err}")
        err, self.device_ptr = rt.cudaHostGetDevicePointer(self.host_ptr, 0)
        if err != rt.cudaError_t.cudaSuccess:
            rt.cudaFreeHost(self.host_ptr)
            raise RuntimeError(f"cudaHostGetDevicePointer failed: {err}")

    def array(self, dtype):
        buf = (self._ctypes.c_uint8 * self.nbytes).from_address(self.host_ptr)
        return np.frombuffer(buf, dtype=dtype)

    def free(self):
        if self.host_ptr:
            self._rt.cudaFreeHost(self.host_ptr)
            self.host_ptr = 0


class L2Flush:
    """Evict L2 between timed steps: write a buffer larger than L2, then read a
    second one, so the written lines are written back before the next timed
    kernel starts (their write-back would otherwise be charged to it)."""

    def __init__(self, torch):
        self.w = torch.empty((L2_FLUSH_BYTES,), dtype=torch.uint8, device="cuda")
        self.r = torch.ones((L2_FLUSH_BYTES // 4,), dtype=torch.float32, device="cuda")
        self.sink = torch.empty((1,), dtype=torch.float32, device="cuda")

    def __call__(self, i):
        self.w.fill_(i & 255)
        self.sink.copy_(self.r.sum(dim=0, keepdim=True))


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="cfg0")
    ap.add_argument("--e2e-steps", type=int, default=300)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-quantizer", action="store_true")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl", "fused"],
                    help="sequence split (cfg4_long, N>1): fused peer-memory exchange kernel "
                         "or NCCL all-gather + merge kernel")
    ap.add_argument("--values", default="f32", choices=["f32", "f16", "bf16"],
                    help="value-pool storage type (keys are INT4 either way)")
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip the config 2 / config 3 sweep and the reference-API records (N=1)")
    ap.add_argument("--no-split", action="store_true",
                    help="skip the sequence-split leg of a multi-GPU run")
    ap.add_argument("--rank-seeds", action="store_true",
                    help="N>1: each rank draws its own config-0 problem (seed 7 + 1000 * rank) "
                         "instead of rank 0's, and also re-times rank 0's problem on every rank")
    ap.add_argument("--reference-api-only", action="store_true",
                    help="time only the reference's two drop-in launchers (cu_flash_decode_int4, "
                         "cu_quantize_int4) at its published shapes and print that record")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic():
    """DRAM bytes per launch of the decode kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "paged_decode_cfg0.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


def workload_config(shape, name, world):
    lens = shape.seq_lens
    if min(lens) == max(lens):
        tokens = f"{lens[0]} tokens"
        seq_len = lens[0]
    else:
        tokens = f"{min(lens)}..{max(lens)} tokens (mean {sum(lens) / len(lens):.0f}, ragged)"
        seq_len = {"min": min(lens), "max": max(lens), "mean": round(sum(lens) / len(lens), 1)}
    heads = (f"{shape.heads} heads" if shape.query_heads == shape.heads else
             f"{shape.query_heads} query heads over {shape.heads} kv heads (GQA)")
    return {"workload": f"{name}: decode step, batch {shape.batch} x {heads} x "
                        f"d{shape.head_dim} x {tokens} per GPU, 16-token pages "
                        "(seeded random block table), INT4 keys / 128-token groups, fp32 q, "
                        f"{'fp32' if shape.value_bytes == 4 else '16-bit'} values",
            "batch_per_gpu": shape.batch, "global_batch": shape.batch * world,
            "heads": shape.query_heads, "kv_heads": shape.heads, "head_dim": shape.head_dim,
            "seq_len": seq_len,
            "page_tokens": 16, "group_tokens": shape.group_tokens,
            "l2": (f"not flushed between steps: inputs {shape.algorithmic_bytes() / 1e6:.1f} MB/GPU "
                   "> 2 x 126 MB L2" if shape.algorithmic_bytes() > 2 * 126e6 else
                   "flushed (256 MiB write + 256 MiB read, untimed) before every timed step; "
                   f"inputs {shape.algorithmic_bytes() / 1e6:.1f} MB/GPU"),
            "parallelism": f"dp{world} (batch x heads sharded, no collective)"}


def _nvml_handle(nv, index):
    """The NVML handle of CUDA device `index`, matched by PCI bus id (NVML and
    CUDA may number the GPUs differently); by index if that fails."""
    try:
        import torch
        pr = torch.cuda.get_device_properties(index)
        bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        return nv.nvmlDeviceGetHandleByPciBusId(bus)
    except Exception:
        return nv.nvmlDeviceGetHandleByIndex(index)


class ClockSampler:
    """NVML sampling of SM and memory clocks and throttle reasons in a
    background thread."""

    def __init__(self, index, period=0.002):
        self.samples = []
        self.ok = False
        self._stop = threading.Event()
        self._mark = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = _nvml_handle(pynvml, index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self.period = period

    def _reasons(self):
        nv = self._nv
        try:
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except Exception:
            r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
        names = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
                 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
                 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}
        return [n for bit, n in names.items() if r & bit]

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM)
                mem = self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_MEM)
                self.samples.append((time.perf_counter(), mhz, self._reasons(), mem))
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def mark(self, t0, t1):
        self._mark = (t0, t1)

    def stop(self):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        t0, t1 = self._mark if self._mark else (-1e30, 1e30)
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        use = inside if len(inside) >= 3 else self.samples
        reasons = sorted({r for s in use for r in s[2]} - {"gpu_idle"})
        return {"sm_mhz": statistics.median(s[1] for s in use), "sm_max_mhz": self.max_mhz,
                "mem_mhz": statistics.median(s[3] for s in use),
                "reasons": reasons, "samples": len(use), "period_ms": round(self.period * 1e3, 1),
                "window": (self.window if use is inside else "warmup + timed loops")}

    window = "timed region"


CLOCK_REASONS = ("applications_clocks_setting", "sw_power_cap", "hw_slowdown",
                 "sw_thermal_slowdown", "hw_thermal_slowdown", "hw_power_brake_slowdown",
                 "display_clock_setting")


def _all_reduce_max(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_baseline(arrays, streams, bytes_per_stream, seconds_target=2.0):
    """Time the oracle (spawn pool, all host cores) on a bounded sample of streams."""
    from oracle.cpu_pool import OraclePool
    pool = OraclePool(arrays)
    try:
        reps, wall = 0, 0.0
        while wall < seconds_target or reps == 0:
            dt, outs = pool.run(streams)
            wall += dt
            reps += 1
    finally:
        pool.close()
    gbs = reps * len(streams) * bytes_per_stream / wall / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": pool.procs, "kind": "port",
            "host_cpu_count": os.cpu_count(), "host_affinity": len(os.sched_getaffinity(0)),
            "threads": f"{pool.procs} spawn processes x 1 thread "
                       "(OMP/OPENBLAS/MKL_NUM_THREADS=1 in each)",
            "sample": f"{len(streams)} of the config's (sequence, head) streams x {reps} reps, "
                      f"oracle online softmax per stream (NumPy, 1 BLAS thread per process, "
                      f"{pool.procs} spawn processes), {wall:.2f} s wall",
            "ms_per_stream": round(1e3 * wall / (reps * len(streams)) * pool.procs, 3)}, outs


def stream_gate(torch, out, query, cache, bt, sl, streams, group_q=1):
    """Max |gpu - float64 arbiter| over (sequence, kv head) streams, each copied
    off the device on its own (no host copy of a whole pool)."""
    import oracle
    o, q = out.cpu().numpy(), query.cpu().numpy()
    bt_h, sl_h = bt.cpu().numpy(), sl.cpu().numpy()
    G, err = group_q, 0.0
    for b, h in streams:
        n = int(sl_h[b])
        got = o[b, h * G:(h + 1) * G]
        if n == 0:
            err = max(err, float(np.abs(got).max()))
            continue
        pages = torch.as_tensor(bt_h[b, :(n + 15) // 16].astype(np.int64), device=out.device)
        ex = oracle.stream_f64(q[b, h * G:(h + 1) * G], cache.k_pool[pages, h].cpu().numpy(),
                               cache.v_pool[pages, h].float().cpu().numpy(),
                               cache.sz_pool[pages, h].cpu().numpy(), n)
        err = max(err, float(np.abs(got - ex).max()))
    return err


def decode_timing(torch, lib, C, shape, prob, vdtype, K, flush, gate_streams=4, seed=0,
                  b2b=False, copies=()):
    """CUDA-event time of the decode kernel alone (events recorded by the C ABI
    around the launch) on a built problem, L2 flushed before every launch,
    behind a float64 gate on `gate_streams` seeded streams. With `b2b`, also K
    launches back to back between one pair of events with no flush, rotating
    over the problem and its `copies` (more problems of the same shape, each
    gated the same way) so that the bytes a launch reads were last read
    len(copies) launches earlier: the caller passes enough copies that this is
    more than twice the L2."""
    import ctypes
    cache, query = prob["cache"], prob["query"]
    ids = list(range(shape.batch))
    bt, sl = cache.block_table(ids)
    hq, h, d = shape.query_heads, shape.heads, shape.head_dim
    ws_bytes = C.paged_decode_workspace_bytes(shape.batch, hq, h, d, value_dtype=vdtype)
    ws = torch.zeros((ws_bytes,), dtype=torch.uint8, device="cuda")
    out = torch.empty_like(query)
    stream = torch.cuda.current_stream()
    vk = C.VALUE_KINDS[vdtype]
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(K)]
    for a, b in ev:
        a.record()
        b.record()

    def args_of(p):
        c, q = p["cache"], p["query"]
        b_t, s_l = (bt, sl) if p is prob else c.block_table(ids)
        return (q.data_ptr(), c.k_pool.data_ptr(), c.v_pool.data_ptr(), vk, c.sz_pool.data_ptr(),
                b_t.data_ptr(), s_l.data_ptr(), shape.batch, hq, h, d, 16, shape.group_tokens,
                b_t.shape[1], c.num_pages, out.data_ptr(), ws.data_ptr(), ws_bytes, None,
                stream.cuda_stream), (b_t, s_l)

    a0, _ = args_of(prob)

    def launch(e0=None, e1=None, a=a0):
        rc = lib.int4kv_paged_decode_ex(*a, e0, e1)
        if rc:
            raise RuntimeError(f"decode launch failed: cudaError {rc}")

    launch()
    torch.cuda.synchronize()
    rng = np.random.default_rng(seed)
    streams = sorted({(int(b), int(x)) for b, x in zip(rng.integers(0, shape.batch, gate_streams),
                                                       rng.integers(0, h, gate_streams))})
    gate = stream_gate(torch, out, query, cache, bt, sl, streams, hq // h)
    if not (torch.isfinite(out).all() and gate <= 1e-6):
        raise RuntimeError(f"decode failed its correctness gate (max err {gate}); not timing")
    for i in range(3):
        flush(i)
        launch()
    for i, (a, b) in enumerate(ev):
        flush(i)
        launch(ctypes.c_void_p(a.cuda_event), ctypes.c_void_p(b.cuda_event))
    torch.cuda.synchronize()
    us = [a.elapsed_time(b) * 1e3 for a, b in ev]
    rec = {"kernel_us": round(sum(us) / K, 2), "kernel_us_p50": round(float(np.median(us)), 2),
           "gate_streams": len(streams), "max_abs_vs_f64_arbiter": gate}
    if b2b:
        rot = [args_of(p) for p in (prob,) + tuple(copies)]  # keeps each copy's tables alive
        for p, (a, (b_t, s_l)) in zip((prob,) + tuple(copies), rot):
            launch(a=a)
            torch.cuda.synchronize()
            g = stream_gate(torch, out, p["query"], p["cache"], b_t, s_l, streams, hq // h)
            if not (torch.isfinite(out).all() and g <= 1e-6):
                raise RuntimeError(f"decode failed its correctness gate on a copy (max err {g})")
            rec["max_abs_vs_f64_arbiter"] = max(rec["max_abs_vs_f64_arbiter"], g)
        for i in range(max(3, len(rot))):  # untimed: the rotation once round
            launch(a=rot[i % len(rot)][0])
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record()
        for i in range(K):
            launch(a=rot[i % len(rot)][0])
        b1.record()
        torch.cuda.synchronize()
        rec["back_to_back_us"] = round(b0.elapsed_time(b1) * 1e3 / K, 2)
        rec["back_to_back_problems"] = len(rot)
    return rec


def sweep_records(torch, lib, C, W, K, flush, peak):
    """The other decode configurations of the benchmark definition on this GPU:
    config 2's context sweep and config 3's ragged batch (d64, d128); then
    config 0's shape with grouped-query heads (32 query heads over 8 and 4 kv
    heads), the same at 32768 tokens (over 8 kv heads), and config 0 with
    16-bit value pools."""
    recs = {}
    runs = [(n, n, torch.float32) for n in ("cfg2_512", "cfg2_8192", "cfg2_32768", "cfg3_d64",
                                            "cfg3_d128", "cfg0_gqa4", "cfg0_gqa8",
                                            "cfg2_32768_gqa4")]
    runs += [("cfg0_f16", "cfg0", torch.float16), ("cfg0_bf16", "cfg0", torch.bfloat16)]
    for label, name, vdtype in runs:
        shape = W.config_shape(name)
        shape.value_bytes = 4 if vdtype == torch.float32 else 2
        prob = W.torch_build_cache(shape, seed=7, value_dtype=vdtype)
        nbytes = shape.algorithmic_bytes()
        # back to back: the problem alone when it is more than twice the 126 MB
        # L2, else rotating over it and copies with other seeds, so that more
        # than twice the L2 is read between two reads of the same bytes
        l2x2 = 2 * 126_000_000
        ncopy = 0 if nbytes > l2x2 else -(-l2x2 // nbytes)
        copies = tuple(W.torch_build_cache(shape, seed=8 + i, value_dtype=vdtype)
                       for i in range(ncopy))
        r = decode_timing(torch, lib, C, shape, prob, vdtype, K, flush, seed=1, b2b=True,
                          copies=copies)
        r.update({"algorithmic_bytes": nbytes,
                  "gbs": round(nbytes / (r["kernel_us"] * 1e-6) / 1e9, 1),
                  "frac": round(nbytes / (r["kernel_us"] * 1e-6) / 1e9 / peak, 4),
                  "back_to_back_frac": round(nbytes / (r["back_to_back_us"] * 1e-6) / 1e9 / peak,
                                             4)})
        recs[label] = r
        del prob, copies
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return recs


def reference_api_records(torch, lib, flush):
    """The reference's own two launchers, through their drop-in C signatures, at
    the shapes its published H100 numbers are quoted on:
    cu_flash_decode_int4 at b8 x h32 x d128 x s2048 (one shared stream of
    256-row pages, one code per byte, float32 values;
    results/three_backend_attention_h100.json:187 of the reference, 0.400 ms)
    and cu_quantize_int4 at 32768 x 128 (results/three_backend_quantize_h100.json:237,
    0.150 ms). Inputs as the reference's benchmark builds them
    (benchmarks/bench_three_backend.py:113-129): randn query, keys and values,
    keys quantized per block."""
    import oracle
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.RandomState(1234)
    B, H, D, bs, L = 8, 32, 128, 256, 2048
    nb = L // bs
    query = rng.randn(B, H, D).astype(np.float32)
    kq, ks, kz, vv = [], [], [], []
    for _ in range(nb):
        k = rng.randn(bs, D).astype(np.float32)
        vv.append(rng.randn(bs, D).astype(np.float32))
        q_, s_, z_ = oracle.quantize_int4(k)
        kq.append(q_), ks.append(s_), kz.append(z_)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    tq, tk, ts, tz, tv = dev(query), dev(np.stack(kq)), dev(np.stack(ks)), dev(np.stack(kz)), dev(np.stack(vv))
    tl = torch.full((nb,), bs, dtype=torch.int32, device="cuda")
    out = torch.empty((B, H, D), device="cuda")

    def attn():
        rc = lib.cu_flash_decode_int4(tq.data_ptr(), tk.data_ptr(), ts.data_ptr(), tz.data_ptr(),
                                      tv.data_ptr(), tl.data_ptr(), B, H, D, nb, bs,
                                      out.data_ptr(), stream)
        if rc:
            raise RuntimeError(f"cu_flash_decode_int4 failed: cudaError {rc}")

    attn()
    torch.cuda.synchronize()
    pages = list(zip(kq, ks, kz))
    gate = float(np.abs(out.cpu().numpy() - oracle.attention_f64(query, pages, vv)).max())
    ref32 = float(np.abs(out.cpu().numpy() - oracle.online_softmax(query, pages, vv)[0]).max())
    if not gate <= 1e-6:
        raise RuntimeError(f"cu_flash_decode_int4 failed its gate ({gate}); not timing")

    rows, ch = 32768, 128
    kv = torch.from_numpy(np.random.RandomState(4321).randn(rows, ch).astype(np.float32)).cuda()
    q_out = torch.empty((rows, ch), dtype=torch.uint8, device="cuda")
    s_out = torch.empty((ch,), device="cuda")
    z_out = torch.empty((ch,), device="cuda")

    def quant():
        rc = lib.cu_quantize_int4(kv.data_ptr(), rows, ch, q_out.data_ptr(), s_out.data_ptr(),
                                  z_out.data_ptr(), stream)
        if rc:
            raise RuntimeError(f"cu_quantize_int4 failed: cudaError {rc}")

    quant()
    torch.cuda.synchronize()
    q_r, s_r, z_r = oracle.quantize_int4(kv.cpu().numpy())
    exact = (np.array_equal(q_out.cpu().numpy(), q_r)
             and np.array_equal(s_out.cpu().numpy().view(np.uint32), s_r.view(np.uint32))
             and np.array_equal(z_out.cpu().numpy().view(np.uint32), z_r.view(np.uint32)))
    if not exact:
        raise RuntimeError("cu_quantize_int4 is not bit-exact with the oracle; not timing")

    def timed(fn, n, flushed):
        for i in range(3):
            fn()
        if not flushed:
            # the reference's method (benchmarks/bench_three_backend.py:273-291):
            # n launches back to back, one pair of CUDA events around the loop
            b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            b0.record()
            for i in range(n):
                fn()
            b1.record()
            torch.cuda.synchronize()
            return round(b0.elapsed_time(b1) / n * 1e3, 2)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(n)]
        for i, (a, b) in enumerate(ev):
            if flushed:
                flush(i)
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return round(sum(a.elapsed_time(b) for a, b in ev) / n * 1e3, 2)

    a_warm, a_cold = timed(attn, 50, False), timed(attn, 50, True)
    q_warm, q_cold = timed(quant, 50, False), timed(quant, 50, True)
    return {
        "cu_flash_decode_int4": {
            "shape": "b8 x h32 x d128, one shared stream of 2048 tokens in 8 pages of 256 rows, "
                     "1-byte codes, float32 values",
            "us_back_to_back": a_warm, "us_l2_flushed": a_cold,
            "reference_h100_us": 400.0,
            "speedup_vs_reference_h100": round(400.0 / a_warm, 2),
            "max_abs_vs_f64_arbiter": gate, "max_abs_vs_oracle_fp32": ref32},
        "cu_quantize_int4": {
            "shape": "32768 rows x 128 channels, group = all rows, 1-byte codes",
            "us_back_to_back": q_warm, "us_l2_flushed": q_cold,
            "gbs_l2_flushed": round((rows * ch * 5 + 8 * ch) / (q_cold * 1e-6) / 1e9, 1),
            "reference_h100_us": 150.0,
            "speedup_vs_reference_h100": round(150.0 / q_warm, 2), "bit_exact": exact},
        "timing": "us_back_to_back: n C-ABI calls back to back between one pair of CUDA "
                  "events, the reference's own method (benchmarks/bench_three_backend.py:"
                  "273-291: back-to-back launches on device-resident inputs, one sync after "
                  "the loop); us_l2_flushed: CUDA events around each call, L2 flushed before it",
    }


def gather_per_rank(torch, vals, world):
    """[[rank 0 values], [rank 1 values], ...] on every rank (one all-gather)."""
    if world == 1:
        return [list(vals)]
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    outs = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(outs, t)
    return [o.tolist() for o in outs]


# --------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------

def run_ours(args):
    import ctypes
    import importlib
    import torch
    rank, world, local = dist_env()
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    importlib.import_module(PKG + "._build").build()
    W = importlib.import_module(PKG + ".workloads")
    C = importlib.import_module(PKG + "._C")
    lib = importlib.import_module(PKG + "._lib").load()

    shape = W.config_shape(args.config)
    vdtype = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[args.values]
    shape.value_bytes = 4 if args.values == "f32" else 2
    # Weak scaling: by default every rank decodes the same seeded problem (rank
    # 0's), so N ranks repeat the one-GPU measurement. The kernel's time
    # depends on where the block table puts the pages (measured on one B200:
    # 61.9-66.5 us over 8 seeds; the table, not the data, sets it), so
    # per-rank problems (--rank-seeds) would add that spread to the max over
    # ranks.
    seed = 7 + 1000 * rank if args.rank_seeds else 7
    prob = W.torch_build_cache(shape, seed=seed, value_dtype=vdtype)
    cache, query = prob["cache"], prob["query"]
    ids = list(range(shape.batch))
    bt, sl = cache.block_table(ids)
    d, h, hq = shape.head_dim, shape.heads, shape.query_heads
    out = torch.empty_like(query)
    ws_bytes = C.paged_decode_workspace_bytes(shape.batch, hq, h, d, value_dtype=vdtype)
    vk = C.VALUE_KINDS[vdtype]
    ws = torch.zeros((ws_bytes,), dtype=torch.uint8, device="cuda")  # zero-filled once
    stream = torch.cuda.current_stream()
    maxp, npages = bt.shape[1], cache.num_pages

    def call_args(q_ptr, out_ptr, ev0=None, ev1=None):
        return (q_ptr, cache.k_pool.data_ptr(), cache.v_pool.data_ptr(), vk,
                cache.sz_pool.data_ptr(), bt.data_ptr(), sl.data_ptr(), shape.batch, hq, h, d, 16,
                shape.group_tokens, maxp, npages, out_ptr, ws.data_ptr(), ws_bytes, None,
                stream.cuda_stream, ev0, ev1)

    # correctness gate before timing: a sample of streams against the float64 arbiter
    C.paged_decode(query, cache.k_pool, cache.v_pool, cache.sz_pool, bt, sl, shape.group_tokens,
                   out=out, workspace=ws)
    torch.cuda.synchronize()
    import oracle
    host = {"query": query.cpu().numpy(), "k_pool": cache.k_pool.cpu().numpy(),
            "v_pool": cache.v_pool.float().cpu().numpy(), "sz_pool": cache.sz_pool.cpu().numpy(),
            "block_table": bt.cpu().numpy(), "seq_lens": sl.cpu().numpy()}
    rng = np.random.default_rng(rank)
    # (sequence, kv head) streams; each covers its G = hq / h query heads
    gate_streams = [(int(b), int(hh)) for b, hh in zip(rng.integers(0, shape.batch, 4),
                                                       rng.integers(0, h, 4))]
    ex = oracle.decode_paged(host["query"], host["k_pool"], host["v_pool"], host["sz_pool"],
                             host["block_table"], host["seq_lens"], method="f64",
                             streams=gate_streams)
    o_host = out.cpu().numpy()
    G = hq // h
    gate_err = max(float(np.abs(o_host[b, hh * G:(hh + 1) * G] - ex[b, hh * G:(hh + 1) * G]).max())
                   for b, hh in gate_streams)
    if not (np.isfinite(o_host).all() and gate_err <= 1e-6):
        raise RuntimeError(f"decode failed its correctness gate (max err {gate_err}); not timing")

    flush = L2Flush(torch)
    K, Wm = args.steps, args.warmup
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    for e in ev:  # materialise the CUDA events so their handles can go through the C ABI
        for x in e:
            x.record()
    torch.cuda.synchronize()
    fn = lib.int4kv_paged_decode_ex
    for i in range(Wm):
        flush(i)
        rc = fn(*call_args(query.data_ptr(), out.data_ptr()))
        if rc:
            raise RuntimeError(f"decode launch failed: cudaError {rc}")
    sampler = ClockSampler(local)
    sampler.start()
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    t_wall0 = time.perf_counter()
    # the step: events around the plain C-ABI call
    step_args = call_args(query.data_ptr(), out.data_ptr())
    for i in range(K):
        flush(i)
        e0, _, _, e3 = ev[i]
        e0.record()
        rc = fn(*step_args)
        e3.record()
        if rc:
            raise RuntimeError(f"decode launch failed: cudaError {rc}")
    torch.cuda.synchronize()
    t_wall1 = time.perf_counter()
    step_ms = [e[0].elapsed_time(e[3]) for e in ev]
    # the kernel alone (roofline): events recorded inside the C-ABI call around
    # the launch, on the launching stream; a separate loop, so these events do
    # not sit inside the step's timed region
    for i in range(K):
        flush(i)
        _, e1, e2, _ = ev[i]
        rc = fn(*call_args(query.data_ptr(), out.data_ptr(), ctypes.c_void_p(e1.cuda_event),
                           ctypes.c_void_p(e2.cuda_event)))
        if rc:
            raise RuntimeError(f"decode launch failed: cudaError {rc}")
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    kern_ms = [e[1].elapsed_time(e[2]) for e in ev]
    mean_step = _all_reduce_max(sum(step_ms) / K, world)
    mean_kern = _all_reduce_max(sum(kern_ms) / K, world)

    # ---- the headline: K steps back to back between one pair of events ----
    # K steps bracketed by a barrier and a device synchronize, no flush between
    # them: the benchmark contract's own procedure (and the reference's,
    # benchmarks/bench_three_backend.py:273-291), valid here because the
    # step's inputs are more than twice the 126 MB L2 -- a launch cannot find
    # the previous launch's bytes there (a streaming read that large evicts
    # them before they are reached again; ncu shows DRAM bytes per launch =
    # algorithmic bytes in this order). Smaller configurations keep the
    # flushed, event-bracketed step above as their headline.
    b2b = None
    bytes_step0 = shape.algorithmic_bytes()
    if bytes_step0 > 2 * 126e6:
        b0 = torch.cuda.Event(enable_timing=True)
        b1 = torch.cuda.Event(enable_timing=True)
        for _ in range(Wm):
            if fn(*step_args):
                raise RuntimeError("decode launch failed")
        torch.cuda.synchronize()
        _barrier(world)
        torch.cuda.synchronize()
        b0.record()
        for _ in range(K):
            rc = fn(*step_args)
            if rc:
                raise RuntimeError(f"decode launch failed: cudaError {rc}")
        b1.record()
        torch.cuda.synchronize()
        b2b_local = b0.elapsed_time(b1) / K
        b2b_ms = _all_reduce_max(b2b_local, world)
        b2b = {"kernel_us": round(b2b_ms * 1e3, 2), "launches": K, "ms": b2b_ms}

    # ---- end to end through the C ABI with host buffers ----
    # The step's inputs (query, block table, lengths) are staged in ONE mapped
    # pinned host buffer and land in one device buffer by one staging launch
    # (int4kv_stage_inputs: SM loads over PCIe, 12.3 us against 17.1 us for the
    # copy engine's cudaMemcpyAsync of the same 135 KB plus a kernel, between
    # events on B200). The decode reads them in place (16-byte aligned views).
    def _al16(n):
        return (n + 15) // 16 * 16
    q_bytes, bt_bytes, sl_bytes = query.numel() * 4, bt.numel() * 4, sl.numel() * 4
    off_bt = _al16(q_bytes)
    off_sl = off_bt + _al16(bt_bytes)
    in_bytes = off_sl + _al16(sl_bytes)
    in_map = MappedHostBuffer(in_bytes)
    in_host = torch.from_numpy(in_map.array(np.uint8))
    in_host.zero_()
    in_host[:q_bytes].view(torch.float32).copy_(query.reshape(-1).cpu())
    in_host[off_bt:off_bt + bt_bytes].view(torch.int32).copy_(bt.reshape(-1).cpu())
    in_host[off_sl:off_sl + sl_bytes].view(torch.int32).copy_(sl.cpu())
    in_dev = torch.empty((in_bytes,), dtype=torch.uint8, device="cuda")
    stage = lib.int4kv_stage_inputs
    stage_args = (ctypes.c_void_p(in_dev.data_ptr()), ctypes.c_void_p(in_map.device_ptr),
                  in_bytes, ctypes.c_void_p(stream.cuda_stream))
    # The output comes back without a copy: the decode stores it straight into
    # mapped pinned host memory (zero-copy; its stores cross PCIe as the last
    # streams finish), which measured 77.8 against 85.5 us per step with a
    # separate device-to-host copy of the 128 KB output.
    out_map = MappedHostBuffer(out.numel() * 4)
    KE = max(1, min(args.e2e_steps, K))
    ee = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(KE)]

    def e2e_args():
        a = list(call_args(in_dev.data_ptr(), out_map.device_ptr))
        a[5], a[6] = in_dev.data_ptr() + off_bt, in_dev.data_ptr() + off_sl
        return a

    ea = e2e_args()
    torch.cuda.synchronize()
    _barrier(world)
    for i in range(KE):
        flush(i)
        ee[i][0].record()
        rc = stage(*stage_args) or fn(*ea)
        ee[i][1].record()
        if rc:
            raise RuntimeError(f"decode launch failed: cudaError {rc}")
    torch.cuda.synchronize()
    e2e_b2b_ms = None
    if b2b is not None:  # the same steps back to back (each still stages its inputs from host)
        _barrier(world)
        torch.cuda.synchronize()
        x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        x0.record()
        for i in range(KE):
            rc = stage(*stage_args) or fn(*ea)
            if rc:
                raise RuntimeError(f"decode launch failed: cudaError {rc}")
        x1.record()
        torch.cuda.synchronize()
        e2e_b2b_ms = _all_reduce_max(x0.elapsed_time(x1) / KE, world)
    t_wall1 = time.perf_counter()
    sampler.window = "timed loops (step, kernel-only, end-to-end)"
    sampler.mark(t_wall0, t_wall1)
    _barrier(world)
    e2e_flushed_ms = _all_reduce_max(sum(a.elapsed_time(b) for a, b in ee) / KE, world)
    e2e_ms = e2e_b2b_ms if e2e_b2b_ms is not None else e2e_flushed_ms
    e2e_out = torch.from_numpy(out_map.array(np.float32).reshape(tuple(out.shape)).copy())
    e2e_diff = float((e2e_out - out.cpu()).abs().max())
    if not (torch.isfinite(e2e_out).all() and e2e_diff <= 1e-6):
        raise RuntimeError(f"end-to-end output differs from the device-resident output ({e2e_diff})")
    out_map.free()
    in_map.free()

    # ---- quantizer GB/s (benchmark config 1), rank-local ----
    quant = None
    if not args.no_quantizer:
        quant = {}
        for n_tok in (2048, 8192, 32768, 131072):
            kv = torch.randn((n_tok, 32, 128), device="cuda")
            C.quantize_int4_grouped(kv, 128)
            evq = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(20)]
            for a, b in evq:
                flush(1)
                a.record()
                C.quantize_int4_grouped(kv, 128)
                b.record()
            torch.cuda.synchronize()
            ms = sum(a.elapsed_time(b) for a, b in evq) / len(evq)
            nbytes = n_tok * 32 * 128 * 4.5 + 2 * 4 * ((n_tok + 127) // 128) * 32 * 128
            quant[str(n_tok)] = {"us": round(ms * 1e3, 2), "gbs": round(nbytes / ms / 1e6, 1)}
            del kv
    sampler.stop()

    # ---- per-rank view of the weak-scaling step (N > 1) ----
    per_rank = None
    if world > 1:
        ck = sampler.summary()
        reason_bits = sum(1 << i for i, n in enumerate(CLOCK_REASONS) if n in ck["reasons"])
        stats = gather_per_rank(torch, [sum(step_ms) / K * 1e3, sum(kern_ms) / K * 1e3, seed,
                                        float(ck["sm_mhz"] or 0), float(ck.get("mem_mhz") or 0),
                                        float(reason_bits),
                                        b2b_local * 1e3 if b2b is not None else 0.0], world)
        per_rank = {"step_us": [round(x[6] if b2b is not None else x[0], 2) for x in stats],
                    "flushed_step_us": [round(x[0], 2) for x in stats],
                    "flushed_kernel_us": [round(x[1], 2) for x in stats],
                    "seed": [int(x[2]) for x in stats],
                    "sm_mhz": [x[3] for x in stats], "mem_mhz": [x[4] for x in stats],
                    "clock_reasons": [[n for i, n in enumerate(CLOCK_REASONS) if int(x[5]) >> i & 1]
                                      for x in stats]}
        # with per-rank problems, every rank decodes rank 0's problem (seed 7)
        # once more: separates each rank's block table / data from its GPU
        if args.rank_seeds:
            prob0 = W.torch_build_cache(shape, seed=7, value_dtype=vdtype)
            r0 = decode_timing(torch, lib, C, shape, prob0, vdtype, K, flush, seed=rank)
            del prob0
            torch.cuda.empty_cache()
            same = gather_per_rank(torch, [r0["kernel_us"]], world)
            per_rank["kernel_us_rank0_problem"] = [round(x[0], 2) for x in same]

    # ---- the sequence split of config 4's long sequence over the same ranks ----
    seq_split = None
    if world > 1 and args.config == "cfg0" and not args.no_split:
        import torch.distributed as dist
        P = importlib.import_module(PKG + ".paged")
        par = importlib.import_module(PKG + ".parallel")
        env = split_setup(torch, P, par, W, "cfg4_long", rank, world)
        seq_split = {"workload": "cfg4_long: one sequence of 131072 tokens x 32 heads x d128 "
                                 f"split across {world} GPUs by 128-token groups (strong scaling)",
                     "algorithmic_bytes": env["shape"].algorithmic_bytes(),
                     "steps": K, "warmup": Wm}
        for mode in ("nccl", "p2p", "fused"):
            seq_split[mode] = split_mode(torch, dist, par, env, mode, rank, world, K, Wm, flush)
        del env
        torch.cuda.empty_cache()

    # ---- the other decode configs and the reference's own launchers (N == 1) ----
    peak, peak_kind = measured_peak()
    sweep = ref_api = None
    if world == 1 and not args.no_sweep:
        sweep = sweep_records(torch, lib, C, W, K, flush, peak)
        ref_api = reference_api_records(torch, lib, flush)

    # ---- CPU baseline: the oracle on a bounded sample (rank 0, N == 1) ----
    bytes_step = shape.algorithmic_bytes()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and hq == h:  # MHA configs
        per_stream = bytes_step / (shape.batch * h)
        sample = [(b, hh) for b in range(shape.batch) for hh in range(h)][::4]
        cpu, outs = cpu_baseline(host, sample, per_stream)
        cpu["max_abs_gpu_vs_oracle_fp32"] = float(max(np.abs(o_host[b, hh] - o).max()
                                                      for (b, hh), o in outs.items()))

    total_bytes = bytes_step * world
    flushed = {"step_us": round(mean_step * 1e3, 2), "kernel_us": round(mean_kern * 1e3, 2),
               "frac": round(bytes_step / (mean_kern * 1e-3) / 1e9 / peak, 4),
               "step_us_percentiles": {k: round(float(np.percentile(step_ms, q)) * 1e3, 2)
                                       for k, q in (("p10", 10), ("p50", 50), ("p90", 90),
                                                    ("max", 100))},
               "timing": "L2 flushed before every launch; step: CUDA events around the C-ABI "
                         "call; kernel: events recorded by the C ABI around the launch",
               "e2e_ms_per_step": round(e2e_flushed_ms, 5)}
    if b2b is not None:  # headline: K steps back to back (inputs > 2 x L2)
        mean_step = mean_kern = b2b["ms"]
        timing = (f"K={K} steps back to back between one pair of CUDA events after a barrier + "
                  f"synchronize, no flush: inputs {bytes_step / 1e6:.1f} MB/GPU > 2 x 126 MB L2 "
                  "(ncu: DRAM bytes per launch = algorithmic bytes in this order, "
                  "profiles/paged_decode_cfg0_back_to_back.md)")
    else:
        timing = ("L2 flushed (256 MiB write + 256 MiB read, untimed) before every timed step; "
                  "CUDA events around each step")
    value = total_bytes / (mean_step * 1e-3) / 1e9
    achieved = bytes_step / (mean_kern * 1e-3) / 1e9
    traffic = profile_traffic() if args.config == "cfg0" else None
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": K, "warmup": Wm, "ms_per_step": round(mean_step, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": f"fp32 (exact integer logits, fp64 recombination), int4 keys, {args.values} values",
        "data": "synthetic (seeded: q~N(0,1); keys N(0,1)*U(0.5,3)+N(0,2) per channel; v~N(0,1))",
        "timing": timing,
        "config": dict(workload_config(shape, args.config, world),
                       problem_per_rank=("own seed per rank: 7 + 1000 * rank" if args.rank_seeds
                                         else "rank 0's seeded problem (seed 7) on every rank")),
        "decode_us": round(mean_step * 1e3, 2),
        "hbm_frac_of_peak": round(value / world / peak, 4),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": f"paged_decode_kernel<{d},4,2> (decode + fused combine)",
                     "kernel_us": round(mean_kern * 1e3, 2),
                     "kernel_us_source": ("the back-to-back step: K launches between one pair "
                                          "of events, the step is one launch" if b2b is not None
                                          else "events recorded by the C ABI around the launch, "
                                          "L2 flushed"),
                     "algorithmic_bytes_per_launch": bytes_step,
                     "traffic_source": ("profiles/paged_decode_cfg0.md: static, from one ncu "
                                        "capture of this kernel at this config (not this run)")
                     if traffic is not None else None,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind ==
                     "measured" else "fallback 6.65 TB/s"},
        "flushed": flushed,
        "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 5), "steps": KE,
                "h2d_bytes_per_step": int(in_bytes),
                "d2h_bytes_per_step": int(out.numel() * 4),
                "path": "ctypes -> int4kv_stage_inputs + int4kv_paged_decode_ex (C ABI); query, "
                        "block table and lengths in one mapped pinned host buffer, pulled into "
                        "HBM by one staging launch (SM loads over PCIe), decode reading them in "
                        "place; the decode stores the output straight into mapped pinned host "
                        "memory (zero-copy, the d2h bytes cross PCIe inside the kernel), read "
                        "on the host after the step; KV pools resident in HBM",
                "max_abs_vs_device_output": e2e_diff},
        "gpu_launches": K,
        "clocks": sampler.summary(),
        "parity": {"gate_streams": len(gate_streams), "max_abs_vs_f64_arbiter": gate_err},
        "quantizer": quant,
    }
    if per_rank is not None:
        result["per_rank"] = per_rank
    if seq_split is not None:
        result["seq_split"] = seq_split
    if sweep is not None:
        result["sweep"] = sweep
    if ref_api is not None:
        result["reference_api"] = ref_api
    if cpu is not None:
        result["cpu_baseline"] = cpu
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# --------------------------------------------------------------------------
# reference arm: the reference's CPU implementation (oracle port), host cores
# --------------------------------------------------------------------------

def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    sys.path.insert(0, ROOT)
    import importlib
    import oracle
    W = importlib.import_module(PKG + ".workloads")
    shape = W.config_shape(args.config)
    h, d = shape.heads, shape.head_dim
    rng = np.random.default_rng(7)
    bt = W.np_block_table(rng, shape.seq_lens, shape.pool_pages)
    k_pool = np.zeros((shape.pool_pages, h, 16, d // 2), np.uint8)
    v_pool = np.zeros((shape.pool_pages, h, 16, d), np.float32)
    sz_pool = np.zeros((shape.pool_pages, h, 2, d), np.float32)
    gp = shape.group_tokens // 16
    for b, n in enumerate(shape.seq_lens):
        keys = W.np_anchor_keys(rng, n, h, d)
        vals = rng.standard_normal((n, h, d)).astype(np.float32)
        q, s, z = oracle.quantize_grouped(keys, shape.group_tokens)
        packed = oracle.pack_int4(q)
        npg = (n + 15) // 16
        for p in range(npg):
            rows = min(16, n - 16 * p)
            k_pool[bt[b, p], :, :rows] = packed[16 * p:16 * p + rows].transpose(1, 0, 2)
            v_pool[bt[b, p], :, :rows] = vals[16 * p:16 * p + rows].transpose(1, 0, 2)
        for g in range(s.shape[0]):
            sz_pool[bt[b, g * gp], :, 0] = s[g]
            sz_pool[bt[b, g * gp], :, 1] = z[g]
    arrays = {"query": rng.standard_normal((shape.batch, h, d)).astype(np.float32),
              "k_pool": k_pool, "v_pool": v_pool, "sz_pool": sz_pool, "block_table": bt,
              "seq_lens": np.asarray(shape.seq_lens, np.int32)}
    from oracle.cpu_pool import OraclePool
    pool = OraclePool(arrays)
    streams = [(b, hh) for b in range(shape.batch) for hh in range(h)]
    per_stream = shape.algorithmic_bytes() / len(streams)
    sample = pool.procs  # one stream per process per step: a bounded sample of the step
    try:
        cursor = 0
        for _ in range(args.warmup):
            pool.run(streams[cursor:cursor + sample])
            cursor = (cursor + sample) % len(streams)
        wall = 0.0
        for _ in range(args.steps):
            chunk = [streams[(cursor + i) % len(streams)] for i in range(sample)]
            cursor = (cursor + sample) % len(streams)
            dt, _ = pool.run(chunk)
            wall += dt
    finally:
        pool.close()
    ms = wall / args.steps * 1e3
    value = sample * per_stream / (ms * 1e-3) / 1e9
    cores = pool.procs
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32 (NumPy)", "data": "synthetic (seeded, same distributions as ours)",
        "config": workload_config(shape, args.config, 1),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                         "host_cpu_count": os.cpu_count(),
                         "host_affinity": len(os.sched_getaffinity(0)),
                         "sample": f"each step = {sample} of the {len(streams)} (sequence, head) "
                                   "streams of one config step, oracle online softmax "
                                   f"(src/flash_decode_ref.py:30-139 restated), {cores} spawn "
                                   "processes x 1 BLAS thread"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


# --------------------------------------------------------------------------
# our arm, sequence split (cfg4_long under torchrun): strong scaling
# --------------------------------------------------------------------------

SPLIT_DESC = {
    "p2p": "partial decode kernel + fused peer-exchange/merge kernel (NVLink stores, "
           "flags, bounded waits; no NCCL)",
    "nccl": "partial decode kernel + NCCL all-gather + merge kernel",
    "fused": "one kernel: decode, push of each stream's record to every rank over "
             "NVLink as its pages finish, bounded wait for the peers' records and "
             "their merge (no NCCL)",
}


def split_setup(torch, P, par, W, name, rank, world):
    """One long sequence (config `name`, e.g. cfg4_long = 1 x 131072 tokens x 32
    heads) drawn identically on every rank; each rank keeps its 128-token-group
    aligned token range in its own cache. Rank 0 also decodes the whole
    sequence on its own GPU: the gate every split mode is checked against."""
    shape = W.config_shape(name)
    L, h, d = shape.seq_lens[0], shape.heads, shape.head_dim
    g = torch.Generator(device="cuda").manual_seed(7)
    sc = torch.rand((h, d), generator=g, device="cuda") * 2.5 + 0.5
    off = torch.randn((h, d), generator=g, device="cuda") * 2.0
    t0, t1 = par.plan_sequence_split(L, world)[rank]
    keys = torch.randn((L, h, d), generator=g, device="cuda") * sc + off
    vals = torch.randn((L, h, d), generator=g, device="cuda")
    query = torch.randn((1, h, d), generator=g, device="cuda")
    cache = P.PagedKVCache((t1 - t0 + 15) // 16 + 8, h, d, device="cuda", seed=rank)
    cache.write_sequences([0], [keys[t0:t1]], [vals[t0:t1]])
    whole_out = None
    if rank == 0:
        whole = P.PagedKVCache((L + 15) // 16 + 8, h, d, device="cuda", seed=99)
        whole.write_sequences([0], [keys], [vals])
        whole_out = whole.decode(query, [0]).clone()
        del whole
    del keys, vals
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return {"shape": shape, "cache": cache, "query": query, "whole_out": whole_out,
            "range": (t0, t1)}


def split_mode(torch, dist, par, env, exchange, rank, world, K, Wm, flush, sampler=None):
    """Time one exchange mode of the sequence split: gate against the whole-
    sequence decode (rank 0), the step captured as one CUDA graph, K replays
    with L2 flushed before each, max over ranks. Every rank takes the same
    collective steps whatever the outcome, so a failed gate is reported, not
    raised half-way."""
    cache, query = env["cache"], env["query"]
    store = dist.distributed_c10d._get_default_store()
    dec = par.SequenceSplitDecoder(
        cache, rank, world, exchange=exchange,
        monitor=par.PeerMonitor(store, rank, world, timeout=60.0, prefix=f"i4kv_split_{exchange}"))
    try:
        out = dec.decode(query).clone()
        gate = torch.zeros((1,), device="cuda", dtype=torch.float64)
        if rank == 0:
            gate[0] = (out - env["whole_out"]).abs().max().double()
        dist.all_reduce(gate, op=dist.ReduceOp.MAX)
        gate_err = float(gate.item())
        st = torch.tensor([float(dec.peer_status())], device="cuda", dtype=torch.float64)
        dist.all_reduce(st, op=dist.ReduceOp.MAX)
        dec.monitor = None  # host liveness checks stay out of the timed loop
        dec.capture(query)
        graph_out = dec.replay()
        torch.cuda.synchronize()
        gerr = float((graph_out - out).abs().max())
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(K)]
        for i in range(Wm):
            flush(i)
            dec.replay()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(K):
            flush(i)
            ev[i][0].record()
            dec.replay()
            ev[i][1].record()
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        dist.barrier()
        if sampler is not None:
            sampler.mark(t0, t1)
        us = [a.elapsed_time(b) * 1e3 for a, b in ev]
        mean = _all_reduce_max(sum(us) / K, world)
        st2 = torch.tensor([float(dec.peer_status())], device="cuda", dtype=torch.float64)
        dist.all_reduce(st2, op=dist.ReduceOp.MAX)
        per_rank = [r[0] for r in gather_per_rank(torch, [sum(us) / K], world)]
    finally:
        dec.close()  # graph (may hold an NCCL call) and peer mappings go before the process group
        torch.cuda.synchronize()
    ok = gate_err <= 2e-6 and gerr == 0.0 and int(st.item()) == 0 and int(st2.item()) == 0
    return {"us_per_step": round(mean, 2), "us_per_step_per_rank": [round(x, 2) for x in per_rank],
            "max_abs_vs_whole_sequence_decode": gate_err, "graph_replay_vs_eager": gerr,
            "peer_status": int(max(st.item(), st2.item())), "gate_ok": ok,
            "launches_per_step": 1 if exchange == "fused" else 2, "step": SPLIT_DESC[exchange]}


def run_split(args):
    """One long sequence split across the ranks by 128-token groups; a step is
    each rank's partial decode + the exchange of the partial records and their
    merge: one fused peer-memory kernel (``--exchange p2p``), one NCCL
    all-gather + the merge kernel (``--exchange nccl``), or no separate step at
    all (``--exchange fused``: the decode kernel pushes, waits and merges
    itself). Total work is fixed as N grows (strong scaling)."""
    import datetime
    import importlib
    import torch
    import torch.distributed as dist
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    importlib.import_module(PKG + "._build").build()
    W = importlib.import_module(PKG + ".workloads")
    P = importlib.import_module(PKG + ".paged")
    par = importlib.import_module(PKG + ".parallel")
    env = split_setup(torch, P, par, W, args.config, rank, world)
    flush = L2Flush(torch)
    sampler = ClockSampler(local)
    sampler.start()
    rec = split_mode(torch, dist, par, env, args.exchange, rank, world, args.steps, args.warmup,
                     flush, sampler)
    sampler.stop()
    if not rec["gate_ok"]:
        raise RuntimeError(f"sequence split failed its gate: {rec}")
    shape = env["shape"]
    L, h, d = shape.seq_lens[0], shape.heads, shape.head_dim
    mean = rec["us_per_step"] * 1e-3
    peak, peak_kind = measured_peak()
    total = shape.algorithmic_bytes()
    value = total / (mean * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(mean, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp32 (exact integer logits, fp64 recombination), int4 keys",
            "data": "synthetic (seeded, config-0 distributions)",
            "config": {"workload": f"{args.config}: one sequence of {L} tokens x {h} heads x d{d}, "
                                   f"split across {world} GPUs by 128-token groups; step = "
                                   + SPLIT_DESC[args.exchange],
                       "exchange": args.exchange,
                       "global_batch": 1, "seq_len": L, "heads": h, "head_dim": d,
                       "l2": "flushed before every timed step",
                       "parallelism": f"sequence split x{world}"},
            "hbm_frac_of_peak": round(value / world / peak, 4), "peak_source": peak_kind,
            "gpu_launches": args.steps * rec["launches_per_step"],
            "step": "CUDA graph: " + SPLIT_DESC[args.exchange],
            "parity": {"max_abs_vs_whole_sequence_decode": rec["max_abs_vs_whole_sequence_decode"]},
            "split": rec,
            "clocks": sampler.summary(),
        }), flush=True)
    torch.cuda.synchronize()
    dist.destroy_process_group()


# --------------------------------------------------------------------------
# our arm, the fused decode step of a 32-layer stack (cfg4_step)
# --------------------------------------------------------------------------

def run_step(args):
    """Config 4 end to end per GPU: 32 attention layers x 32 sequences (the
    256-sequence batch of config 4 sharded over 8 GPUs) x 32 heads x d128 with
    4096-token prompts. A step is one token for every sequence in every layer:
    RoPE + quantize-on-append (one launch) and the paged decode (one launch)
    per layer, 64 launches replayed as one CUDA graph; lengths advance on the
    device. Weak scaling: each rank runs its own stack (no collective)."""
    import importlib
    import torch
    rank, world, local = dist_env()
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    importlib.import_module(PKG + "._build").build()
    S = importlib.import_module(PKG + ".stepper")
    layers, seqs, heads, d, L0 = 32, 32, 32, 128, 4096
    K, Wm = min(args.steps, 200), args.warmup  # each step grows the cache: bound the pools
    KE = max(1, min(args.e2e_steps, K))
    vdtype = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[args.values]
    max_tokens = L0 + Wm + K + KE + 2 + 16
    stack = S.LayerStack(layers, seqs, heads, d, max_tokens, value_dtype=vdtype, seed=7 + rank)
    g = torch.Generator(device="cuda").manual_seed(7 + 1000 * rank)
    keys, vals = [], []
    for _ in range(seqs):  # the anchor distribution, one layer's prompts
        sc = torch.rand((heads, d), generator=g, device="cuda") * 2.5 + 0.5
        off = torch.randn((heads, d), generator=g, device="cuda") * 2.0
        keys.append(torch.randn((L0, heads, d), generator=g, device="cuda") * sc + off)
        vals.append(torch.randn((L0, heads, d), generator=g, device="cuda"))
    stack.prefill(keys, vals, layers=[0])
    del keys, vals
    for l in range(1, layers):
        stack.copy_layer(0, l)
    q = torch.randn((seqs, heads, d), generator=g, device="cuda")
    k = torch.randn((seqs, heads, d), generator=g, device="cuda") * 2.0 + 0.5
    v = torch.randn((seqs, heads, d), generator=g, device="cuda")
    torch.cuda.synchronize()

    # correctness gate: one eager step, layer 0, sampled streams vs the float64 arbiter
    import oracle
    pos = np.array(stack.host_lens)
    out = stack.step(q, k, v)
    torch.cuda.synchronize()
    cos_h, sin_h = stack.rope[0].cpu().numpy(), stack.rope[1].cpu().numpy()
    q_rot = oracle.apply_rope(q.cpu().numpy(), pos, cos_h, sin_h)
    rng = np.random.default_rng(rank)
    gate_streams = [(int(b), int(hh)) for b, hh in zip(rng.integers(0, seqs, 3),
                                                       rng.integers(0, heads, 3))]
    ex = oracle.decode_paged(q_rot, stack.k_pools[0].cpu().numpy(),
                             stack.v_pools[0].float().cpu().numpy(), stack.sz_pools[0].cpu().numpy(),
                             stack.block_table.cpu().numpy(), stack.lens.cpu().numpy(), method="f64",
                             streams=gate_streams)
    o0 = out[0].cpu().numpy()
    gate_err = max(float(np.abs(o0[b, hh] - ex[b, hh]).max()) for b, hh in gate_streams)
    if not (np.isfinite(o0).all() and gate_err <= 1e-6):
        raise RuntimeError(f"decode step failed its correctness gate (max err {gate_err})")

    # ---- the step as one CUDA graph, inputs resident ----
    stack.capture(q, k, v)
    for _ in range(Wm):
        stack.replay()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(K)]
    step_bytes = []
    sampler = ClockSampler(local)
    sampler.start()
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    t_wall0 = time.perf_counter()
    for i in range(K):
        step_bytes.append(stack.step_bytes())
        ev[i][0].record()
        stack.replay()
        ev[i][1].record()
    torch.cuda.synchronize()
    t_wall1 = time.perf_counter()
    _barrier(world)
    torch.cuda.synchronize()
    sampler.mark(t_wall0, t_wall1)
    mean = _all_reduce_max(sum(a.elapsed_time(b) for a, b in ev) / K, world)
    bytes_per_step = sum(step_bytes) / K

    # ---- end to end: inputs from pinned host memory, outputs back, every step ----
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    out_host = torch.empty(stack.out.shape, dtype=torch.float32).pin_memory()
    ee = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(KE)]
    e2e_bytes = []
    torch.cuda.synchronize()
    _barrier(world)
    for i in range(KE):
        e2e_bytes.append(stack.step_bytes())
        ee[i][0].record()
        q.copy_(hq, non_blocking=True)
        k.copy_(hk, non_blocking=True)
        v.copy_(hv, non_blocking=True)
        stack.replay()
        out_host.copy_(stack.out, non_blocking=True)
        ee[i][1].record()
    torch.cuda.synchronize()
    sampler.stop()
    _barrier(world)
    e2e_ms = _all_reduce_max(sum(a.elapsed_time(b) for a, b in ee) / KE, world)
    stack.release()

    peak, peak_kind = measured_peak()
    value = bytes_per_step * world / (mean * 1e-3) / 1e9
    e2e_value = sum(e2e_bytes) / KE * world / (e2e_ms * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
            "steps": K, "warmup": Wm, "ms_per_step": round(mean, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": f"fp32 (exact int logits, fp64 recombination), int4 keys, {args.values} values",
            "data": "synthetic (seeded anchor distribution; one layer's prompts copied to all layers)",
            "config": {"workload": f"cfg4_step: decode step of {layers} attention layers x "
                                   f"{seqs} sequences x {heads} heads x d{d}, {L0}-token prompts "
                                   "growing one token per step; per layer RoPE + quantize-on-append "
                                   "+ paged decode (2 launches), the step one CUDA graph",
                       "layers": layers, "batch_per_gpu": seqs, "global_batch": seqs * world,
                       "heads": heads, "head_dim": d, "seq_len": L0,
                       "l2": f"not flushed: a step moves {bytes_per_step / 1e9:.1f} GB > 126 MB L2",
                       "parallelism": f"dp{world} (sequences sharded, no collective)"},
            "hbm_frac_of_peak": round(value / world / peak, 4), "peak_source": peak_kind,
            "bytes_per_step": int(bytes_per_step),
            "roofline": {"bound": "hbm", "achieved": round(bytes_per_step / (mean * 1e-3) / 1e9, 1),
                         "peak": peak, "unit": "GB/s",
                         "frac": round(bytes_per_step / (mean * 1e-3) / 1e9 / peak, 4),
                         "traffic": None,
                         "kernel": "whole step (64 launches: append_quant_kernel + paged_decode_kernel "
                                   "per layer)"},
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                    "steps": KE,
                    "h2d_bytes_per_step": int((q.numel() + k.numel() + v.numel()) * 4),
                    "d2h_bytes_per_step": int(stack.out.numel() * 4),
                    "path": "q/k/v from pinned host into the graph's input buffers, graph replay, "
                            "all layers' outputs back to pinned host"},
            "gpu_launches": K * layers * 2,
            "clocks": sampler.summary(),
            "parity": {"gate_streams": len(gate_streams), "max_abs_vs_f64_arbiter": gate_err},
        }), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_reference_api(args):
    """The `reference_api` record alone (one GPU): a small, self-contained case."""
    import importlib
    import torch
    importlib.import_module(PKG + "._build").build()
    lib = importlib.import_module(PKG + "._lib").load()
    rec = reference_api_records(torch, lib, L2Flush(torch))
    print(json.dumps({"reference_api": rec}), flush=True)


def main():
    args = parse()
    if args.reference_api_only:
        run_reference_api(args)
        return
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "cfg4_long" and dist_env()[1] > 1:
        run_split(args)
    elif args.config == "cfg4_step":
        run_step(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
