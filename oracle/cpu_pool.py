"""Parallel CPU timing of the attention oracle (test / baseline infrastructure only).

Used by ``bench.py`` for the CPU baseline and the reference arm: the paged
pools are saved as ``.npy`` files once, worker processes (started with the
``spawn`` method, each with single-threaded BLAS) memory-map them, and each
worker runs the oracle's per-stream online softmax
(``oracle.attention.decode_paged``, restating src/flash_decode_ref.py:30-139)
on its share of the streams.
"""

import multiprocessing as mp
import os
import tempfile
import time

import numpy as np

_ARR = {}


def _init(paths):
    for name, path in paths.items():
        _ARR[name] = np.load(path, mmap_mode="r")


def _work(streams):
    from .attention import decode_paged
    a = _ARR
    t0 = time.perf_counter()
    out = decode_paged(a["query"], a["k_pool"], a["v_pool"], a["sz_pool"], a["block_table"],
                       a["seq_lens"], streams=streams)
    dt = time.perf_counter() - t0
    return dt, [(b, h, out[b, h].copy()) for b, h in streams]


class OraclePool:
    """A pool of `procs` spawn workers holding one paged problem."""

    def __init__(self, arrays, procs=None, tmpdir=None):
        self.procs = procs or len(os.sched_getaffinity(0))
        base = tmpdir or ("/dev/shm" if os.path.isdir("/dev/shm") else None)
        self._dir = tempfile.TemporaryDirectory(prefix="i4kv_oracle_", dir=base)
        paths = {}
        for name, arr in arrays.items():
            p = os.path.join(self._dir.name, name + ".npy")
            np.save(p, np.ascontiguousarray(arr))
            paths[name] = p
        env_keep = {k: os.environ.get(k) for k in ("OPENBLAS_NUM_THREADS", "OMP_NUM_THREADS",
                                                   "MKL_NUM_THREADS")}
        for k in env_keep:
            os.environ[k] = "1"  # one core per worker; inherited at spawn
        try:
            self._pool = mp.get_context("spawn").Pool(self.procs, initializer=_init,
                                                      initargs=(paths,))
            self._pool.map(_work, [[] for _ in range(self.procs)])  # warm: imports + mmaps
        finally:
            for k, v in env_keep.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v

    def run(self, streams):
        """Run the oracle over `streams` [(b, h)...]; returns (wall seconds, {(b,h): out})."""
        chunks = [streams[i::self.procs] for i in range(self.procs)]
        chunks = [c for c in chunks if c]
        t0 = time.perf_counter()
        res = self._pool.map(_work, chunks)
        wall = time.perf_counter() - t0
        outs = {}
        for _, lst in res:
            for b, h, o in lst:
                outs[(b, h)] = o
        return wall, outs

    def close(self):
        self._pool.close()
        self._pool.join()
        self._dir.cleanup()
