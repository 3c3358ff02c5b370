"""Multi-GPU decode: batch x head sharding and the single-sequence split.

One process per GPU (``torch.distributed``, NCCL over NVLink / NVSwitch).
Two layouts, both of which keep every KV page on the GPU that owns it:

* **Batch x head sharding** (``plan_batch_heads``): the (sequence, kv-head)
  streams of a decode batch are partitioned across ranks -- whole sequences
  when there are at least as many sequences as ranks, head slices of each
  sequence otherwise -- balanced by the bytes each rank must stream. Each rank
  runs the one-GPU kernel on its own pages; there is no collective on the
  data path. Aggregate throughput = sum of bytes / slowest rank.
* **Sequence split** (``plan_sequence_split``, ``SequenceSplitDecoder``): one
  long sequence is cut into 128-token-group-aligned token ranges, one per
  rank, so that no quantization group straddles two GPUs. Each rank decodes
  its range into per-head partial records ``(m, l, acc)``
  (``int4kv_paged_decode_partials``); ONE all-gather over NCCL lands every
  rank's records in every rank's memory; ``int4kv_merge_partials`` combines
  them (the log-sum-exp merge of the reference's kernel,
  csrc/flash_decode_int4.cu:199-220, across GPUs instead of warps). With
  ``exchange="p2p"`` the gather and the merge are one kernel instead
  (``PeerExchange``): each rank stores its records straight into every
  rank's buffer over NVLink (CUDA IPC mappings), raises a flag per chunk of
  streams, waits (bounded) for the peers' flags and merges. With
  ``exchange="fused"`` the whole step is ONE kernel
  (``int4kv_paged_decode_split``): the decode itself pushes each stream's
  GPU-local result to every rank as soon as it is final and merges the
  ranks' records at the end, so the exchange overlaps the decode.

Failure detection stays on the host: ``PeerMonitor`` has every rank post a
heartbeat key to the process group's store before each collective step and
wait, with a short timeout, for the other ranks' keys -- a rank that died or
never joined is reported as ``PeerFailure`` before anyone launches the
collective, and the process group's own timeout bounds the collective itself.

No counterpart in the reference, which is single-GPU.
"""

import datetime
import heapq
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

from . import _C

PAGE_TOKENS = 16


def partial_record_bytes(head_dim: int) -> int:
    """Bytes of one (m f64, l f64, acc f32[head_dim]) partial record."""
    return 16 + 4 * head_dim


def stream_bytes(seq_len: int, head_dim: int, group_tokens: int = 128) -> int:
    """Algorithmic HBM bytes of one (sequence, head) stream of length seq_len."""
    groups = (seq_len + group_tokens - 1) // group_tokens
    return seq_len * head_dim // 2 + 4 * seq_len * head_dim + 8 * head_dim * groups + 8 * head_dim


# --------------------------------------------------------------------------
# batch x head sharding (no collective)
# --------------------------------------------------------------------------

@dataclass(frozen=True)
class Shard:
    """Work of one rank: ``units`` of (sequence, first kv head), each covering
    kv heads [h0, h0 + width). The rank decodes them as one local batch of
    ``len(units)`` sequences with ``width`` heads each."""
    rank: int
    units: Tuple[Tuple[int, int], ...]
    width: int
    bytes: int

    @property
    def seqs(self) -> Tuple[int, ...]:
        return tuple(b for b, _ in self.units)


def plan_batch_heads(seq_lens: Sequence[int], heads: int, world: int, head_dim: int = 128,
                     group_tokens: int = 128) -> List[Shard]:
    """Partition a decode batch's (sequence, kv-head) streams over `world` ranks.

    With ``len(seq_lens) >= world`` the units are whole sequences (a rank's
    block table stays local). With fewer sequences than ranks each sequence is
    cut into k equal head slices, k the smallest divisor of ``heads`` with
    ``k * len(seq_lens) >= world``. Units are assigned longest-first to the
    least-loaded rank (bytes to stream). Every (sequence, head) stream lands on
    exactly one rank; a rank is empty only when there are fewer units than
    ranks.
    """
    if world <= 0 or heads <= 0:
        raise ValueError("world and heads must be positive")
    lens = [int(n) for n in seq_lens]
    if any(n < 0 for n in lens):
        raise ValueError("sequence lengths must be >= 0")
    nb = len(lens)
    k = 1
    if 0 < nb < world:
        k = next((d for d in range(1, heads + 1) if heads % d == 0 and d * nb >= world), heads)
    width = heads // k
    units = [(b, i * width) for b in range(nb) for i in range(k)]
    cost = [width * stream_bytes(lens[b], head_dim, group_tokens) for b, _ in units]
    order = sorted(range(len(units)), key=lambda u: (-cost[u], u))
    heap = [(0, r) for r in range(world)]
    owned = {r: [] for r in range(world)}
    for u in order:
        load, r = heapq.heappop(heap)
        owned[r].append(u)
        heapq.heappush(heap, (load + cost[u], r))
    return [Shard(r, tuple(units[u] for u in sorted(owned[r])), width,
                  sum(cost[u] for u in owned[r])) for r in range(world)]


# --------------------------------------------------------------------------
# sequence split (one NCCL all-gather of partial records)
# --------------------------------------------------------------------------

def plan_sequence_split(seq_len: int, world: int, group_tokens: int = 128) -> List[Tuple[int, int]]:
    """Token ranges [t0, t1) per rank, boundaries on quantization-group edges.

    Groups are dealt out as evenly as possible (the first ``G % world`` ranks
    take one more group); the last range ends at ``seq_len`` (its final group
    may be partial). Ranks beyond the number of groups get empty ranges.
    """
    if world <= 0 or seq_len < 0 or group_tokens <= 0 or group_tokens % PAGE_TOKENS:
        raise ValueError("bad split arguments")
    groups = -(-seq_len // group_tokens)
    base, extra = divmod(groups, world)
    ranges, g = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        t0 = min(seq_len, g * group_tokens)
        t1 = min(seq_len, (g + n) * group_tokens)
        ranges.append((t0, t1))
        g += n
    return ranges


class PeerFailure(RuntimeError):
    """A rank did not reach a collective step in time (died, hung or never joined)."""


class PeerMonitor:
    """Host-side liveness check before each collective step.

    Every rank sets ``<prefix>/<step>/<rank>`` in the process group's store,
    then waits up to ``timeout`` seconds for all ranks' keys of the same step.
    A missing key raises ``PeerFailure`` naming the absent ranks, so a dead
    rank is detected on the host before any collective is launched.
    """

    def __init__(self, store, rank: int, world: int, timeout: float = 5.0, prefix: str = "i4kv"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout = timeout
        self.prefix = prefix
        self.step = 0

    def check(self) -> None:
        step = self.step
        self.step += 1
        key = f"{self.prefix}/{step}/"
        self.store.set(key + str(self.rank), "1")
        keys = [key + str(r) for r in range(self.world)]
        try:
            self.store.wait(keys, datetime.timedelta(seconds=self.timeout))
        except Exception as e:  # the store raises on timeout; find who is missing
            missing = []
            for r in range(self.world):
                try:
                    if not self.store.check([key + str(r)]):
                        missing.append(r)
                except Exception:
                    missing.append(r)
            raise PeerFailure(f"ranks {missing or '?'} did not reach step {step} within "
                              f"{self.timeout:.1f} s") from e


def exchange_partials(local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather a rank's partial records (uint8 [n]) into [world, n] on every rank.

    The one collective of the sequence split: ``all_gather_into_tensor`` over
    the process group (NCCL on GPUs, gloo on CPU ranks).
    """
    import torch.distributed as dist
    if local.dtype != torch.uint8 or local.dim() != 1:
        raise ValueError("partials must be a flat uint8 tensor")
    out = torch.empty((world * local.numel(),), dtype=torch.uint8, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out.view(world, local.numel())


# --------------------------------------------------------------------------
# fused peer exchange (push + flag + merge in one kernel, no NCCL)
# --------------------------------------------------------------------------

EXCHANGE_MAX_RANKS = 8
EXCHANGE_CHUNK = 8  # streams per CTA of the exchange kernel


def _align128(x: int) -> int:
    return (x + 127) // 128 * 128


def exchange_layout(streams: int, head_dim: int) -> dict:
    """Byte offsets of one rank's exchange buffer (csrc/exchange.cu):
    ``step u32[chunks]``, ``flag u32[2][8][chunks]``, ``recs [2][8][streams]``
    partial records. Used by tests that stand in for a peer on the host."""
    chunks = -(-streams // EXCHANGE_CHUNK)
    off_flag = _align128(chunks * 4)
    off_recs = off_flag + _align128(2 * EXCHANGE_MAX_RANKS * chunks * 4)
    rec = partial_record_bytes(head_dim)
    return {"chunks": chunks, "off_flag": off_flag, "off_recs": off_recs, "record": rec,
            "bytes": off_recs + 2 * EXCHANGE_MAX_RANKS * streams * rec}


def split_layout(streams: int, head_dim: int) -> dict:
    """Byte offsets of one rank's buffer for the fused split decode
    (``int4kv_paged_decode_split``): ``step u32[S]``, ``flag u32[2][8][S]``,
    ``recs [2][8][S]`` records, per query stream. Used by tests that stand in
    for a peer on the host."""
    off_flag = _align128(streams * 4)
    off_recs = off_flag + _align128(2 * EXCHANGE_MAX_RANKS * streams * 4)
    rec = partial_record_bytes(head_dim)
    return {"off_flag": off_flag, "off_recs": off_recs, "record": rec,
            "bytes": off_recs + 2 * EXCHANGE_MAX_RANKS * streams * rec}


class _DeviceBytes:
    """``__cuda_array_interface__`` of a raw device allocation (uint8)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (int(ptr), False), "version": 3}


def device_bytes(ptr: int, nbytes: int, device) -> torch.Tensor:
    """A uint8 tensor viewing ``nbytes`` at device address ``ptr`` (no copy)."""
    return torch.as_tensor(_DeviceBytes(ptr, nbytes), device=device)


class PeerExchange:
    """Every rank's exchange buffer, mapped on this rank's GPU over CUDA IPC.

    Each rank allocates one zero-filled buffer (``int4kv_exchange_alloc``),
    all-gathers its IPC handle over the process group (a host object
    exchange, once), and maps the other ranks' buffers (``int4kv_ipc_open``;
    NVLink peer access). ``merge(partials, out)`` then runs the fused
    exchange kernel: one launch per step, no collective library call.
    ``close()`` must be called on every rank (it synchronizes and barriers
    before unmapping, so no peer is still writing).
    """

    def __init__(self, rank: int, world: int, streams: int, head_dim: int, device, group=None,
                 nbytes: Optional[int] = None):
        import torch.distributed as dist
        if not 1 <= world <= EXCHANGE_MAX_RANKS:
            raise ValueError(f"the peer exchange supports 1..{EXCHANGE_MAX_RANKS} ranks")
        self.rank, self.world, self.group = rank, world, group
        self.streams, self.head_dim = streams, head_dim
        self.device = torch.device(device)
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        # the buffer of the separate exchange kernel, or `nbytes` for another layout
        self.nbytes = nbytes if nbytes is not None else _C.exchange_bytes(world, streams, head_dim)
        self.own = _C.exchange_alloc(idx, self.nbytes)
        self._opened = []
        handles = [None] * world
        if world > 1:
            dist.all_gather_object(handles, _C.ipc_handle(self.own), group=group)
        self.ptrs = []
        with torch.cuda.device(self.device):
            for r in range(world):
                if r == rank:
                    self.ptrs.append(self.own)
                else:
                    ptr = _C.ipc_open(handles[r])
                    self._opened.append(ptr)
                    self.ptrs.append(ptr)
        if world > 1:
            dist.barrier(group=group)  # every buffer is mapped before the first push
        self.status = torch.zeros((1,), dtype=torch.int32, device=self.device)

    def merge(self, partials: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        if self.ptrs is None:
            raise RuntimeError("exchange closed")
        return _C.exchange_merge(partials, self.ptrs, self.rank, self.streams, self.head_dim, out,
                                 self.status)

    def close(self) -> None:
        import torch.distributed as dist
        if self.ptrs is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)  # no peer kernel is still pushing into our buffer
        for ptr in self._opened:
            _C.ipc_close(ptr)
        _C.exchange_free(self.own)
        self.ptrs, self._opened = None, []


class SequenceSplitDecoder:
    """Decode of one long sequence whose token range is split across ranks.

    ``cache`` holds this rank's token range ``ranges[rank]`` of the sequence
    (written from position 0 of the range: ranges start on group edges, so the
    groups -- and therefore the codes and scales -- are those of the whole
    sequence). ``decode(query)`` returns the full attention output on every
    rank.
    """

    def __init__(self, cache, rank: int, world: int, group=None, monitor: Optional[PeerMonitor] = None,
                 exchange: str = "nccl"):
        if exchange not in ("nccl", "p2p", "fused"):
            raise ValueError("exchange must be 'nccl', 'p2p' or 'fused'")
        self.cache, self.rank, self.world, self.group = cache, rank, world, group
        self.monitor = monitor
        d, h = cache.head_dim, cache.heads
        dev = cache.device
        self.rec = partial_record_bytes(d)
        self.partials = torch.empty((h * self.rec,), dtype=torch.uint8, device=dev)
        self.workspace = torch.zeros((_C.paged_decode_workspace_bytes(
            1, h, h, d, dev, value_dtype=cache.value_dtype),), dtype=torch.uint8, device=dev)
        self._tables = {}
        self.exchange = exchange
        self.peers = None
        if exchange == "p2p":
            self.peers = PeerExchange(rank, world, h, d, dev, group)
            self.out = torch.empty((h, d), dtype=torch.float32, device=dev)
        elif exchange == "fused":  # one launch: decode + exchange + merge
            self.peers = PeerExchange(rank, world, h, d, dev, group,
                                      nbytes=_C.paged_decode_split_bytes(1, h, d))
            self.out = torch.empty((1, h, d), dtype=torch.float32, device=dev)

    def refresh(self) -> None:
        """Forget cached block tables (call after the cache's pages change)."""
        self._tables.clear()

    def local_partials(self, query: torch.Tensor, seq_id: int = 0) -> torch.Tensor:
        if seq_id not in self._tables:
            self._tables[seq_id] = self.cache.block_table([seq_id])
        bt, sl = self._tables[seq_id]
        _C.paged_decode_partials(query, self.cache.k_pool, self.cache.v_pool, self.cache.sz_pool,
                                 bt, sl, self.cache.group_tokens, out=self.partials,
                                 workspace=self.workspace)
        return self.partials

    def _step(self, query: torch.Tensor, seq_id: int) -> torch.Tensor:
        if self.exchange == "fused":
            if seq_id not in self._tables:
                self._tables[seq_id] = self.cache.block_table([seq_id])
            bt, sl = self._tables[seq_id]
            return _C.paged_decode_split(query, self.cache.k_pool, self.cache.v_pool,
                                         self.cache.sz_pool, bt, sl, self.peers.ptrs, self.rank,
                                         self.cache.group_tokens, out=self.out,
                                         workspace=self.workspace, status=self.peers.status)
        parts = self.local_partials(query, seq_id)
        if self.peers is not None:
            return self.peers.merge(parts, self.out).view(1, self.cache.heads, self.cache.head_dim)
        gathered = exchange_partials(parts, self.world, self.group)
        return _C.merge_partials(gathered, self.cache.heads, self.cache.head_dim).view(
            1, self.cache.heads, self.cache.head_dim)

    def decode(self, query: torch.Tensor, seq_id: int = 0) -> torch.Tensor:
        """query [1, H, D] float32 on this rank's GPU -> [1, H, D] on every rank."""
        if self.monitor is not None:
            self.monitor.check()
        return self._step(query, seq_id)

    # ---- CUDA graph of the whole step ----
    graph = None

    def capture(self, query: torch.Tensor, seq_id: int = 0, warmup: int = 2) -> torch.Tensor:
        """Record one step as a CUDA graph (partial decode -> all-gather -> merge
        with NCCL; partial decode -> exchange kernel with p2p; the one split
        decode kernel with fused).

        ``query`` becomes the graph's input buffer: copy each new query into it
        and call ``replay()``, which returns the (static) output tensor. Every
        rank must capture, and release the graph (``release()``) before the
        process group is destroyed.
        """
        side = torch.cuda.Stream(device=query.device)
        side.wait_stream(torch.cuda.current_stream(query.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._step(query, seq_id)
        torch.cuda.current_stream(query.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.graph_out = self._step(query, seq_id)
        return self.graph_out

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            raise RuntimeError("capture() first")
        if self.monitor is not None:
            self.monitor.check()
        self.graph.replay()
        return self.graph_out

    def peer_status(self) -> int:
        """INT4KV_STATUS_* bits the peer exchange raised (PEER_TIMEOUT = 8); 0 for NCCL."""
        return int(self.peers.status.item()) if self.peers is not None else 0

    def release(self) -> None:
        self.graph = None
        self.graph_out = None

    def close(self) -> None:
        """Release the graph and unmap the peer buffers (every rank, before
        ``destroy_process_group``)."""
        self.release()
        if self.peers is not None:
            self.peers.close()
            self.peers = None
