"""Device-resident paged INT4 KV cache (the "prepared cache").

Replaces two host-side structures of the reference: the dense padding of page
lists done on every call (src/ops.py:293-308) and the dict-of-pages cache of
the vLLM shim (src/vllm_integration.py:42-60). Everything lives in HBM:

  k_pool  uint8   [num_pages, kv_heads, 16, head_dim/2]  nibble-packed keys
  v_pool  float32 / float16 / bfloat16 [num_pages, kv_heads, 16, head_dim] values
  sz_pool float32 [num_pages, kv_heads, 2, head_dim]     [scale; zp] of the
          128-token group whose first token lives in this page

Each (page, head) slab of K (1 KiB at d128) and V (8 KiB) is contiguous, so
the decode kernel moves it with one bulk async copy. A sequence owns a list
of physical pages (its block-table row); the group of token ``t`` takes its
scale/zp from page ``row[(t // 128) * 8]``.
"""

from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from . import _C

PAGE_TOKENS = 16


class PagedKVCache:
    def __init__(self, num_pages: int, num_kv_heads: int, head_dim: int,
                 group_tokens: int = 128, device="cuda", seed: Optional[int] = None,
                 values: bool = True, value_dtype=torch.float32, max_open_sequences: int = 64):
        if head_dim % 4:
            raise ValueError(f"head_dim must be a multiple of 4, got {head_dim}")
        if group_tokens % PAGE_TOKENS or group_tokens <= 0 or group_tokens > 128:
            raise ValueError("group_tokens must be a multiple of 16 in [16, 128]")
        self.num_pages = num_pages
        self.heads = num_kv_heads
        self.head_dim = head_dim
        self.group_tokens = group_tokens
        self.device = torch.device(device)
        self.k_pool = torch.zeros((num_pages, num_kv_heads, PAGE_TOKENS, head_dim // 2),
                                  dtype=torch.uint8, device=self.device)
        if value_dtype not in _C.VALUE_KINDS:
            raise ValueError(f"value_dtype must be one of {list(_C.VALUE_KINDS)}")
        self.value_dtype = value_dtype
        self.v_pool = (torch.zeros((num_pages, num_kv_heads, PAGE_TOKENS, head_dim),
                                   dtype=value_dtype, device=self.device) if values else None)
        self.sz_pool = torch.zeros((num_pages, num_kv_heads, 2, head_dim), dtype=torch.float32,
                                   device=self.device)
        order = (np.random.default_rng(seed).permutation(num_pages) if seed is not None
                 else np.arange(num_pages))
        self._free: List[int] = [int(p) for p in order[::-1]]
        self.pages: Dict[int, List[int]] = {}
        self.lens: Dict[int, int] = {}
        # float32 keys of each sequence's open (partial) group, for appends:
        # slot [group_tokens, heads * head_dim], allocated on first need
        self.max_open = max_open_sequences
        self.k_stage: Optional[torch.Tensor] = None
        self._stage_slot: Dict[int, int] = {}
        self._stage_free: List[int] = list(range(max_open_sequences - 1, -1, -1))

    # ---- page allocation ----
    def _alloc(self, n: int) -> List[int]:
        if n > len(self._free):
            raise MemoryError(f"paged KV cache out of pages: need {n}, {len(self._free)} free")
        return [self._free.pop() for _ in range(n)]

    def free_sequence(self, seq_id: int) -> None:
        for p in self.pages.pop(seq_id, []):
            self._free.append(p)
        self.lens.pop(seq_id, None)
        slot = self._stage_slot.pop(seq_id, None)
        if slot is not None:
            self._stage_free.append(slot)

    def _slot_of(self, seq_id: int) -> int:
        if seq_id not in self._stage_slot:
            if not self._stage_free:  # grow the staging pool (twice the slots)
                old, n = self.k_stage, self.max_open
                self.max_open = 2 * n
                self.k_stage = torch.zeros((self.max_open,) + tuple(old.shape[1:]),
                                           dtype=torch.float32, device=self.device)
                self.k_stage[:n] = old
                self._stage_free = list(range(self.max_open - 1, n - 1, -1))
            if self.k_stage is None:
                self.k_stage = torch.zeros((self.max_open, self.group_tokens,
                                            self.heads * self.head_dim), dtype=torch.float32,
                                           device=self.device)
            self._stage_slot[seq_id] = self._stage_free.pop()
        return self._stage_slot[seq_id]

    # ---- writes ----
    def write_sequences(self, seq_ids: Sequence[int], keys: Sequence[torch.Tensor],
                        values: Optional[Sequence[torch.Tensor]] = None, rope=None) -> None:
        """Quantize and store whole sequences ([len, heads, head_dim] float32 each).

        One kernel launch quantizes every 128-token group of every sequence and
        scatters keys and values into freshly allocated pages. With
        ``rope = (cos, sin)`` the keys are first rotated at positions 0..len-1
        on the GPU (``int4kv_rope``): the cache holds post-RoPE keys.
        """
        if len(seq_ids) != len(keys):
            raise ValueError("one key tensor per sequence")
        lens = [int(k.shape[0]) for k in keys]
        for s, n in zip(seq_ids, lens):
            if s in self.pages:
                self.free_sequence(s)
            self.pages[s] = self._alloc((n + PAGE_TOKENS - 1) // PAGE_TOKENS)
            self.lens[s] = n
        if sum(lens) == 0:
            return
        k = torch.cat([t.to(self.device, torch.float32) for t in keys]).contiguous()
        if rope is not None:
            pos = torch.from_numpy(np.concatenate([np.arange(n, dtype=np.int32) for n in lens]))
            k = _C.rope(k, pos.to(self.device), rope[0], rope[1])
        v = None
        if values is not None and self.v_pool is not None:
            v = torch.cat([t.to(self.device, torch.float32) for t in values]).contiguous()
        offs = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32,
                            device=self.device)
        bt, _ = self.block_table(seq_ids)
        _C.cache_write(k, v, offs, bt, self.k_pool, self.v_pool, self.sz_pool,
                       max_rows_per_seq=max(lens), group_tokens=self.group_tokens)
        # keep the float32 keys of each open last group, so appends can requantize it
        for s, n, o in zip(seq_ids, lens, offs[:-1].tolist()):
            open_rows = n % self.group_tokens
            if open_rows:
                slot = self._slot_of(s)
                self.k_stage[slot, :open_rows] = k[o + n - open_rows:o + n].reshape(open_rows, -1)

    def append(self, seq_ids: Sequence[int], keys: torch.Tensor,
               values: Optional[torch.Tensor] = None, rope=None,
               query: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        """Append one token to each sequence: keys / values [B, heads, head_dim].

        One kernel launch: each sequence's open 128-token group is quantized
        again over its valid rows (the new token included), so the cache equals
        a bulk write of the same tokens after every step. Sequences may be new
        (length 0); a new page is taken whenever a sequence crosses a 16-token
        boundary. With ``rope = (cos, sin)`` the new keys are rotated at their
        positions first, and ``query`` [B, q_heads, head_dim] (optional) is
        rotated at the same positions in the same launch and returned.
        """
        ids = list(seq_ids)
        if len(set(ids)) != len(ids):
            raise ValueError("a sequence may append only one token per call")
        k = keys.to(self.device, torch.float32).contiguous()
        if k.dim() != 3 or tuple(k.shape) != (len(ids), self.heads, self.head_dim):
            raise ValueError(f"keys must be [{len(ids)}, {self.heads}, {self.head_dim}]")
        v = None
        if values is not None and self.v_pool is not None:
            v = values.to(self.device, torch.float32).contiguous()
            if v.shape != k.shape:
                raise ValueError("values must have the shape of keys")
        pos = []
        for s in ids:
            n = self.lens.setdefault(s, 0)
            self.pages.setdefault(s, [])
            if n % PAGE_TOKENS == 0:
                self.pages[s].extend(self._alloc(1))
            pos.append(n)
        slots = [self._slot_of(s) for s in ids]
        bt, _ = self.block_table(ids)
        positions = torch.tensor(pos, dtype=torch.int32, device=self.device)
        slot_t = torch.tensor(slots, dtype=torch.int32, device=self.device)
        q = None
        if query is not None:
            q = query.to(self.device, torch.float32).contiguous()
        q_rot = _C.cache_append(k, v, positions, slot_t, self.k_stage, bt, self.k_pool,
                                self.v_pool, self.sz_pool, group_tokens=self.group_tokens,
                                rope=rope, q=q)
        for s in ids:
            self.lens[s] += 1
        return q_rot

    def decode_step(self, seq_ids: Sequence[int], query: torch.Tensor, keys: torch.Tensor,
                    values: torch.Tensor, rope) -> torch.Tensor:
        """One decode step of a Llama-style attention layer: RoPE of the step's
        query and key at each sequence's position, quantize-on-append of the
        rotated key and the value, then the paged decode of the rotated query
        over the cache (the new token included). Two launches."""
        q_rot = self.append(seq_ids, keys, values, rope=rope, query=query)
        return self.decode(q_rot, seq_ids)

    # ---- reads ----
    def block_table(self, seq_ids: Sequence[int]):
        """(block_table int32 [B, max_pages], seq_lens int32 [B]) on the cache's device."""
        maxp = max([1] + [len(self.pages[s]) for s in seq_ids])
        bt = np.zeros((len(seq_ids), maxp), np.int32)
        for i, s in enumerate(seq_ids):
            bt[i, :len(self.pages[s])] = self.pages[s]
        lens = np.array([self.lens[s] for s in seq_ids], np.int32)
        return (torch.from_numpy(bt).to(self.device), torch.from_numpy(lens).to(self.device))

    def decode(self, query: torch.Tensor, seq_ids: Sequence[int]) -> torch.Tensor:
        """query [B, heads, head_dim] -> attention output [B, heads, head_dim] (device)."""
        bt, sl = self.block_table(seq_ids)
        return _C.paged_decode(query.to(self.device, torch.float32).contiguous(), self.k_pool,
                               self.v_pool, self.sz_pool, bt, sl, self.group_tokens)

    def memory_stats(self) -> dict:
        used = sum(len(p) for p in self.pages.values())
        per_page = (self.k_pool[0].numel() + self.sz_pool[0].numel() * 4
                    + (self.v_pool[0].numel() * 4 if self.v_pool is not None else 0))
        return {"pages_used": used, "pages_total": self.num_pages,
                "bytes_used": used * per_page, "tokens": sum(self.lens.values())}
