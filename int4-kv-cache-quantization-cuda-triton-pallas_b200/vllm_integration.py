"""vLLM-style paged INT4 KV cache: the reference's ``INT4PagedKVCache`` API,
device-resident.

Same constructor, methods and return types as the reference shim
(src/vllm_integration.py:29-102): ``write_block(block_id, k, v)`` quantizes
the block's keys per channel (one group = the block's rows) and stores them
nibble-packed, values as FP16; ``decode_attention(query, block_table)`` runs
fused INT4 attention of every query over the listed blocks; ``free_block``;
``memory_stats``.

What changed: the reference keeps NumPy arrays in dicts and, on every decode,
unpacks every page and up-casts every value on the host before copying
everything to the GPU (src/vllm_integration.py:62-78). Here the blocks live in
HBM slabs indexed by block id; writes quantize on the GPU; decode reads the
listed blocks where they are stored (packed codes, float16 values) with the shared-stream
kernel; ``append_token`` adds one token to a block on the GPU.
Block ids must lie in ``[0, num_blocks)``.
"""

from collections.abc import Mapping

import numpy as np
import torch

from . import _C
from . import ops


class _BlockView(Mapping):
    """Read-only mapping block_id -> device tensor slab, over present blocks."""

    def __init__(self, cache, store, per_block_rows):
        self._c = cache
        self._s = store
        self._rows = per_block_rows

    def __getitem__(self, b):
        if not self._c._present[b]:
            raise KeyError(b)
        return self._s[b, : self._c._lens[b]] if self._rows else self._s[b]

    def __iter__(self):
        return iter(int(i) for i in np.flatnonzero(self._c._present))

    def __len__(self):
        return int(self._c._present.sum())


class INT4PagedKVCache:
    """Paged KV cache with nibble-packed INT4 keys and FP16 values, in HBM."""

    def __init__(self, num_blocks: int, block_size: int, head_dim: int, device="cuda"):
        ops._require_cuda(None)
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.head_dim = head_dim
        self.device = torch.device(device)
        half = (head_dim + 1) // 2
        self._k = torch.zeros((num_blocks, block_size, half), dtype=torch.uint8, device=self.device)
        self._s = torch.zeros((num_blocks, head_dim), dtype=torch.float32, device=self.device)
        self._z = torch.zeros((num_blocks, head_dim), dtype=torch.float32, device=self.device)
        self._v = torch.zeros((num_blocks, block_size, head_dim), dtype=torch.float16,
                              device=self.device)
        self._lens = np.zeros(num_blocks, np.int64)
        self._lens_dev = torch.zeros(num_blocks, dtype=torch.int32, device=self.device)
        self._present = np.zeros(num_blocks, bool)
        self._stage = {}  # block id -> float32 keys of a block still being filled
        self.k_packed = _BlockView(self, self._k, True)
        self.k_scale = _BlockView(self, self._s, False)
        self.k_zp = _BlockView(self, self._z, False)
        self.v = _BlockView(self, self._v, True)

    def _slot(self, block_id):
        b = int(block_id)
        if not 0 <= b < self.num_blocks:
            raise IndexError(f"block_id {block_id} outside [0, {self.num_blocks})")
        return b

    def write_block(self, block_id: int, k_block, v_block) -> None:
        """Quantize (one group = the block's rows), pack and store one block."""
        b = self._slot(block_id)
        k = torch.as_tensor(np.asarray(k_block, np.float32) if not isinstance(k_block, torch.Tensor)
                            else k_block).to(self.device, torch.float32).contiguous()
        v = torch.as_tensor(np.asarray(v_block) if not isinstance(v_block, torch.Tensor)
                            else v_block).to(self.device)
        if tuple(k.shape) != tuple(v.shape):
            raise ValueError(f"key block {tuple(k.shape)} and value block {tuple(v.shape)} differ")
        rows, d = k.shape
        if d != self.head_dim or not 0 < rows <= self.block_size:
            raise ValueError(f"block must be [1..{self.block_size}, {self.head_dim}], got {tuple(k.shape)}")
        self._quantize_rows(b, k)
        self._v[b, :rows] = v.to(torch.float16)
        self._lens[b] = rows
        self._lens_dev[b] = rows
        self._present[b] = True
        self._stage.pop(b, None)

    def _quantize_rows(self, b: int, k: torch.Tensor) -> None:
        """Quantize rows k [rows, head_dim] as one group into block b."""
        rows, d = k.shape
        if d % 4 == 0:
            packed, scale, zp = _C.quantize_int4_grouped(k.contiguous().view(rows, 1, d),
                                                         group_tokens=rows)
            self._k[b, :rows] = packed.view(rows, d // 2)
            self._s[b] = scale.view(d)
            self._z[b] = zp.view(d)
        else:
            q, scale, zp = _C.quantize_int4(k.contiguous())
            if d % 2:
                q = torch.cat([q, torch.zeros((rows, 1), dtype=torch.uint8, device=self.device)], 1)
            self._k[b, :rows] = q[:, 0::2] | (q[:, 1::2] << 4)
            self._s[b] = scale
            self._z[b] = zp

    def free_block(self, block_id: int) -> None:
        b = self._slot(block_id)
        self._present[b] = False
        self._lens[b] = 0
        self._lens_dev[b] = 0
        self._stage.pop(b, None)

    def append_token(self, block_id: int, k_row, v_row) -> None:
        """Add one token to a block (the vLLM decode-step write): the block's keys
        are quantized again over all its rows so far (one group = the block), so
        a block filled token by token equals one written with write_block."""
        b = self._slot(block_id)
        rows = int(self._lens[b]) if self._present[b] else 0
        if rows >= self.block_size:
            raise ValueError(f"block {block_id} is full ({self.block_size} rows)")
        k = torch.as_tensor(np.asarray(k_row, np.float32) if not isinstance(k_row, torch.Tensor)
                            else k_row).to(self.device, torch.float32).reshape(self.head_dim)
        v = torch.as_tensor(np.asarray(v_row) if not isinstance(v_row, torch.Tensor)
                            else v_row).to(self.device).reshape(self.head_dim)
        if b not in self._stage:
            self._stage[b] = torch.zeros((self.block_size, self.head_dim), dtype=torch.float32,
                                         device=self.device)
        stage = self._stage[b]
        stage[rows] = k
        self._v[b, rows] = v.to(torch.float16)
        self._quantize_rows(b, stage[:rows + 1])
        self._lens[b] = rows + 1
        self._lens_dev[b] = rows + 1
        self._present[b] = True
        if rows + 1 == self.block_size:
            del self._stage[b]  # block complete: its codes are final

    def decode_attention(self, query, block_table) -> np.ndarray:
        """Fused INT4 attention of query [batch, heads, head_dim] over the listed blocks.

        The kernel reads the listed blocks where they are stored -- packed codes,
        float16 values, per-block scale / zero-point -- with no unpack, cast or
        gather copy (the reference unpacks and up-casts every block on the host
        on every call, src/vllm_integration.py:72-78)."""
        ids = [self._slot(b) for b in block_table]
        for b in ids:
            if not self._present[b]:
                raise KeyError(b)
        q = torch.as_tensor(np.asarray(query, np.float32) if not isinstance(query, torch.Tensor)
                            else query).to(self.device, torch.float32).contiguous()
        if q.dim() != 3 or q.shape[2] != self.head_dim:
            raise ValueError(f"query must be [batch, heads, {self.head_dim}], got {tuple(q.shape)}")
        if not ids:
            return np.zeros(tuple(q.shape), np.float32)
        idx = torch.tensor(ids, dtype=torch.int32, device=self.device)
        out = _C.block_decode(q, self._k, self._s, self._z, self._v, self._lens_dev, idx)
        return out.cpu().numpy()

    def memory_stats(self) -> dict:
        """Stored footprint vs FP16-equivalent, from the bytes actually held per block."""
        n = int(self._present.sum())
        if n == 0:
            return {'blocks': 0, 'stored_mb': 0.0, 'fp16_equiv_mb': 0.0, 'ratio': 0.0}
        half = (self.head_dim + 1) // 2
        rows = self._lens[self._present]
        stored = int(rows.sum()) * (half + 2 * self.head_dim) + n * 2 * 4 * self.head_dim
        fp16 = int(rows.sum()) * self.head_dim * 2 * 2
        return {'blocks': n, 'stored_mb': round(stored / 1048576, 3),
                'fp16_equiv_mb': round(fp16 / 1048576, 3), 'ratio': round(fp16 / max(stored, 1), 2)}
