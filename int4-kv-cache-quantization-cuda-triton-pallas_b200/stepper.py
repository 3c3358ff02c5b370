"""Decode steps of a Llama-style attention stack over INT4 paged KV caches.

One decode step of a layer is: rotary embedding of the step's query and key at
each sequence's position, quantize-on-append of the rotated key (and the
value) into the layer's pools, then the fused paged decode of the rotated
query over the whole cache, the new token included. The reference measures
this pipeline only as fake quantization inside a Hugging Face Llama
(scripts/validate_llama.py:23-31: post-RoPE keys quantized where attention
reads them); here each layer's step is two launches on the GPU:

  1. ``int4kv_cache_append_rope``: RoPE of q and k (transformers'
     rotate-half form), the key's open 128-token group quantized again over
     its valid rows, codes / scale / zero-point / value written to the pools;
  2. ``int4kv_paged_decode``: the split-KV flash-decode with its fused combine.

``LayerStack`` keeps every layer's pools in HBM. The sequences' pages have the
same ids in every layer's pool, so one block table and one length vector serve
all layers, and the lengths advance on the device: a whole step (all layers)
can be captured once as a CUDA graph and replayed per token with no host
work. Projections and the MLP are not part of this path (no weights exist
here); the step's q / k / v are inputs.
"""

from typing import List, Optional, Sequence

import numpy as np
import torch

from . import _C
from .rope import rope_table

PAGE_TOKENS = 16


class LayerStack:
    def __init__(self, num_layers: int, num_seqs: int, num_kv_heads: int, head_dim: int,
                 max_tokens: int, num_q_heads: Optional[int] = None, group_tokens: int = 128,
                 value_dtype=torch.float32, rope_base: float = 10000.0, device="cuda",
                 seed: int = 0):
        if num_layers <= 0 or num_seqs <= 0 or max_tokens <= 0:
            raise ValueError("num_layers, num_seqs and max_tokens must be positive")
        hq = num_q_heads if num_q_heads is not None else num_kv_heads
        if hq % num_kv_heads:
            raise ValueError("num_q_heads must be a multiple of num_kv_heads")
        if head_dim not in (64, 128, 256):
            raise ValueError("head_dim must be 64, 128 or 256")
        if group_tokens % PAGE_TOKENS or not 0 < group_tokens <= 128:
            raise ValueError("group_tokens must be a multiple of 16 in [16, 128]")
        self.layers, self.seqs = num_layers, num_seqs
        self.kv_heads, self.q_heads, self.head_dim = num_kv_heads, hq, head_dim
        self.group_tokens, self.max_tokens = group_tokens, max_tokens
        self.device = torch.device(device)
        self.value_dtype = value_dtype
        dev = self.device
        pages_per_seq = (max_tokens + PAGE_TOKENS - 1) // PAGE_TOKENS
        self.num_pages = num_seqs * pages_per_seq
        # every sequence's pages: a seeded scatter over the pool, the same in every layer
        perm = np.random.default_rng(seed).permutation(self.num_pages).astype(np.int32)
        self.block_table = torch.from_numpy(perm.reshape(num_seqs, pages_per_seq)).to(dev)
        shape_k = (self.num_pages, num_kv_heads, PAGE_TOKENS, head_dim // 2)
        shape_v = (self.num_pages, num_kv_heads, PAGE_TOKENS, head_dim)
        shape_sz = (self.num_pages, num_kv_heads, 2, head_dim)
        self.k_pools = [torch.zeros(shape_k, dtype=torch.uint8, device=dev) for _ in range(num_layers)]
        self.v_pools = [torch.zeros(shape_v, dtype=value_dtype, device=dev) for _ in range(num_layers)]
        self.sz_pools = [torch.zeros(shape_sz, dtype=torch.float32, device=dev)
                         for _ in range(num_layers)]
        # float32 post-RoPE keys of each sequence's open group, per layer (slot b = sequence b)
        self.stages = [torch.zeros((num_seqs, group_tokens, num_kv_heads * head_dim),
                                   dtype=torch.float32, device=dev) for _ in range(num_layers)]
        self.slots = torch.arange(num_seqs, dtype=torch.int32, device=dev)
        self.lens = torch.zeros((num_seqs,), dtype=torch.int32, device=dev)
        self.next_lens = torch.zeros_like(self.lens)
        self.host_lens = [0] * num_seqs
        self.rope = rope_table(max_tokens, head_dim, rope_base, dev)
        self.q_rot = torch.zeros((num_seqs, hq, head_dim), dtype=torch.float32, device=dev)
        self.out = torch.zeros((num_layers, num_seqs, hq, head_dim), dtype=torch.float32,
                               device=dev)
        self.workspace = torch.zeros((_C.paged_decode_workspace_bytes(
            num_seqs, hq, num_kv_heads, head_dim, dev, value_dtype=value_dtype),),
            dtype=torch.uint8, device=dev)
        self.graph = None

    # ---- prefill ----
    def prefill(self, keys: Sequence[torch.Tensor], values: Sequence[torch.Tensor],
                layers: Optional[Sequence[int]] = None) -> None:
        """Write every sequence's prompt ([len_b, kv_heads, head_dim] float32,
        pre-RoPE keys) into `layers` (default all): the keys are rotated at
        positions 0..len_b-1 on the GPU, quantized per 128-token group and
        scattered with the values; the open groups' rotated keys go to staging."""
        if len(keys) != self.seqs or len(values) != self.seqs:
            raise ValueError("one key and one value tensor per sequence")
        lens = [int(k.shape[0]) for k in keys]
        if max(lens) >= self.max_tokens:
            raise ValueError("prompt longer than max_tokens - 1")
        layers = list(range(self.layers)) if layers is None else list(layers)
        k = torch.cat([t.to(self.device, torch.float32) for t in keys]).contiguous()
        v = torch.cat([t.to(self.device, torch.float32) for t in values]).contiguous()
        pos = torch.from_numpy(np.concatenate([np.arange(n, dtype=np.int32) for n in lens]))
        k = _C.rope(k, pos.to(self.device), self.rope[0], self.rope[1])
        offs_np = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        offs = torch.from_numpy(offs_np).to(self.device)
        for l in layers:
            _C.cache_write(k, v, offs, self.block_table, self.k_pools[l], self.v_pools[l],
                           self.sz_pools[l], max_rows_per_seq=max(1, max(lens)),
                           group_tokens=self.group_tokens)
            for b, n in enumerate(lens):
                r = n % self.group_tokens
                if r:
                    o = int(offs_np[b]) + n - r
                    self.stages[l][b, :r] = k[o:o + r].reshape(r, -1)
        self.host_lens = lens
        self.lens.copy_(torch.tensor(lens, dtype=torch.int32))

    def copy_layer(self, src: int, dst: int) -> None:
        """Make layer `dst` hold the same cache as layer `src` (synthetic setups)."""
        self.k_pools[dst].copy_(self.k_pools[src])
        self.v_pools[dst].copy_(self.v_pools[src])
        self.sz_pools[dst].copy_(self.sz_pools[src])
        self.stages[dst].copy_(self.stages[src])

    # ---- the step ----
    def _layer_input(self, t: torch.Tensor, l: int) -> torch.Tensor:
        return t[l] if t.dim() == 4 else t

    def _launch(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        torch.add(self.lens, 1, out=self.next_lens)
        for l in range(self.layers):
            _C.cache_append(self._layer_input(k, l), self._layer_input(v, l), self.lens,
                            self.slots, self.stages[l], self.block_table, self.k_pools[l],
                            self.v_pools[l], self.sz_pools[l], group_tokens=self.group_tokens,
                            rope=self.rope, q=self._layer_input(q, l), q_out=self.q_rot)
            _C.paged_decode(self.q_rot, self.k_pools[l], self.v_pools[l], self.sz_pools[l],
                            self.block_table, self.next_lens, self.group_tokens,
                            out=self.out[l], workspace=self.workspace)
        self.lens.copy_(self.next_lens)
        return self.out

    def _advance(self) -> None:
        if max(self.host_lens) + 1 > self.max_tokens:
            raise RuntimeError(f"a sequence would exceed max_tokens ({self.max_tokens})")
        self.host_lens = [n + 1 for n in self.host_lens]

    def step(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """One token for every sequence in every layer. q [B, q_heads, D] or
        [layers, B, q_heads, D] (pre-RoPE); k, v [B, kv_heads, D] or per layer.
        Returns the attention outputs [layers, B, q_heads, D] (a view of a
        buffer that the next step overwrites)."""
        self._advance()
        return self._launch(q, k, v)

    def capture(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """Record one step as a CUDA graph with q / k / v as its input buffers
        (copy each token's inputs into them, then ``replay()``). Capturing does
        not advance the cache: the recorded launches run only on replay."""
        lens0 = self.lens.clone()
        # One warm-up step outside the capture (kernels loaded, launch attributes
        # set). It writes exactly the cells the first replay rewrites -- the
        # open groups re-quantized from the staged rows plus the new row at
        # position lens -- so restoring the lengths restores the cache.
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._launch(q, k, v)
        torch.cuda.current_stream(self.device).wait_stream(side)
        self.lens.copy_(lens0)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._launch(q, k, v)
        torch.cuda.synchronize(self.device)
        self.lens.copy_(lens0)  # capture records but executes nothing
        return self.out

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            raise RuntimeError("capture() first")
        self._advance()
        self.graph.replay()
        return self.out

    def release(self) -> None:
        self.graph = None

    # ---- accounting ----
    def step_bytes(self) -> int:
        """Algorithmic HBM bytes of the next step: per layer, the decode over
        every sequence's length + 1 tokens (packed keys, values, scale/zp, query,
        output, block-table entries) and the append (the open group's staged
        rows read, its codes rewritten, the new key / value / scale / zp written,
        q read and rotated q written)."""
        d, h, hq = self.head_dim, self.kv_heads, self.q_heads
        vb = 4 if self.value_dtype == torch.float32 else 2
        c = h * d
        total = 0
        for n in self.host_lens:
            L = n + 1
            groups = (L + self.group_tokens - 1) // self.group_tokens
            pages = (L + PAGE_TOKENS - 1) // PAGE_TOKENS
            dec = h * (L * d // 2 + vb * L * d + 8 * d * groups) + 4 * pages + 8 * hq * d
            rows = n % self.group_tokens + 1
            app = (rows - 1) * c * 4 + 3 * c * 4 + rows * c // 2 + vb * c + 8 * c + 8 * hq * d
            total += dec + app
        return total * self.layers
