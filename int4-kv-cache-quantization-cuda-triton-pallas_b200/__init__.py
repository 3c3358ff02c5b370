"""B200-native (sm_100a) INT4 KV-cache quantization and fused paged flash-decoding.

A drop-in for the quantize / flash-decode operator surface of the reference
``flash_decode_int4`` package (its ``src/ops.py``), backed by hand-written
CUDA kernels in ``libint4kv_b200.so`` (C ABI: ``include/int4kv_b200.h``).

Modules:
  ops               -- the reference's operator API (+ paged / grouped operators)
  _C                -- torch-tensor binding of the C ABI (the reference's ``_C``)
  paged             -- device-resident paged INT4 KV cache
  vllm_integration  -- the reference's INT4PagedKVCache shim, device-resident
  int4_pack         -- host view of the nibble-packed storage format
  parallel          -- multi-GPU sharding and the sequence-split merge
  workloads         -- seeded synthetic inputs of the benchmark configurations

The package directory name is not a Python identifier; import it with
``importlib.import_module("int4-kv-cache-quantization-cuda-triton-pallas_b200")``.
"""

__version__ = "0.1.0"

from . import _lib  # noqa: F401
from ._lib import available as library_available  # noqa: F401
