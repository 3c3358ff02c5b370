"""CPU oracle for the INT4 KV quantizer and the paged INT4 flash-decode attention.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this
directory: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
legs of ``bench.py`` use it, and only as the checker / the timed CPU baseline.
The CUDA path never falls back to it.

What it is: a NumPy restatement of the reference's own NumPy algorithm for the
hot path (the reference itself is Python, so there is no C source to compile
into ``oracle/_ref``). Every function names the reference file:line it
restates. The restatement keeps the reference's arithmetic -- the same float32
operations in the same order -- because the quantizer gate is bit-exact.

Pinning: ``tests/golden/make_golden.py`` imported the reference package in the
build container and recorded its outputs on seeded inputs into
``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this oracle
against those vectors (quantizer and packing bit-exact; attention to 1e-6,
because the reference's BLAS summation order is not specified across CPUs).
"""

from .quantize import (  # noqa: F401
    quantize_int4,
    dequantize_int4,
    quantize_grouped,
)
from .pack import pack_int4, unpack_int4, packed_nbytes  # noqa: F401
from .attention import (  # noqa: F401
    online_softmax,
    online_softmax_state,
    merge_partials,
    decode_paged_state,
    attention_f64,
    attention_exact_f32_keys,
    paged_stream_pages,
    decode_paged,
    stream_f64,
)
from .rope import apply_rope, rope_table_f32  # noqa: F401
