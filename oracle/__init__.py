"""CPU oracle for the CARE-KV decode hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference project's algorithm for the
path the B200 build accelerates: per-group INT2/3/4 quantize-and-pack on
append, the paged packed cache with int8 page scales, per-page residual
enumeration and 4-bit slot storage, the combined_kvscore router with joint
top-k, and the exact softmax K correction.  Every function cites the
reference file:line it follows (paths are relative to the reference
project root, which is imported as ``CARE_KV.care_kv``).

Who may use it: ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``, and only as the
checker or the timed CPU baseline.  The product package never imports it;
its GPU path fails loudly when the CUDA library is missing.

Parity pin: the restatement is checked against golden vectors produced by
running the reference itself (``tests/golden/make_golden.py``; fixtures in
``tests/golden/*.npz``) by ``tests/test_oracle_golden.py``.
"""

from .numerics import round_to, bf16_round, f16_round, F32, F16, BF16
from .quant import (
    quantize, dequantize, quantize_and_residual,
    pack_codes_2d, unpack_codes_2d, packed_row_bytes,
    pack_4bit, unpack_4bit, int8_scale_write, int8_scale_read,
    int8_scale_append,
)
from .store import StoreConfig, process_page, sketch_projection
from .cache import OracleCache
from .attention import (
    RouteConfig, base_attention, vectorized_joint_correction,
    exact_softmax_correction, decode_attention_kvh,
)

__all__ = [
    "round_to", "bf16_round", "f16_round", "F32", "F16", "BF16",
    "quantize", "dequantize", "quantize_and_residual",
    "pack_codes_2d", "unpack_codes_2d", "packed_row_bytes",
    "pack_4bit", "unpack_4bit", "int8_scale_write", "int8_scale_read",
    "int8_scale_append",
    "StoreConfig", "process_page", "sketch_projection",
    "OracleCache",
    "RouteConfig", "base_attention", "vectorized_joint_correction",
    "exact_softmax_correction", "decode_attention_kvh",
]
