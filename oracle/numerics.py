"""Rounding helpers that reproduce torch CPU arithmetic on fp16 / bf16 tensors.

torch computes every elementwise op on a half or bfloat16 tensor in fp32 and
rounds the result back to the tensor dtype (round-to-nearest-even).  The
oracle keeps all values as float32 arrays holding numbers that are exactly
representable in the logical dtype, and calls ``round_to`` after each op the
reference performs in that dtype.
"""

import numpy as np

F32, F16, BF16 = "fp32", "fp16", "bf16"


def f16_round(x):
    """fp32 -> nearest-even fp16 -> fp32 (numpy's float16 cast is RNE)."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def bf16_round(x):
    """fp32 -> nearest-even bfloat16 -> fp32, the c10::BFloat16 rounding rule."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    b = x.view(np.uint32).astype(np.uint64)
    lsb = (b >> np.uint64(16)) & np.uint64(1)
    b = (b + np.uint64(0x7FFF) + lsb) & np.uint64(0xFFFF0000)
    out = b.astype(np.uint32).view(np.float32).reshape(x.shape)
    return np.where(np.isnan(x), np.float32(np.nan), out).astype(np.float32)


def round_to(x, dt):
    """Round an fp32 array to the logical dtype ``dt`` (kept as float32)."""
    if dt == F32:
        return np.asarray(x, dtype=np.float32)
    if dt == F16:
        return f16_round(x)
    if dt == BF16:
        return bf16_round(x)
    raise ValueError(f"unknown dtype {dt!r}")


def scalar_in(dt, v):
    """A Python float scalar as torch converts it for clamp() on a ``dt`` tensor."""
    return float(round_to(np.array([v], np.float32), dt)[0])


def to_int8_like_torch(x):
    """float -> int8 the way torch's CPU cast behaves for the values seen here.

    Finite in-range values are exact integers already.  NaN (0/0 in the fp16
    quantizer on an all-zero padded row) converts through a 32-bit integer
    cast to 0x80000000, whose low byte is 0.
    """
    x = np.asarray(x, dtype=np.float32)
    out = np.where(np.isnan(x), 0.0, x)
    return out.astype(np.int8)


def bf16_bits(x):
    """bf16 values held as float32 -> their uint16 bit patterns."""
    return (np.ascontiguousarray(bf16_round(x)).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b):
    b = np.asarray(b, dtype=np.uint32) << np.uint32(16)
    return b.view(np.float32)
