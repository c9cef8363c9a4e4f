"""Base quantizer, bit packers, 4-bit residual packer and int8 page scales.

Restates quantizer.py, residual_store.py:121-146 and cache.py:592-615,
656-701 of the reference in numpy.  All floating values are float32 arrays
holding numbers exactly representable in the logical dtype ``dt``.
"""

import numpy as np

from .numerics import round_to, scalar_in, to_int8_like_torch, F16


def quantize(x, bits, group_size, dt, clip_ratio=1.0):
    """Symmetric per-group quantizer (quantizer.py:31-64).

    x: (..., D) in ``dt``.  Returns int8 codes (..., D) and scales (..., D/g)
    in ``dt``.  scale = max|x|·clip / qmax with clamp(min=1e-8) done in ``dt``
    (1e-8 underflows to 0 in fp16, so an all-zero fp16 group gives 0/0 = NaN
    codes, which torch casts to int8 0).
    """
    x = np.asarray(x, dtype=np.float32)
    D = x.shape[-1]
    g = group_size
    assert D % g == 0
    xg = x.reshape(*x.shape[:-1], D // g, g)
    max_abs = np.abs(xg).max(axis=-1, keepdims=True)
    if clip_ratio != 1.0:
        max_abs = round_to(max_abs * np.float32(clip_ratio), dt)
    max_abs = np.maximum(max_abs, np.float32(scalar_in(dt, 1e-8)))
    qmax = 2 ** (bits - 1) - 1
    scale = round_to(max_abs / np.float32(qmax), dt)
    with np.errstate(divide="ignore", invalid="ignore"):
        xq = round_to(xg / scale, dt)
    xq = np.round(xq)
    xq = np.clip(xq, -qmax - 1, qmax)
    codes = to_int8_like_torch(xq).reshape(x.shape)
    return codes, scale[..., 0]


def dequantize(codes, scale, group_size, dt):
    """codes·scale in fp32, cast to the scale dtype (quantizer.py:67-82)."""
    codes = np.asarray(codes)
    D = codes.shape[-1]
    g = group_size
    cg = codes.reshape(*codes.shape[:-1], D // g, g).astype(np.float32)
    out = cg * np.asarray(scale, dtype=np.float32)[..., None]
    return round_to(out.reshape(codes.shape), dt)


def quantize_and_residual(x, bits, group_size, dt):
    """quantizer.py:85-99: codes, scale, residual x - x_hat (in ``dt``)."""
    codes, scale = quantize(x, bits, group_size, dt)
    x_hat = dequantize(codes, scale, group_size, dt)
    residual = round_to(np.asarray(x, np.float32) - x_hat, dt)
    return codes, scale, residual


def packed_row_bytes(D, bits):
    """quantizer.py:350-361."""
    if bits == 2:
        assert D % 4 == 0
        return D // 4
    if bits == 3:
        assert D % 8 == 0
        return D * 3 // 8
    if bits == 4:
        assert D % 2 == 0
        return D // 2
    raise ValueError(f"unsupported bits {bits}")


def pack_codes_2d(codes, bits):
    """(T, D) int8 -> (T, rowB) uint8 in the reference's row format.

    INT2: 4 codes per byte, lsb first (quantizer.py:257-264).
    INT3: 8 codes -> 24-bit little-endian word, 3 bits each, lsb first
          (quantizer.py:304-324).
    INT4: low nibble = even index (quantizer.py:283-290).
    """
    codes = np.asarray(codes, dtype=np.int8)
    T, D = codes.shape
    u = (codes.astype(np.int16) & 0xFF).astype(np.uint32)
    if bits == 2:
        u = (u & 0x3).reshape(T, D // 4, 4)
        return (u[..., 0] | (u[..., 1] << 2) | (u[..., 2] << 4) | (u[..., 3] << 6)).astype(np.uint8)
    if bits == 3:
        u = (u & 0x7).reshape(T, D // 8, 8)
        word = np.zeros(u.shape[:-1], dtype=np.uint32)
        for i in range(8):
            word |= u[..., i] << np.uint32(3 * i)
        b = np.stack([word & 0xFF, (word >> 8) & 0xFF, (word >> 16) & 0xFF], axis=-1)
        return b.reshape(T, D * 3 // 8).astype(np.uint8)
    if bits == 4:
        u = (u & 0xF).reshape(T, D // 2, 2)
        return (u[..., 0] | (u[..., 1] << 4)).astype(np.uint8)
    raise ValueError(bits)


def unpack_codes_2d(packed, bits, D):
    """Inverse of pack_codes_2d (quantizer.py:267-301, 327-343)."""
    p = np.asarray(packed).astype(np.uint8).astype(np.uint32)
    T = p.shape[0]
    if bits == 2:
        out = np.stack([(p >> (2 * i)) & 0x3 for i in range(4)], axis=-1).reshape(T, D)
        out = out.astype(np.int16)
        out[out >= 2] -= 4
        return out.astype(np.int8)
    if bits == 3:
        p = p.reshape(T, D // 8, 3)
        word = p[..., 0] | (p[..., 1] << 8) | (p[..., 2] << 16)
        out = np.stack([(word >> (3 * i)) & 0x7 for i in range(8)], axis=-1).reshape(T, D)
        out = out.astype(np.int16)
        out[out >= 4] -= 8
        return out.astype(np.int8)
    if bits == 4:
        out = np.stack([p & 0xF, (p >> 4) & 0xF], axis=-1).reshape(T, D).astype(np.int16)
        out[out >= 8] -= 16
        return out.astype(np.int8)
    raise ValueError(bits)


def pack_4bit(x):
    """4-bit symmetric residual slot (residual_store.py:121-136).

    s = max(max|x|, 1e-8)/7 in fp32; codes = round(x/s).clamp(-8, 7) over the
    row-major flattening; even index -> low nibble.  The stored scale is fp16(s).
    Returns (packed uint8, fp16 scale as float32, fp32 s used for the codes).
    """
    x = np.asarray(x, dtype=np.float32).reshape(-1)
    max_abs = np.maximum(np.abs(x).max(), np.float32(1e-8))
    s = np.float32(max_abs / np.float32(7.0))
    codes = np.clip(np.round(x / s), -8, 7).astype(np.int8)
    if codes.size % 2:
        codes = np.concatenate([codes, np.zeros(1, np.int8)])
    u = codes.astype(np.int16) & 0xF
    packed = (u[0::2] | (u[1::2] << 4)).astype(np.uint8)
    return packed, np.float32(np.float16(s)), s


def unpack_4bit(packed, scale, numel):
    """residual_store.py:139-146: nibbles -> signed -> · float(fp16 scale)."""
    p = np.asarray(packed).astype(np.uint8)
    lo = (p & 0xF).astype(np.int16)
    hi = (p >> 4).astype(np.int16)
    v = np.stack([lo, hi], axis=-1).reshape(-1)[:numel]
    v[v > 7] -= 16
    return v.astype(np.float32) * np.float32(scale)


def int8_scale_write(scale_in, dt):
    """Per-page int8 scale codes with one fp16 master (cache.py:592-606).

    master = fp16(max(max|s|, 1e-8 in dt) / 127) and
    code = round(s / master) clamped to [-128, 127], both in fp32.
    Returns (int8 codes, fp16 master as float32).
    """
    s = np.asarray(scale_in, dtype=np.float32)
    max_abs = np.maximum(np.abs(s).max(), np.float32(scalar_in(dt, 1e-8)))
    master = np.float32(np.float16(np.float32(max_abs / np.float32(127.0))))
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.round(s / master)
    codes = to_int8_like_torch(np.clip(q, -128, 127))
    return codes, master


def int8_scale_append(scale_row, master):
    """append_to_page's scale codes against a held master (cache.py:689-695)."""
    m = max(np.float32(master), np.float32(1e-8))
    q = np.round(np.asarray(scale_row, np.float32) / np.float32(m))
    return to_int8_like_torch(np.clip(q, -128, 127))


def int8_scale_read(codes, master):
    """_maybe_dequant_scale (cache.py:713-718): fp16(code · master)."""
    return round_to(np.asarray(codes, np.float32) * np.float32(master), F16)


def kivi_quant_dequant(x, bits, dt, axis):
    """quant_dequant_kivi_k (axis=-2: per-channel scale over the token axis)
    and quant_dequant_kivi_v (axis=-1: per-token scale over the channels) of
    kivi_helpers.py:35-59.  scale = amax / qmax, then clamp(min=1e-8), all in
    ``dt``; codes = clamp(round(x / scale), qmin, qmax); out = codes * scale.
    NaN (0/0 on an all-zero fp16 slice, where the clamp bound is 0) stays NaN."""
    x = np.asarray(x, dtype=np.float32)
    qmax = 2 ** (bits - 1) - 1
    amax = np.abs(x).max(axis=axis, keepdims=True)
    scale = round_to(amax / np.float32(qmax), dt)
    lo = np.float32(scalar_in(dt, 1e-8))
    scale = np.where(scale < lo, lo, scale)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        q = np.round(round_to(x / scale, dt))
        q = np.clip(q, -qmax - 1, qmax)
        return round_to(q * scale, dt)
