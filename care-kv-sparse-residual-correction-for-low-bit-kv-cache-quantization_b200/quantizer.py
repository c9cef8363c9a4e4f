"""Quantizer API of the reference (quantizer.py, residual_store.py:121-176) on the GPU.

Same names, arguments and return conventions; every function runs the
library's CUDA kernels on CUDA tensors and raises for CPU tensors.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Tuple

import torch
from torch import Tensor

from . import _lib

_DT = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


@dataclass
class QuantConfig:
    bits: int = 2
    group_size: int = 64
    symmetric: bool = True
    clip_ratio: float = 1.0


def _cuda(t: Tensor, what: str) -> Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"{what}: the B200 build runs on CUDA tensors only (got {t.device})")
    return t.contiguous()


def _stream(t: Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def quantize(x: Tensor, cfg: QuantConfig) -> Tuple[Tensor, Tensor]:
    """quantizer.py:31-64 -> (int8 codes (..., D), scale (..., D/g) in x.dtype)."""
    if cfg.clip_ratio != 1.0:
        raise NotImplementedError("clip_ratio != 1 is not built")
    x = _cuda(x, "quantize")
    D, g = x.shape[-1], cfg.group_size
    assert D % g == 0, f"head_dim {D} must be divisible by group_size {g}"
    rows = x.numel() // D
    codes = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    scale = torch.empty(*x.shape[:-1], D // g, dtype=x.dtype, device=x.device)
    _lib.check(_lib.lib().carekv_quantize(x.data_ptr(), codes.data_ptr(), scale.data_ptr(), rows, D, cfg.bits, g,
                                          _DT[x.dtype], _stream(x)), "quantize")
    return codes, scale


def dequantize(codes: Tensor, scale: Tensor, orig_shape, cfg: QuantConfig) -> Tensor:
    """quantizer.py:67-82: codes*scale in fp32, cast to scale.dtype."""
    codes = _cuda(codes, "dequantize")
    scale = _cuda(scale, "dequantize")
    D = orig_shape[-1]
    rows = codes.numel() // D
    out = torch.empty(tuple(orig_shape), dtype=scale.dtype, device=codes.device)
    _lib.check(_lib.lib().carekv_dequantize(codes.data_ptr(), scale.data_ptr(), out.data_ptr(), rows, D,
                                            cfg.group_size, _DT[scale.dtype], _stream(codes)), "dequantize")
    return out


def quantize_and_residual(x: Tensor, cfg: QuantConfig):
    """quantizer.py:85-99."""
    codes, scale = quantize(x, cfg)
    x_hat = dequantize(codes, scale, x.shape, cfg)
    return codes, scale, x - x_hat, x.shape


class KQuantizer:
    def __init__(self, cfg: QuantConfig):
        self.cfg = cfg

    def encode(self, K: Tensor):
        return quantize_and_residual(K, self.cfg)

    def decode(self, codes, scale, shape) -> Tensor:
        return dequantize(codes, scale, shape, self.cfg)


class VQuantizer(KQuantizer):
    pass


def packed_row_bytes(D: int, bits: int) -> int:
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
    raise ValueError(f"Unsupported base_bits={bits} for packed storage")


def pack_codes_2d(codes: Tensor, bits: int) -> Tensor:
    """(T, D) int8 -> (T, packed_row_bytes) int8 (quantizer.py:364-372)."""
    if bits not in (2, 3, 4):
        raise ValueError(f"Unsupported base_bits={bits}")
    codes = _cuda(codes.to(torch.int8), "pack_codes_2d")
    T, D = codes.shape
    out = torch.empty(T, packed_row_bytes(D, bits), dtype=torch.int8, device=codes.device)
    _lib.check(_lib.lib().carekv_pack_codes(codes.data_ptr(), out.data_ptr(), T, D, bits, _stream(codes)),
               "pack_codes_2d")
    return out


def unpack_codes_2d(packed: Tensor, bits: int, D: int) -> Tensor:
    """Inverse of pack_codes_2d (quantizer.py:375-383). Returns (T, D) int8."""
    if bits not in (2, 3, 4):
        raise ValueError(f"Unsupported base_bits={bits}")
    packed = _cuda(packed, "unpack_codes_2d")
    T = packed.shape[0]
    out = torch.empty(T, D, dtype=torch.int8, device=packed.device)
    _lib.check(_lib.lib().carekv_unpack_codes(packed.data_ptr(), out.data_ptr(), T, D, bits, _stream(packed)),
               "unpack_codes_2d")
    return out


def pack_int2_2d(codes):
    return pack_codes_2d(codes, 2)


def unpack_int2_2d(packed, D):
    return unpack_codes_2d(packed, 2, D)


def pack_int3_2d(codes):
    return pack_codes_2d(codes, 3)


def unpack_int3_2d(packed, D):
    return unpack_codes_2d(packed, 3, D)


def pack_int4_2d(codes):
    return pack_codes_2d(codes, 4)


def unpack_int4_2d(packed, D):
    return unpack_codes_2d(packed, 4, D)


def pack_4bit(x: Tensor, scale_hint=None) -> Tuple[Tensor, Tensor]:
    """residual_store.py:121-136: 4-bit slot of x -> (packed int8, fp16 scale (1,))."""
    x = _cuda(x.float(), "pack_4bit").reshape(-1)
    n = x.numel()
    if n % 2:
        x = torch.cat([x, x.new_zeros(1)])
    packed = torch.empty(x.numel() // 2, dtype=torch.uint8, device=x.device)
    sc = torch.empty(1, dtype=torch.float16, device=x.device)
    _lib.check(_lib.lib().carekv_pack_4bit(x.data_ptr(), packed.data_ptr(), sc.data_ptr(), 1, x.numel(),
                                           _stream(x)), "pack_4bit")
    return packed.view(torch.int8), sc


def unpack_4bit(packed: Tensor, scale: Tensor, numel: int) -> Tensor:
    """residual_store.py:139-146 -> float values."""
    packed = _cuda(packed, "unpack_4bit").reshape(-1)
    n2 = packed.numel() * 2
    out = torch.empty(n2, dtype=torch.float32, device=packed.device)
    sc = _cuda(scale.reshape(-1)[:1].to(torch.float16), "unpack_4bit")
    _lib.check(_lib.lib().carekv_unpack_4bit(packed.data_ptr(), sc.data_ptr(), out.data_ptr(), 1, n2,
                                             _stream(packed)), "unpack_4bit")
    return out[:numel]


def quant_dequant_kivi_k(K: Tensor, bits: int) -> Tensor:
    """kivi_helpers.py:35-46: K (..., T, D) -> symmetric INT`bits`
    quantize-dequantize with a per-channel scale over T, in K's dtype."""
    K = _cuda(K, "quant_dequant_kivi_k").contiguous()
    T, D = K.shape[-2], K.shape[-1]
    n = K.numel() // (T * D) if T * D else 0
    out = torch.empty_like(K)
    _lib.check(_lib.lib().carekv_kivi_quant_dequant_k(K.data_ptr(), out.data_ptr(), n, T, D, bits, _DT[K.dtype],
                                                      _stream(K)), "quant_dequant_kivi_k")
    return out


def quant_dequant_kivi_v(V: Tensor, bits: int) -> Tensor:
    """kivi_helpers.py:49-59: V (..., T, D) -> symmetric INT`bits`
    quantize-dequantize with a per-token scale over D, in V's dtype."""
    V = _cuda(V, "quant_dequant_kivi_v").contiguous()
    D = V.shape[-1]
    rows = V.numel() // D if D else 0
    out = torch.empty_like(V)
    _lib.check(_lib.lib().carekv_kivi_quant_dequant_v(V.data_ptr(), out.data_ptr(), rows, D, bits, _DT[V.dtype],
                                                      _stream(V)), "quant_dequant_kivi_v")
    return out
