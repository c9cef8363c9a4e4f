"""B200-native CARE-KV decode hot path.

Drop-in for the reference package's cache / quantizer / attention / layer /
HF-patch surface on the decode path, backed by hand-written sm_100a CUDA
kernels in lib/libcarekv_b200.so (C ABI: include/carekv_b200.h).
"""

from . import _lib, partition
from .config import (CacheConfig, apply_carekv_env_overrides, layer_budget_multiplier,
                     resolve_route_params, resolve_store_params, k_correction_mode)
from .cache import CAREKVCache, PageMeta
from .quantizer import (QuantConfig, KQuantizer, VQuantizer, quantize, dequantize, quantize_and_residual,
                        pack_int2_2d, unpack_int2_2d, pack_int3_2d, unpack_int3_2d, pack_int4_2d, unpack_int4_2d,
                        pack_codes_2d, unpack_codes_2d, packed_row_bytes, pack_4bit, unpack_4bit,
                        quant_dequant_kivi_k, quant_dequant_kivi_v)
from .engine import DecodeEngine
from .layer import CAREKVLayer, causal_attention, resolve_prefill_mode
from .llama_patch import CAREKVLlamaAttention, patch_llama_model, reset_all_caches
from .adapter import CAREKVAdapter

__version__ = "0.2.0+b200"

__all__ = [
    "CacheConfig", "CAREKVCache", "PageMeta", "apply_carekv_env_overrides", "layer_budget_multiplier",
    "resolve_route_params", "resolve_store_params", "k_correction_mode",
    "QuantConfig", "KQuantizer", "VQuantizer", "quantize", "dequantize", "quantize_and_residual",
    "pack_int2_2d", "unpack_int2_2d", "pack_int3_2d", "unpack_int3_2d", "pack_int4_2d", "unpack_int4_2d",
    "pack_codes_2d", "unpack_codes_2d", "packed_row_bytes", "pack_4bit", "unpack_4bit",
    "quant_dequant_kivi_k", "quant_dequant_kivi_v",
    "DecodeEngine", "CAREKVLayer", "causal_attention", "resolve_prefill_mode",
    "CAREKVLlamaAttention", "patch_llama_model", "reset_all_caches", "CAREKVAdapter",
]
