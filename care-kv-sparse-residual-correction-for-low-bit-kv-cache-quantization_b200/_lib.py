"""ctypes binding of libcarekv_b200.so (the C ABI in include/carekv_b200.h).

The library is the only compute path: if it is missing or cannot be loaded
every entry point raises; there is no CPU fallback.
"""

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libcarekv_b200.so")

# status codes
OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED = 2
ERR_CACHE_FULL = 3
ERR_CUDA = 4
ERR_WORKSPACE = 5
ERR_DEVICE_CHECK = 6

F32, F16, BF16 = 0, 1, 2
SCALE_INT8, SCALE_F16, SCALE_BF16, SCALE_F32 = 0, 1, 2, 3
KIND_BOTH, KIND_K, KIND_V, KIND_NONE = 0, 1, 2, 3
NUM_BUFFERS = 26
BASE_UNIFORM, BASE_KIVI = 0, 1

i32 = ctypes.c_int32
i64 = ctypes.c_int64
f32 = ctypes.c_float
vp = ctypes.c_void_p


class Config(ctypes.Structure):
    _fields_ = [(n, i32) for n in (
        "num_layers", "num_heads", "num_kv_heads", "head_dim", "page_size", "max_pages",
        "base_bits", "group_size", "k_channel_group", "v_token_block", "sketch_dim",
        "residual_bits", "scale_mode", "k_slots_per_page", "v_slots_per_page", "base_kind", "kivi_window_pages")]


CACHE_PTR_FIELDS = (
    "k_codes", "v_codes", "k_scale", "v_scale", "k_master", "v_master", "valid", "num_pages",
    "v_norm2", "k_slot_group", "k_slot_data", "k_slot_scale", "k_slot_id", "v_slot_block",
    "v_slot_data", "v_slot_scale", "v_slot_id", "k_err", "v_err", "k_sketch", "slot_counter",
    "read_counter", "error_flag", "k_chan_scale", "k_window", "prefill_tokens")
assert len(CACHE_PTR_FIELDS) == NUM_BUFFERS


class Cache(ctypes.Structure):
    _fields_ = [("batch", i32)] + [(n, vp) for n in CACHE_PTR_FIELDS]


class StoreParams(ctypes.Structure):
    _fields_ = [("k_budget", i32), ("v_budget", i32), ("joint_budget", i32), ("store_nothing", i32),
                ("sink_tokens", i32), ("token_start", i32), ("sensitivity", f32), ("input_dtype", i32),
                ("decode_page_master", i32)]


class RouteParams(ctypes.Structure):
    _fields_ = [("kind", i32), ("joint", i32), ("score_normalize", i32), ("kscore_live", i32),
                ("exact", i32), ("budget_mode", i32), ("read_k", i32), ("read_v", i32),
                ("ratio_k", ctypes.c_double), ("ratio_v", ctypes.c_double), ("k_corr_scale", f32), ("sensitivity", f32),
                ("lambda_k", f32), ("lambda_v", f32), ("legacy", i32), ("policy", i32), ("baseline_score", i32),
                ("adaptive_score", i32), ("rel_threshold", f32), ("abs_threshold", f32), ("min_keep", i32)]


POLICY = {"separate": 0, "joint": 1, "k_first": 2, "adaptive": 3}
SCORE = {"carekv": 0, "magnitude_only": 1, "attention_only": 2, "oracle_proxy": 3}


class Shard(ctypes.Structure):
    _fields_ = [("kvh_begin", i32), ("kvh_total", i32)]


# (name, restype, argtypes) of every exported symbol declared in the header
SIGNATURES = [
    ("carekv_abi_version", i32, []),
    ("carekv_status_string", ctypes.c_char_p, [i32]),
    ("carekv_cache_layout", i32, [ctypes.POINTER(Config), i32, ctypes.POINTER(ctypes.c_size_t)]),
    ("carekv_cache_init", i32, [ctypes.POINTER(Config), ctypes.POINTER(Cache), vp]),
    ("carekv_quantize", i32, [vp, vp, vp, i64, i32, i32, i32, i32, vp]),
    ("carekv_dequantize", i32, [vp, vp, vp, i64, i32, i32, i32, vp]),
    ("carekv_pack_codes", i32, [vp, vp, i64, i32, i32, vp]),
    ("carekv_unpack_codes", i32, [vp, vp, i64, i32, i32, vp]),
    ("carekv_pack_4bit", i32, [vp, vp, vp, i64, i32, vp]),
    ("carekv_unpack_4bit", i32, [vp, vp, vp, i64, i32, vp]),
    ("carekv_kivi_quant_dequant_k", i32, [vp, vp, i64, i32, i32, i32, i32, vp]),
    ("carekv_kivi_quant_dequant_v", i32, [vp, vp, i64, i32, i32, i32, vp]),
    ("carekv_prefill_store", i32, [ctypes.POINTER(Config), ctypes.POINTER(Cache), i32, vp, vp, i32, i32, i32,
                                   ctypes.POINTER(StoreParams), vp, vp]),
    ("carekv_append", i32, [ctypes.POINTER(Config), ctypes.POINTER(Cache), i32, vp, vp, i32, i32,
                            ctypes.POINTER(StoreParams), vp, i32, vp]),
    ("carekv_decode_workspace_bytes", i32, [ctypes.POINTER(Config), i32, i32, ctypes.POINTER(ctypes.c_size_t)]),
    ("carekv_decode_attention", i32, [ctypes.POINTER(Config), ctypes.POINTER(Cache), i32, vp, vp, i32, i32, i32,
                                      i32, ctypes.POINTER(RouteParams), vp, vp, ctypes.c_size_t, vp]),
    ("carekv_check_device_errors", i32, [ctypes.POINTER(Cache), ctypes.POINTER(i32), vp]),
    ("carekv_decode_attention_launches", i32, [ctypes.POINTER(Config), i32, ctypes.POINTER(i32)]),
    ("carekv_prefill_workspace_bytes", i32, [ctypes.POINTER(Config), i32, i32, ctypes.POINTER(ctypes.c_size_t)]),
    ("carekv_prefill_correction", i32, [ctypes.POINTER(Config), ctypes.POINTER(Cache), i32, i32, i32, i32, vp, vp,
                                        vp, vp, vp, vp, vp, vp, vp, vp, i32, ctypes.POINTER(RouteParams), vp, vp,
                                        ctypes.c_size_t, vp]),
    ("carekv_decode_attention_noalloc", i32, [ctypes.POINTER(Config), ctypes.POINTER(Cache), i32, vp, vp, i32, i32,
                                              i32, i32, ctypes.POINTER(RouteParams), vp, vp]),
    ("carekv_prefill_store_shard", i32, [ctypes.POINTER(Config), ctypes.POINTER(Cache), i32, vp, vp, i32, i32, i32,
                                         ctypes.POINTER(StoreParams), vp, ctypes.POINTER(Shard), vp]),
    ("carekv_append_shard", i32, [ctypes.POINTER(Config), ctypes.POINTER(Cache), i32, vp, vp, i32, i32,
                                  ctypes.POINTER(StoreParams), vp, i32, ctypes.POINTER(Shard), vp]),
    ("carekv_decode_attention_shard", i32, [ctypes.POINTER(Config), ctypes.POINTER(Cache), i32, vp, vp, i32, i32,
                                            i32, i32, ctypes.POINTER(RouteParams), vp, vp, ctypes.c_size_t,
                                            ctypes.POINTER(Shard), vp]),
]
NOALLOC_MAX_BYTES = 64 << 20

_lib = None
_load_error = None


def load(path=LIB_PATH):
    """dlopen the library and bind every declared symbol (no GPU needed)."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        _load_error = f"{path} not found; build it with build_lib.py (or __graft_entry__.build())"
        raise RuntimeError(_load_error)
    lib = ctypes.CDLL(path)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def lib():
    return load()


class CareKVError(RuntimeError):
    def __init__(self, status, where):
        msg = lib().carekv_status_string(status).decode()
        super().__init__(f"{where}: {msg} (status {status})")
        self.status = status


def check(status, where):
    if status != OK:
        if status == ERR_CACHE_FULL:
            raise CacheFullError(status, where)
        raise CareKVError(status, where)


class CacheFullError(CareKVError, AssertionError):
    """Raised when a page beyond max_pages is needed (the reference asserts
    "KV cache is full", cache.py:544)."""
