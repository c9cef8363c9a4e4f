"""Seeded inputs of the layer-level golden cases (numpy only).

Shared by make_golden.py (which runs the reference CAREKVLayer on them) and
tests/test_gpu_layer.py (which runs this library's CAREKVLayer), so the
fixture holds outputs only.
"""

import numpy as np

# name, Hq, Hkv, D, prompt tokens T, decode steps, CAREKV_PREFILL_MODE, seed
LAYER_CASES = [
    ("gqa2_d64_fp", 4, 2, 64, 40, 24, "fp", 11),
    ("mha_d128_fp", 2, 2, 128, 33, 20, "fp", 12),
    ("gqa2_d64_base_quant", 4, 2, 64, 40, 6, "base_quant", 13),
]
# KIVI-style base (INT2, per-channel K / per-token V): name, Hq, Hkv, D, T,
# steps, prefill mode, seed, base quantizer
KIVI_LAYER_CASES = [
    ("gqa2_d64_kivi_base_quant", 4, 2, 64, 40, 24, "base_quant", 14, "kivi_style"),
]
DM = 96   # model width of the cases


def layer_inputs(Hq, Hkv, D, L, seed):
    """Weights W_Q/K/V/O, hidden states [L, DM] and RoPE tables cos/sin [1, L, D]."""
    rng = np.random.default_rng(seed)
    f = np.float32
    W_Q = (rng.standard_normal((Hq * D, DM)) / np.sqrt(DM)).astype(f)
    W_K = (rng.standard_normal((Hkv * D, DM)) / np.sqrt(DM)).astype(f)
    for h in range(Hkv):
        W_K[h * D:h * D + 4] *= 8.0     # outlier channels, as in the reference's tests
    W_V = (rng.standard_normal((Hkv * D, DM)) / np.sqrt(DM)).astype(f)
    W_O = (rng.standard_normal((DM, Hq * D)) / np.sqrt(Hq * D)).astype(f)
    hidden = rng.standard_normal((L, DM)).astype(f)
    inv = 1.0 / (10000.0 ** (np.arange(0, D, 2, dtype=np.float64) / D))
    fr = np.outer(np.arange(L, dtype=np.float64), inv)
    emb = np.concatenate([fr, fr], axis=-1)
    return W_Q, W_K, W_V, W_O, hidden, np.cos(emb).astype(f)[None], np.sin(emb).astype(f)[None]


def layer_cfg_kwargs(Hq, Hkv, D, L, base="uniform"):
    """CacheConfig keywords of a case: INT3 g32 packed, int8 scales, 1 K + 1 V
    slot stored per page, read budget 0 (base decode; the reference's decode
    step routes through its legacy cached router when a read budget is set)."""
    kw = dict(num_layers=1, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, page_size=16,
              max_pages=(L + 15) // 16 + 2, base_bits=3, group_size=32, k_channel_group=32,
              v_token_block=4, packed_base=True, scale_quant="int8", store_budget_mode="absolute",
              store_abs_k=1, store_abs_v=1, read_budget_mode="ratio", read_budget_ratio=0.0,
              route_policy="joint")
    if base != "uniform":
        # KIVI: INT2, the fp16 side buffer holds the base (no int8 scale step)
        kw.update(base_quantizer=base, base_bits=2, scale_quant="none")
    return kw
