"""CacheConfig, the CAREKV_* environment overrides and per-layer policy resolution.

Mirrors cache.py:51-384 of the reference (same field names, defaults and
validation errors) and resolves, once per call, the environment knobs the
reference reads deep inside its hot path (attention.py:89-93, 678, 839-842;
layer.py:505-509, 1150; residual_store.py:104-114) into the plain-data
parameter structs of the C ABI.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import List, Optional

from . import _lib


def apply_carekv_env_overrides(kwargs: dict) -> dict:
    """Mutate ``kwargs`` in place to honour CAREKV_* env vars (cache.py:51-125)."""
    def _ovr(env, key, conv):
        if env in os.environ and os.environ[env] != "":
            kwargs[key] = conv(os.environ[env])

    _b = lambda v: v == "1"  # noqa: E731
    for env, key, conv in (
        ("CAREKV_PAGE_SIZE", "page_size", int), ("CAREKV_V_TOKEN_BLOCK", "v_token_block", int),
        ("CAREKV_K_CHANNEL_GROUP", "k_channel_group", int), ("CAREKV_SKETCH_DIM", "sketch_dim", int),
        ("CAREKV_GROUP_SIZE", "group_size", int), ("CAREKV_MAX_PAGES", "max_pages", int),
        ("CAREKV_BASE_BITS", "base_bits", int), ("CAREKV_RESIDUAL_BITS", "residual_bits", int),
        ("CAREKV_STORE_BUDGET", "store_budget_ratio", float), ("CAREKV_READ_BUDGET", "read_budget_ratio", float),
        ("CAREKV_PACKED_BASE", "packed_base", _b), ("CAREKV_SCALE_DTYPE", "scale_dtype", str),
        ("CAREKV_SCALE_QUANT", "scale_quant", str), ("CAREKV_ROUTE_POLICY", "route_policy", str),
        ("CAREKV_STORE_BUDGET_MODE", "store_budget_mode", str), ("CAREKV_READ_BUDGET_MODE", "read_budget_mode", str),
        ("CAREKV_STORE_BUDGET_K", "store_budget_ratio_k", float), ("CAREKV_STORE_BUDGET_V", "store_budget_ratio_v", float),
        ("CAREKV_READ_BUDGET_K", "read_budget_ratio_k", float), ("CAREKV_READ_BUDGET_V", "read_budget_ratio_v", float),
        ("CAREKV_STORE_ABS_K", "store_abs_k", int), ("CAREKV_STORE_ABS_V", "store_abs_v", int),
        ("CAREKV_READ_ABS_K", "read_abs_k", int), ("CAREKV_READ_ABS_V", "read_abs_v", int),
        ("CAREKV_CORRECTION_IMPL", "correction_impl", str), ("CAREKV_PACK_IMPL", "pack_impl", str),
        ("CAREKV_BUDGET_POLICY", "budget_policy", str), ("CAREKV_VDOM_OPTIMIZED", "vdom_optimized", _b),
        ("CAREKV_READ_RELATIVE_THRESHOLD", "read_relative_threshold", float),
        ("CAREKV_READ_ABSOLUTE_THRESHOLD", "read_absolute_threshold", float),
        ("CAREKV_READ_MIN_KEEP", "read_min_keep", int),
        ("CAREKV_READ_SCORE_TEMPERATURE", "read_score_temperature", float),
        ("CAREKV_CORRECTION_NORM_CLIP", "correction_norm_clip", float),
        ("CAREKV_BASE_QUANTIZER", "base_quantizer", str), ("CAREKV_K_BITS", "k_bits_override", int),
        ("CAREKV_V_BITS", "v_bits_override", int), ("CAREKV_K_STORE_MODE", "k_store_mode", str),
        ("CAREKV_BASELINE_SCORE", "baseline_score", str),
    ):
        _ovr(env, key, conv)
    if os.environ.get("CAREKV_LAYER_SENSITIVITY"):
        try:
            kwargs["layer_sensitivity"] = [float(x) for x in os.environ["CAREKV_LAYER_SENSITIVITY"].split(",")
                                           if x.strip()]
        except ValueError:
            pass
    return kwargs


def _u_shape_multipliers(L: int) -> List[float]:
    """cache.py:166-177."""
    if L <= 1:
        return [1.0]
    raw = [0.5 + 1.5 * abs(2 * (l / (L - 1)) - 1) for l in range(L)]
    mean_w = sum(raw) / L
    return [w / mean_w for w in raw]


def layer_budget_multiplier(cfg: "CacheConfig", layer_id: int) -> float:
    """cache.py:180-202."""
    policy = getattr(cfg, "budget_policy", "uniform")
    L = cfg.num_layers
    if policy == "uniform" or L <= 1:
        return 1.0
    if policy == "u_shaped":
        return _u_shape_multipliers(L)[layer_id]
    if policy == "sensitivity":
        s = cfg.layer_sensitivity or [1.0] * L
        mean_s = sum(s) / max(L, 1)
        return 1.0 if mean_s <= 0 else s[layer_id] / mean_s
    return 1.0


@dataclass
class CacheConfig:
    """Same fields, defaults and validation as the reference (cache.py:209-384)."""
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: Optional[int] = None
    head_dim: int = 128
    page_size: int = 16
    max_pages: int = 512
    base_bits: int = 2
    residual_bits: int = 4
    group_size: int = 64
    k_channel_group: int = 32
    v_token_block: int = 4
    store_budget_ratio: float = 0.10
    read_budget_ratio: float = 0.03
    sketch_dim: int = 32
    layer_sensitivity: Optional[List[float]] = None
    packed_base: bool = False
    packed_storage: bool = False
    scale_dtype: str = "fp16"
    scale_quant: str = "none"
    store_budget_mode: str = "ratio"
    read_budget_mode: str = "ratio"
    store_budget_ratio_k: Optional[float] = None
    store_budget_ratio_v: Optional[float] = None
    read_budget_ratio_k: Optional[float] = None
    read_budget_ratio_v: Optional[float] = None
    store_abs_k: int = 0
    store_abs_v: int = 0
    read_abs_k: int = 0
    read_abs_v: int = 0
    route_policy: str = "separate"
    vdom_optimized: bool = False
    read_relative_threshold: float = 0.0
    read_absolute_threshold: float = 0.0
    read_min_keep: int = 0
    read_score_temperature: float = 1.0
    correction_norm_clip: float = 0.0
    base_quantizer: str = "uniform"
    k_bits_override: int = -1
    v_bits_override: int = -1
    k_store_mode: str = "post_rope"
    baseline_score: str = "carekv"
    correction_impl: str = "cached"
    pack_impl: str = "vectorized"
    budget_policy: str = "uniform"
    # B200 build only: keep the fp16 K sketches (read by the cached router and
    # the vectorized router's sketch proxy score; combined_kvscore never reads
    # them).  None: kept unless correction_impl is "vectorized" (the
    # reference stores them always; its cached router needs them).
    store_sketch: Optional[bool] = None
    # B200 build only, KIVI-style base: pages of fp16 K rows per (sequence,
    # layer, kv head) kept for decode-appended tokens (the reference keeps
    # them in its fp16 side buffer, cache.py:487-499)
    kivi_window_pages: int = 8

    def __post_init__(self):
        if self.layer_sensitivity is None:
            self.layer_sensitivity = [1.0] * self.num_layers
        if self.num_kv_heads is None:
            self.num_kv_heads = self.num_heads
        if self.packed_storage and not self.packed_base:
            self.packed_base = True
        if self.scale_dtype not in {"fp16", "bf16", "fp32"}:
            raise ValueError(f"scale_dtype must be fp16/bf16/fp32, got {self.scale_dtype}")
        if self.scale_quant not in {"none", "int8"}:
            raise ValueError(f"scale_quant must be none/int8, got {self.scale_quant}")
        if self.store_budget_mode not in {"ratio", "absolute"}:
            raise ValueError(f"store_budget_mode={self.store_budget_mode}")
        if self.read_budget_mode not in {"ratio", "absolute", "adaptive_score"}:
            raise ValueError(f"read_budget_mode={self.read_budget_mode}")
        if self.route_policy not in {"joint", "separate", "k_first", "adaptive"}:
            raise ValueError(f"route_policy={self.route_policy}")
        if self.correction_impl not in {"python", "cached", "vectorized"}:
            raise ValueError(f"correction_impl={self.correction_impl}")
        if self.pack_impl not in {"python", "vectorized"}:
            raise ValueError(f"pack_impl={self.pack_impl}")
        if self.budget_policy not in {"uniform", "u_shaped", "sensitivity", "layer_head_impact"}:
            raise ValueError(f"budget_policy={self.budget_policy}")
        if self.store_sketch is None:
            self.store_sketch = self.correction_impl != "vectorized"

    def scale_torch_dtype(self):
        import torch
        return {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[self.scale_dtype]

    # ── B200 build helpers ───────────────────────────────────────────
    @property
    def num_k_groups(self) -> int:
        return self.head_dim // self.k_channel_group

    @property
    def num_v_blocks(self) -> int:
        return math.ceil(self.page_size / self.v_token_block)

    @property
    def padded_max_pages(self) -> int:
        return ((self.max_pages + 7) // 8) * 8

    def scale_mode(self) -> int:
        if self.scale_quant == "int8":
            return _lib.SCALE_INT8
        return {"fp16": _lib.SCALE_F16, "bf16": _lib.SCALE_BF16, "fp32": _lib.SCALE_F32}[self.scale_dtype]

    def slot_capacity(self):
        """Per-page K / V slot capacity: the largest store budget of any layer."""
        sk = sv = 0
        for l in range(self.num_layers):
            sp = resolve_store_params(self, l, _lib.F32)
            if sp.joint_budget > 0:
                sk = max(sk, min(sp.joint_budget, self.num_k_groups))
                sv = max(sv, min(sp.joint_budget, self.num_v_blocks))
            else:
                sk = max(sk, min(sp.k_budget, self.num_k_groups))
                sv = max(sv, min(sp.v_budget, self.num_v_blocks))
        return sk, sv

    @property
    def is_kivi(self) -> bool:
        """KIVI-style base (kivi_style; kvquant_style is its post-RoPE twin,
        kivi_helpers.py:187-189)."""
        return self.base_quantizer in ("kivi_style", "kvquant_style")

    def c_config(self) -> "_lib.Config":
        if self.base_quantizer not in ("uniform", "kivi_style", "kvquant_style"):
            raise NotImplementedError(
                f"base_quantizer={self.base_quantizer!r}: the uniform and KIVI-style bases are built")
        if self.is_kivi:
            for o in (self.k_bits_override, self.v_bits_override):
                if o > 0 and o != self.base_bits:
                    raise NotImplementedError("KIVI base: K and V bits must both equal base_bits")
            if self.k_store_mode != "post_rope":
                raise NotImplementedError("KIVI base: only the post-RoPE K store is built")
        if self.residual_bits != 4:
            raise NotImplementedError("residual_bits must be 4")
        sk, sv = self.slot_capacity()
        c = _lib.Config()
        c.num_layers = self.num_layers
        c.num_heads = self.num_heads
        c.num_kv_heads = self.num_kv_heads
        c.head_dim = self.head_dim
        c.page_size = self.page_size
        c.max_pages = self.padded_max_pages
        c.base_bits = self.base_bits
        # KIVI: one V scale per token (group = head_dim), scales kept as fp32
        # holding their activation-dtype values
        c.group_size = self.head_dim if self.is_kivi else self.group_size
        c.k_channel_group = self.k_channel_group
        c.v_token_block = self.v_token_block
        c.sketch_dim = self.sketch_dim if self.store_sketch else 0
        c.residual_bits = self.residual_bits
        c.scale_mode = _lib.SCALE_F32 if self.is_kivi else self.scale_mode()
        c.k_slots_per_page = sk
        c.v_slots_per_page = sv
        c.base_kind = _lib.BASE_KIVI if self.is_kivi else _lib.BASE_UNIFORM
        c.kivi_window_pages = self.kivi_window_pages if self.is_kivi else 0
        return c


# ── store policy (residual_store.py:104-114, 370-423) ─────────────────
def _store_env():
    policy = os.environ.get("CAREKV_STORE_POLICY", "residual_kind_aware").lower()
    kind = os.environ.get("CAREKV_PREFILL_RESIDUAL_KIND", "both").lower()
    mpk = int(os.environ.get("CAREKV_STORE_MIN_PER_KIND", "1"))
    kf = float(os.environ.get("CAREKV_STORE_K_FRACTION", "1.0"))
    vf = float(os.environ.get("CAREKV_STORE_V_FRACTION", "1.0"))
    if policy not in {"joint", "per_kind", "residual_kind_aware"}:
        raise ValueError(f"Unknown CAREKV_STORE_POLICY={policy}")
    if kind not in {"v", "k", "both"}:
        raise ValueError(f"Unknown CAREKV_PREFILL_RESIDUAL_KIND={kind}")
    return policy, kind, mpk, kf, vf


def resolve_store_params(cfg: CacheConfig, layer_id: int, input_dtype: int,
                         token_start: int = 0, sink_tokens: int = 4) -> "_lib.StoreParams":
    policy, kind, mpk, kf, vf = _store_env()
    use_k = not (policy == "residual_kind_aware" and kind == "v")
    use_v = not (policy == "residual_kind_aware" and kind == "k")
    lm = layer_budget_multiplier(cfg, layer_id)
    kt, vt = max(1, cfg.num_k_groups), max(1, cfg.num_v_blocks)
    if cfg.store_budget_mode == "absolute":
        kb = int(round(max(0, int(cfg.store_abs_k)) * lm)) if use_k else 0
        vb = int(round(max(0, int(cfg.store_abs_v)) * lm)) if use_v else 0
        joint = kb + vb
    else:
        def _res(o, fb):
            return fb if (o is None or o < 0) else o
        rk = _res(cfg.store_budget_ratio_k, cfg.store_budget_ratio) * kf * lm
        rv = _res(cfg.store_budget_ratio_v, cfg.store_budget_ratio) * vf * lm
        kb = max(mpk, int(kt * rk)) if (use_k and rk > 0) else 0
        vb = max(mpk, int(vt * rv)) if (use_v and rv > 0) else 0
        joint = max(1, int((kt + vt) * cfg.store_budget_ratio * lm))
    nothing = (cfg.store_budget_ratio <= 0 and cfg.store_budget_mode != "absolute"
               and (cfg.store_budget_ratio_k or 0) <= 0 and (cfg.store_budget_ratio_v or 0) <= 0)
    p = _lib.StoreParams()
    p.k_budget = max(0, kb)
    p.v_budget = max(0, vb)
    p.joint_budget = joint if (policy == "joint" and not nothing) else 0
    p.store_nothing = 1 if nothing else 0
    p.sink_tokens = sink_tokens
    p.token_start = token_start
    p.sensitivity = float(cfg.layer_sensitivity[layer_id])
    p.input_dtype = input_dtype
    # CAREKV_DECODE_PAGE_MASTER=1: a page opened during decode takes its int8
    # master from its first row instead of keeping the reference's 0
    # (cache.py:689-695, whose appended rows then read back as zero)
    p.decode_page_master = 1 if os.environ.get("CAREKV_DECODE_PAGE_MASTER", "0").lower() in {"1", "true", "yes"} else 0
    return p


# ── routing / correction policy ────────────────────────────────────────
def k_correction_mode() -> str:
    """attention.py:89-93."""
    m = os.environ.get("CAREKV_K_CORRECTION_MODE", "linear").lower()
    if m not in {"linear", "exact"}:
        raise ValueError(f"Unknown CAREKV_K_CORRECTION_MODE={m}")
    return m


# Ablation knobs of vectorized_joint_correction (attention.py:698-810) that
# change which slots are read or how their scores are formed; none is built
# here, so a non-default value fails loudly instead of being ignored.
# (CAREKV_CHUNKED_CORRECTION only bounds the reference's memory: per-query
# results are unchanged, and this library needs no chunking of that kind.)
_UNBUILT_ROUTE_KNOBS = (
    ("CAREKV_ROUTER_PREFILTER_C", "0"), ("CAREKV_K_QDOTR_CLAMP_PCT", "0"), ("CAREKV_K_NORM_GUARD_PCT", "0"),
    ("CAREKV_RESIDUAL_SCORE", "raw_error"), ("CAREKV_SELECTOR_VARIANT", "current"),
    ("CAREKV_POSITION_POLICY", "none"),
)


def _check_unbuilt_route_knobs() -> None:
    for name, default in _UNBUILT_ROUTE_KNOBS:
        val = os.environ.get(name, default) or default
        try:
            same = float(val) == float(default)
        except ValueError:
            same = val.lower() == default
        if not same:
            raise NotImplementedError(f"{name}={val}: this router ablation (attention.py:698-810) is not built; "
                                      f"unset it (default {default})")


def resolve_route_params(cfg: CacheConfig, layer_id: int, kind: Optional[str] = None,
                         score_normalize: Optional[bool] = None,
                         k_corr_scale: Optional[float] = None, legacy: bool = False) -> "_lib.RouteParams":
    """Budget resolution of residual_router.py:37-76 plus the env knobs of
    vectorized_joint_correction (attention.py:576-957), or, legacy=True, of
    the cached router ResidualRouter.route (residual_router.py:88-452): sketch
    K scores, the route policy (joint / separate / k_first / adaptive), the
    baseline_score ablations and the adaptive_score thresholds."""
    _check_unbuilt_route_knobs()
    if kind is None:
        kind = os.environ.get("CAREKV_PREFILL_RESIDUAL_KIND", "both").lower()
    if kind not in {"v", "k", "both"}:
        raise ValueError(f"Unknown kind={kind}")
    if score_normalize is None:
        score_normalize = os.environ.get("CAREKV_SCORE_NORMALIZE", "0") == "1"
    if k_corr_scale is None:
        k_corr_scale = float(os.environ.get("CAREKV_K_CORRECTION_SCALE", "0.1"))
    lm = layer_budget_multiplier(cfg, layer_id)
    p = _lib.RouteParams()
    p.kind = {"both": _lib.KIND_BOTH, "k": _lib.KIND_K, "v": _lib.KIND_V}[kind]
    p.joint = 1 if cfg.route_policy == "joint" else 0
    p.score_normalize = 1 if score_normalize else 0
    p.kscore_live = 1 if os.environ.get("CAREKV_KSCORE_LIVE", "0") == "1" else 0
    p.exact = 1 if k_correction_mode() == "exact" else 0
    if cfg.read_budget_mode in ("absolute", "adaptive_score"):
        p.budget_mode = 0
        p.read_k = int(round(max(0, int(cfg.read_abs_k)) * lm))
        p.read_v = int(round(max(0, int(cfg.read_abs_v)) * lm))
    else:
        def _r(o, fb):
            return fb if (o is None or o < 0) else o
        p.budget_mode = 1
        p.ratio_k = _r(cfg.read_budget_ratio_k, cfg.read_budget_ratio) * lm
        p.ratio_v = _r(cfg.read_budget_ratio_v, cfg.read_budget_ratio) * lm
    p.k_corr_scale = k_corr_scale
    p.sensitivity = float(cfg.layer_sensitivity[layer_id])
    p.lambda_k = float(os.environ.get("CAREKV_KSCORE_LAMBDA_K", "1") or 1)
    p.lambda_v = float(os.environ.get("CAREKV_KSCORE_LAMBDA_V", "1") or 1)
    if legacy:
        if cfg.baseline_score not in _lib.SCORE:
            raise NotImplementedError(f"baseline_score={cfg.baseline_score!r}: built are {sorted(_lib.SCORE)}")
        if not cfg.store_sketch:
            raise ValueError("the cached router scores K slots from their sketches: CacheConfig(store_sketch=True)")
        p.legacy = 1
        p.kscore_live = 0
        p.joint = 1 if cfg.route_policy == "joint" else 0
        p.policy = _lib.POLICY[cfg.route_policy]
        p.baseline_score = _lib.SCORE[cfg.baseline_score]
        p.adaptive_score = 1 if cfg.read_budget_mode == "adaptive_score" else 0
        p.rel_threshold = float(cfg.read_relative_threshold or 0.0)
        p.abs_threshold = float(cfg.read_absolute_threshold or 0.0)
        p.min_keep = int(cfg.read_min_keep or 0)
    return p


def legacy_router(cfg: CacheConfig) -> bool:
    """Does a correction of this configuration take the reference's cached
    router?  The reference's prefill correction does unless correction_impl is
    "vectorized" (layer.py:522-630).  (Its decode step always does,
    attention.py:1025; this library's decode runs the vectorized router
    unless CAREKV_DECODE_ROUTER=cached.)"""
    return cfg.correction_impl != "vectorized"


def any_read_budget(cfg: CacheConfig) -> bool:
    """layer.py:359-365: does any positive read budget exist?"""
    return bool((cfg.read_budget_mode in ("absolute", "adaptive_score")
                 and (cfg.read_abs_k > 0 or cfg.read_abs_v > 0))
                or cfg.read_budget_ratio > 0
                or (cfg.read_budget_ratio_k or 0) > 0
                or (cfg.read_budget_ratio_v or 0) > 0)
