"""CPU-only checks of the C ABI library and the host-side policy resolution.

No kernel runs here: the library is dlopen'ed (it needs no GPU to load),
every symbol the header declares must be exported, and the pure-host
entry points (layout, validation, status strings) are exercised.
"""

import ctypes
import os
import re

import pytest

from conftest import ROOT, load_pkg

import oracle
from oracle.attention import resolve_read_budgets
from oracle.store import store_budgets
from helpers import env, route_cfg_from, store_cfg_from

HEADER = os.path.join(ROOT, "include", "carekv_b200.h")


def _lib():
    pkg = load_pkg()
    return pkg, pkg._lib.load()


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(carekv_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    pkg, lib = _lib()
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/carekv_b200.h but not exported"
    bound = {s[0] for s in pkg._lib.SIGNATURES}
    assert bound == set(names), "ctypes bindings and header disagree"
    assert lib.carekv_abi_version() == 2


def test_status_strings():
    _, lib = _lib()
    assert lib.carekv_status_string(0) == b"ok"
    assert lib.carekv_status_string(3) == b"KV cache is full"
    assert lib.carekv_status_string(99) == b"unknown status"


def _cfg(pkg, **kw):
    base = dict(num_layers=2, num_heads=8, num_kv_heads=2, head_dim=128, page_size=16, max_pages=16,
                base_bits=3, group_size=32, scale_quant="int8", store_budget_mode="absolute",
                store_abs_k=2, store_abs_v=4, read_budget_mode="absolute", read_abs_k=2, read_abs_v=4)
    base.update(kw)
    return pkg.CacheConfig(**base)


def test_cache_layout_sizes():
    pkg, lib = _lib()
    cfg = _cfg(pkg, store_sketch=True)
    c = cfg.c_config()
    sizes = (ctypes.c_size_t * pkg._lib.NUM_BUFFERS)()
    assert lib.carekv_cache_layout(ctypes.byref(c), 3, sizes) == 0
    B, L, H, P, T, D = 3, 2, 2, 16, 16, 128
    pages = B * L * H * P
    exp = dict(k_codes=pages * T * 48, k_scale=pages * T * 4, k_master=pages * 2, valid=pages * 4,
               num_pages=B * L * H * 4, k_slot_group=pages * 2, k_slot_data=pages * 2 * 256,
               v_slot_data=pages * 4 * 256, k_err=pages * 4 * 2, v_err=pages * 4 * 2,
               k_sketch=pages * 4 * 32 * 2, slot_counter=B * 8, read_counter=L * H * 16, error_flag=4)
    got = dict(zip(pkg._lib.CACHE_PTR_FIELDS, list(sizes)))
    for k, v in exp.items():
        assert got[k] == v, (k, got[k], v)


@pytest.mark.parametrize("field,value,status", [
    ("head_dim", 96, 2), ("page_size", 8, 2), ("max_pages", 12, 1), ("base_bits", 5, 1),
    ("group_size", 24, 1), ("k_channel_group", 16, 2), ("residual_bits", 8, 2),
    ("k_slots_per_page", 9, 1), ("num_heads", 12, 2),
])
def test_config_validation(field, value, status):
    pkg, lib = _lib()
    c = _cfg(pkg).c_config()
    setattr(c, field, value)
    sizes = (ctypes.c_size_t * pkg._lib.NUM_BUFFERS)()
    assert lib.carekv_cache_layout(ctypes.byref(c), 1, sizes) == status


def test_null_cache_is_rejected_without_touching_the_gpu():
    pkg, lib = _lib()
    c = _cfg(pkg).c_config()
    empty = pkg._lib.Cache()
    empty.batch = 1
    assert lib.carekv_cache_init(ctypes.byref(c), ctypes.byref(empty), None) == 1
    assert lib.carekv_quantize(None, None, None, 4, 128, 3, 32, 0, None) == 1


def test_misaligned_cache_buffer_is_rejected_without_touching_the_gpu():
    # every buffer must start on a 16-byte boundary (the kernels stage rows
    # and slots with 16-byte and bulk copies); the check runs before any
    # CUDA call, so fake addresses are enough
    pkg, lib = _lib()
    c = _cfg(pkg).c_config()
    cache = pkg._lib.Cache()
    cache.batch = 1
    names = [n for n, _ in pkg._lib.Cache._fields_ if n != "batch"]
    for i, n in enumerate(names):
        setattr(cache, n, 0x10000 * (i + 1))
    cache.v_scale = 0x10000 * 100 + 8   # 8-byte aligned only: rejected before any launch or copy
    assert lib.carekv_cache_init(ctypes.byref(c), ctypes.byref(cache), None) == 1


def test_cache_config_validation_mirrors_reference():
    pkg = load_pkg()
    with pytest.raises(ValueError, match="scale_dtype"):
        pkg.CacheConfig(scale_dtype="fp8")
    with pytest.raises(ValueError, match="route_policy"):
        pkg.CacheConfig(route_policy="greedy")
    c = pkg.CacheConfig(num_heads=8)
    assert c.num_kv_heads == 8 and c.layer_sensitivity == [1.0] * 32


@pytest.mark.parametrize("mode,sk,sv,ratio,policy,kind", [
    ("absolute", 2, 4, 0.0, "residual_kind_aware", "both"),
    ("absolute", 1, 1, 0.0, "residual_kind_aware", "v"),
    ("ratio", 0, 0, 0.1, "residual_kind_aware", "both"),
    ("ratio", 0, 0, 0.25, "joint", "both"),
    ("ratio", 0, 0, 0.0, "per_kind", "both"),
])
def test_store_budget_resolution_matches_oracle(mode, sk, sv, ratio, policy, kind):
    pkg = load_pkg()
    with env(CAREKV_STORE_POLICY=policy, CAREKV_PREFILL_RESIDUAL_KIND=kind):
        cfg = _cfg(pkg, store_budget_mode=mode, store_abs_k=sk, store_abs_v=sv, store_budget_ratio=ratio)
        sp = pkg.resolve_store_params(cfg, 0, 0)
        kb, vb, joint, nothing = store_budgets(store_cfg_from(cfg), cfg.num_k_groups, cfg.num_v_blocks)
    assert sp.k_budget == kb and sp.v_budget == vb
    assert sp.store_nothing == int(nothing)
    assert sp.joint_budget == (joint if policy == "joint" and not nothing else 0)


@pytest.mark.parametrize("mode,rk,rv,ratio,n_k,n_v", [
    ("absolute", 2, 4, 0.0, 40, 80), ("absolute", 9, 9, 0.0, 3, 5), ("ratio", 0, 0, 0.03, 32, 32),
    ("ratio", 0, 0, 0.03, 100, 100), ("adaptive_score", 3, 1, 0.0, 10, 10),
])
def test_read_budget_resolution_matches_oracle(mode, rk, rv, ratio, n_k, n_v):
    """The device resolves ratio budgets with the same double arithmetic."""
    pkg = load_pkg()
    cfg = _cfg(pkg, read_budget_mode=mode, read_abs_k=rk, read_abs_v=rv, read_budget_ratio=ratio)
    rp = pkg.resolve_route_params(cfg, 0, kind="both")
    bk, bv = resolve_read_budgets(route_cfg_from(cfg), n_k, n_v)
    if rp.budget_mode == 0:
        got = (min(rp.read_k, n_k), min(rp.read_v, n_v))
    else:
        got = (min(max(1, int(n_k * rp.ratio_k)) if rp.ratio_k > 0 else 0, n_k),
               min(max(1, int(n_v * rp.ratio_v)) if rp.ratio_v > 0 else 0, n_v))
    assert got == (bk, bv)


def test_layer_budget_multiplier_u_shape():
    pkg = load_pkg()
    cfg = _cfg(pkg, num_layers=5, budget_policy="u_shaped")
    m = [pkg.layer_budget_multiplier(cfg, l) for l in range(5)]
    assert abs(sum(m) / 5 - 1.0) < 1e-12 and m[0] == m[4] > m[2]


@pytest.mark.parametrize("knob,value", [("CAREKV_ROUTER_PREFILTER_C", "8"), ("CAREKV_K_QDOTR_CLAMP_PCT", "99"),
                                        ("CAREKV_K_NORM_GUARD_PCT", "95"),
                                        ("CAREKV_RESIDUAL_SCORE", "attention_output"),
                                        ("CAREKV_SELECTOR_VARIANT", "random"), ("CAREKV_POSITION_POLICY", "recent")])
def test_unbuilt_router_ablations_fail_loudly(knob, value):
    pkg = load_pkg()
    cfg = pkg.CacheConfig(num_layers=1, num_heads=4, num_kv_heads=2, head_dim=64, max_pages=4)
    with env(**{knob: value}):
        with pytest.raises(NotImplementedError, match=knob):
            pkg.resolve_route_params(cfg, 0)
    with env(**{knob: None}):
        pkg.resolve_route_params(cfg, 0)      # default: accepted


def test_decode_page_master_flag_resolution():
    """CAREKV_DECODE_PAGE_MASTER reaches carekv_store_params_t (default 0 =
    the reference's master-0 decode pages, cache.py:689-695)."""
    pkg = load_pkg()
    cfg = pkg.CacheConfig(num_layers=1, num_heads=4, num_kv_heads=2, head_dim=64, max_pages=4)
    with env(CAREKV_DECODE_PAGE_MASTER=None):
        assert pkg.resolve_store_params(cfg, 0, 0).decode_page_master == 0
    with env(CAREKV_DECODE_PAGE_MASTER="1"):
        assert pkg.resolve_store_params(cfg, 0, 0).decode_page_master == 1
    fields = [f for f, _ in pkg._lib.StoreParams._fields_]
    hdr = open(os.path.join(ROOT, "include", "carekv_b200.h")).read()
    body = hdr[hdr.index("typedef struct carekv_store_params"):hdr.index("} carekv_store_params_t;")]
    assert re.findall(r"int32_t\s+(\w+);|float\s+(\w+);", body) and \
        [a or b for a, b in re.findall(r"int32_t\s+(\w+);|float\s+(\w+);", body)] == fields
