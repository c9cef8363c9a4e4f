"""Shared helpers for the parity tests: build the same cache state in the
CPU oracle and in the GPU arena, and read GPU state back in oracle layout."""

import contextlib
import math
import os

import numpy as np

import oracle
from oracle import OracleCache, RouteConfig, StoreConfig

PAPER_BEST_ENV = dict(
    CAREKV_K_CORRECTION_MODE="exact", CAREKV_KSCORE_LIVE="1", CAREKV_SCORE_NORMALIZE="1",
    CAREKV_PREFILL_RESIDUAL_KIND="both", CAREKV_STORE_POLICY="residual_kind_aware",
)

DT_NAME = {"fp32": "float32", "fp16": "float16", "bf16": "bfloat16"}


@contextlib.contextmanager
def env(**kw):
    old = {k: os.environ.get(k) for k in kw}
    try:
        for k, v in kw.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = str(v)
        yield
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def store_cfg_from(cfg):
    """oracle StoreConfig equivalent of a package CacheConfig + current env."""
    return StoreConfig(
        head_dim=cfg.head_dim, page_size=cfg.page_size, base_bits=cfg.base_bits, group_size=cfg.group_size,
        k_channel_group=cfg.k_channel_group, v_token_block=cfg.v_token_block, sketch_dim=cfg.sketch_dim,
        store_budget_mode=cfg.store_budget_mode, store_abs_k=cfg.store_abs_k, store_abs_v=cfg.store_abs_v,
        store_budget_ratio=cfg.store_budget_ratio, store_budget_ratio_k=cfg.store_budget_ratio_k,
        store_budget_ratio_v=cfg.store_budget_ratio_v,
        store_policy=os.environ.get("CAREKV_STORE_POLICY", "residual_kind_aware"),
        residual_kind=os.environ.get("CAREKV_PREFILL_RESIDUAL_KIND", "both"))


def route_cfg_from(cfg):
    return RouteConfig(
        head_dim=cfg.head_dim, page_size=cfg.page_size, k_channel_group=cfg.k_channel_group,
        v_token_block=cfg.v_token_block, sketch_dim=cfg.sketch_dim,
        kind=os.environ.get("CAREKV_PREFILL_RESIDUAL_KIND", "both"),
        route_policy="joint" if cfg.route_policy == "joint" else "separate",
        score_normalize=os.environ.get("CAREKV_SCORE_NORMALIZE", "0") == "1",
        kscore_live=os.environ.get("CAREKV_KSCORE_LIVE", "0") == "1",
        k_correction_mode=os.environ.get("CAREKV_K_CORRECTION_MODE", "linear"),
        k_corr_scale=float(os.environ.get("CAREKV_K_CORRECTION_SCALE", "0.1")),
        read_budget_mode=cfg.read_budget_mode, read_abs_k=cfg.read_abs_k, read_abs_v=cfg.read_abs_v,
        read_budget_ratio=cfg.read_budget_ratio, read_budget_ratio_k=cfg.read_budget_ratio_k,
        read_budget_ratio_v=cfg.read_budget_ratio_v)


def oracle_cache_for(cfg, num_layers=None):
    return OracleCache(num_layers or cfg.num_layers, cfg.num_kv_heads, cfg.head_dim,
                       cfg.padded_max_pages, store_cfg_from(cfg), page_size=cfg.page_size,
                       scale_quant=cfg.scale_quant, scale_dtype=cfg.scale_dtype)


def oracle_selection(info, qn):
    """{query: sorted [(kind, page, group)]} from an oracle correction info dict."""
    out = {}
    for i in range(qn):
        items = []
        if info.get("sel_k") is not None:
            for si in np.nonzero(info["sel_k"][i])[0]:
                e = info["k_index"][si]
                items.append(("K", e["page"], e["cg"]))
        if info.get("sel_v") is not None:
            for j in np.nonzero(info["sel_v"][i])[0]:
                e = info["v_index"][j]
                items.append(("V", e["page"], e["vb"]))
        out[i] = sorted(items)
    return out


def compare_cache_state(gpu_cache, oc, b, layer, check_sketch=False, err_ulps=True):
    """Assert the GPU arena's (sequence b, layer) equals the oracle's state."""
    import torch
    H = oc.H
    valid = gpu_cache.view("valid")[b, layer].cpu().numpy()
    assert np.array_equal(valid, oc.valid[layer]), "valid tokens"
    npg = gpu_cache.view("num_pages")[b, layer].cpu().numpy()
    assert np.array_equal(npg, oc.next_page[layer]), "page counts"
    kc = gpu_cache.view("k_codes")[b, layer].cpu().numpy()
    vc = gpu_cache.view("v_codes")[b, layer].cpu().numpy()
    for h in range(H):
        for p in range(int(npg[h])):
            n = int(valid[h, p])
            # rows past the valid count of a prefill page are padding (their
            # fp16 codes come from 0/0); compare the valid rows bit for bit
            assert np.array_equal(kc[h, p, :n], oc.k_codes[layer, h, p, :n]), ("K codes", h, p)
            assert np.array_equal(vc[h, p, :n], oc.v_codes[layer, h, p, :n]), ("V codes", h, p)
    if oc.scale_quant == "int8":
        ks = gpu_cache.view("k_scale")[b, layer].cpu().numpy()
        vs = gpu_cache.view("v_scale")[b, layer].cpu().numpy()
        km = gpu_cache.view("k_master")[b, layer].float().cpu().numpy()
        vm = gpu_cache.view("v_master")[b, layer].float().cpu().numpy()
        for h in range(H):
            for p in range(int(npg[h])):
                n = int(valid[h, p])
                assert np.array_equal(ks[h, p, :n], oc.k_scale[layer, h, p, :n]), ("K scale codes", h, p)
                assert np.array_equal(vs[h, p, :n], oc.v_scale[layer, h, p, :n]), ("V scale codes", h, p)
                assert km[h, p] == oc.k_master[layer, h, p], ("K master", h, p)
                assert vm[h, p] == oc.v_master[layer, h, p], ("V master", h, p)
    else:
        ks = gpu_cache.view("k_scale")[b, layer].float().cpu().numpy()
        for h in range(H):
            for p in range(int(npg[h])):
                n = int(valid[h, p])
                assert np.array_equal(ks[h, p, :n], oc.k_scale[layer, h, p, :n]), ("K scales", h, p)
    # residual slots: ids per page and payloads by id
    kdata = gpu_cache.view("k_slot_data")
    vdata = gpu_cache.view("v_slot_data")
    kdata = kdata[b, layer].cpu().numpy() if kdata is not None else None
    vdata = vdata[b, layer].cpu().numpy() if vdata is not None else None
    kscale = gpu_cache.view("k_slot_scale")
    vscale = gpu_cache.view("v_slot_scale")
    kgrp = gpu_cache.view("k_slot_group")
    vblk = gpu_cache.view("v_slot_block")
    for h in range(H):
        for p in range(int(npg[h])):
            om = oc.meta[layer][h][p]
            gm = gpu_cache.page_meta(layer, h, p, seq=b)
            if om is None:
                assert all(x < 0 for x in gm.k_residual_slots) and all(x < 0 for x in gm.v_residual_slots)
                continue
            assert gm.k_residual_slots == om["k_slots"], ("K slot ids", h, p, gm.k_residual_slots, om["k_slots"])
            assert gm.v_residual_slots == om["v_slots"], ("V slot ids", h, p, gm.v_residual_slots, om["v_slots"])
            np.testing.assert_allclose(gm.k_error_norm.float().cpu().numpy(), om["k_err"], rtol=1e-3, atol=1e-7)
            np.testing.assert_allclose(gm.v_error_norm.float().cpu().numpy(), om["v_err"], rtol=1e-3, atol=1e-7)
            if check_sketch and gm.k_sketch is not None:
                np.testing.assert_allclose(gm.k_sketch.float().cpu().numpy(), om["k_sketch"], rtol=2e-3, atol=1e-5)
            if kdata is not None and kgrp is not None:
                g = kgrp[b, layer, h, p].cpu().numpy()
                for j, cg in enumerate(g):
                    if cg < 0:
                        continue
                    sid = om["k_slots"][cg]
                    packed, sc = oc.k_slots[sid]
                    assert np.array_equal(kdata[h, p, j], packed), ("K payload", h, p, cg)
                    assert float(kscale[b, layer, h, p, j].float().item()) == float(sc), ("K slot scale", h, p)
            if vdata is not None and vblk is not None:
                g = vblk[b, layer, h, p].cpu().numpy()
                for j, vb in enumerate(g):
                    if vb < 0:
                        continue
                    sid = om["v_slots"][vb]
                    packed, sc = oc.v_slots[sid]
                    assert np.array_equal(vdata[h, p, j], packed), ("V payload", h, p, vb)
                    assert float(vscale[b, layer, h, p, j].float().item()) == float(sc), ("V slot scale", h, p)


def saturated_attention(info, q, eps=1e-4):
    """True when query q's attention is saturated in fp32 (1 - max A < eps).

    combined_kvscore weighs every token by A(1 - A); for the dominant token of
    such a query 1 - A sits at the rounding level of fp32 (one ulp of 1.0 is
    6e-8), so the K score of its page is rounding noise in the reference as in
    any other fp32 evaluation, and the selection among the slots it competes
    with is not determined by the algorithm."""
    A = info.get("A")
    if A is None:
        return False
    return 1.0 - float(np.max(A[q])) < eps


def selection_margin(info, q, qn_total=None):
    """Gap between the last selected and the first unselected normalised
    score of query q (joint list), for tie-aware selection checks."""
    parts = []
    if info.get("score_K_r") is not None:
        parts.append(info["score_K_r"][q])
    if info.get("score_V_r") is not None:
        parts.append(info["score_V_r"][q])
    if not parts:
        return math.inf
    s = np.sort(np.concatenate(parts))[::-1]
    k = (info["budget_k"] + info["budget_v"])
    if k <= 0 or k >= s.size:
        return math.inf
    return float(s[k - 1] - s[k]) / max(abs(float(s[k - 1])), 1e-30)


def classify_selection(got, want, info, q, tie_margin=1e-5):
    """Compare one query's selected (kind, page, group) set with the oracle's.

    Returns "equal" for identical sets, "tie" when they differ only where
    the normalised scores at the cut are within tie_margin (a tie within
    fp32 accumulation order), "saturated" when they differ on a query whose
    attention is saturated in fp32 (saturated_attention), and "mismatch"
    otherwise."""
    if sorted(got) == sorted(want):
        return "equal"
    if selection_margin(info, q) < tie_margin:
        return "tie"
    if saturated_attention(info, q):
        return "saturated"
    return "mismatch"


def compare_kivi_state(gpu_cache, oc, b, layer, check_payloads=True):
    """KIVI base: the GPU arena's (sequence b, layer) against the oracle's
    fp16 side buffers (bit for bit, NaN where the reference has NaN), valid
    counts and residual slots."""
    import torch
    valid = gpu_cache.view("valid")[b, layer].cpu().numpy()
    assert np.array_equal(valid, oc.valid[layer]), "valid tokens"
    npg = gpu_cache.view("num_pages")[b, layer].cpu().numpy()
    assert np.array_equal(npg, oc.next_page[layer]), "page counts"
    for h in range(oc.H):
        Kg, Vg, lens = gpu_cache.read_base_hat_concat(layer, h, seq=b)
        Ko, Vo, lens_o = oc.read_base_concat(layer, h)
        assert lens == lens_o, ("valid lengths", h)
        np.testing.assert_array_equal(Kg.float().cpu().numpy(), Ko, err_msg=f"K_hat kv head {h}")
        np.testing.assert_array_equal(Vg.float().cpu().numpy(), Vo, err_msg=f"V_hat kv head {h}")
    kdata, vdata = gpu_cache.view("k_slot_data"), gpu_cache.view("v_slot_data")
    kgrp, vblk = gpu_cache.view("k_slot_group"), gpu_cache.view("v_slot_block")
    for h in range(oc.H):
        for p in range(int(npg[h])):
            om = oc.meta[layer][h][p]
            gm = gpu_cache.page_meta(layer, h, p, seq=b)
            if om is None:
                continue
            assert gm.k_residual_slots == om["k_slots"], ("K slot ids", h, p, gm.k_residual_slots, om["k_slots"])
            assert gm.v_residual_slots == om["v_slots"], ("V slot ids", h, p, gm.v_residual_slots, om["v_slots"])
            np.testing.assert_allclose(gm.k_error_norm.float().cpu().numpy(), om["k_err"], rtol=1e-3, atol=1e-7)
            np.testing.assert_allclose(gm.v_error_norm.float().cpu().numpy(), om["v_err"], rtol=1e-3, atol=1e-7)
            if not check_payloads:
                continue
            if kdata is not None:
                for j, cg in enumerate(kgrp[b, layer, h, p].cpu().numpy()):
                    if cg >= 0:
                        assert np.array_equal(kdata[b, layer, h, p, j].cpu().numpy(), oc.k_slots[om["k_slots"][cg]][0])
            if vdata is not None:
                for j, vb in enumerate(vblk[b, layer, h, p].cpu().numpy()):
                    if vb >= 0:
                        assert np.array_equal(vdata[b, layer, h, p, j].cpu().numpy(), oc.v_slots[om["v_slots"][vb]][0])
