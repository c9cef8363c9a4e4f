"""GPU decode path against the oracle on seeded inputs: configurations the
reference supports (INT2/3/4, head_dim 64/128, GQA groups 1/2/4/8, fp32 /
fp16 / bf16 activations, absolute and ratio budgets, joint and separate
routing, combined_kvscore and sketch proxy, exact and linear K correction),
ragged batches, page boundaries, edge cases, and a full-context sample."""

import math

import zlib

import numpy as np
import pytest
import torch

import oracle
from conftest import load_pkg
from helpers import (PAPER_BEST_ENV, compare_cache_state, env, oracle_cache_for, oracle_selection,
                     route_cfg_from, saturated_attention, selection_margin)

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 2e-3
TDT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


@pytest.fixture(scope="module")
def pkg():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_pkg()


def _inputs(rng, H, T, D, dt, outliers=True):
    K = rng.standard_normal((H, T, D)).astype(np.float32)
    if outliers:
        K[:, :, :4] *= 20.0
    V = rng.standard_normal((H, T, D)).astype(np.float32)
    return oracle.round_to(K, dt), oracle.round_to(V, dt)


def _check_step(pkg, eng, oc, cfg, q_np, dt, seqs, layer=0, correction=True):
    """Run attend on all sequences and compare every (seq, kv head) with the oracle."""
    H, D = cfg.num_kv_heads, cfg.head_dim
    grp = cfg.num_heads // H
    q = torch.from_numpy(q_np).cuda().to(TDT[dt])
    pages = max(eng._pages(b, layer) for b in range(len(seqs)))
    out = eng.attend(layer, q, correction=correction, pages=pages).float().cpu().numpy()
    sel = eng.last_selection(layer, 0, len(seqs), pages) if correction else None
    rc = route_cfg_from(cfg)
    for b, ocb in enumerate(seqs):
        for h in range(H):
            qh = oracle.round_to(q_np[b, h * grp:(h + 1) * grp], dt)
            O, info = oracle.decode_attention_kvh(ocb, layer, h, qh, rc, correction=correction,
                                                  sketch_P=ocb.sketch_P)
            tol = {"fp32": (RTOL, ATOL), "fp16": (3e-3, 3e-3), "bf16": (1e-2, 1e-2)}[dt]
            np.testing.assert_allclose(out[b, h * grp:(h + 1) * grp], oracle.round_to(O, dt),
                                       rtol=tol[0], atol=tol[1], err_msg=f"seq {b} kv head {h}")
            if correction and info is not None and "sel_k" in info:
                want = oracle_selection(info, grp)
                for i in range(grp):
                    got = sorted(sel[(b, h, i)])
                    if got != want[i]:
                        m = selection_margin(info, i)
                        assert m < 1e-5 or saturated_attention(info, i), (b, h, i, got, want[i], m)


CASES = [
    # name, D, bits, g, Hq, Hkv, dt, T(prefill), steps, store(k,v), read mode, read(k,v)/ratio, policy, live, kmode, kind
    ("int3_d128_mha_bf16", 128, 3, 32, 2, 2, "bf16", 100, 20, (1, 1), "ratio", 0.03, "joint", True, "exact", "both"),
    ("int3_d64_gqa8_fp16", 64, 3, 32, 16, 2, "fp16", 77, 24, (2, 4), "absolute", (2, 4), "joint", True, "exact", "both"),
    ("int2_d128_gqa4_fp32", 128, 2, 32, 8, 2, "fp32", 64, 17, (2, 2), "absolute", (2, 2), "joint", True, "exact", "both"),
    ("int4_d128_g64_gqa2", 128, 4, 64, 4, 2, "fp32", 50, 15, (1, 2), "absolute", (1, 2), "separate", True, "exact", "both"),
    ("proxy_linear", 64, 3, 32, 8, 2, "fp32", 90, 10, (2, 2), "absolute", (2, 2), "joint", False, "linear", "both"),
    ("kind_v_exact", 64, 3, 32, 4, 1, "fp16", 40, 8, (2, 4), "absolute", (2, 4), "joint", True, "exact", "v"),
    ("kind_k_linear", 128, 3, 32, 8, 1, "fp32", 48, 8, (2, 4), "absolute", (3, 0), "joint", True, "linear", "k"),
    ("ratio_gqa8_d64", 64, 3, 32, 32, 4, "fp32", 512, 4, (1, 1), "ratio", 0.03, "joint", True, "exact", "both"),
    ("int4_d64_mha_fp16", 64, 4, 32, 3, 3, "fp16", 70, 12, (1, 1), "absolute", (2, 2), "joint", True, "exact", "both"),
    ("int4_d128_g64_mha_bf16", 128, 4, 64, 2, 2, "bf16", 96, 10, (1, 1), "ratio", 0.05, "joint", True, "exact", "both"),
    # one query head per kv head at the fp32 tolerance (V scales carried by the P operand)
    ("int3_d128_mha_fp32", 128, 3, 32, 4, 4, "fp32", 150, 20, (1, 1), "absolute", (2, 2), "joint", True, "exact", "both"),
    ("int3_d64_mha_fp32_g64", 64, 3, 64, 3, 3, "fp32", 61, 9, (2, 2), "absolute", (2, 3), "joint", True, "linear", "both"),
    ("int4_d128_mha_fp32", 128, 4, 32, 2, 2, "fp32", 83, 6, (1, 2), "ratio", 0.05, "separate", True, "exact", "both"),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_decode_matches_oracle(pkg, case):
    name, D, bits, g, Hq, Hkv, dt, T, steps, (sk, sv), rmode, rb, policy, live, kmode, kind = case
    rng = np.random.default_rng(zlib.crc32(name.encode()))   # stable across processes
    e = dict(PAPER_BEST_ENV, CAREKV_KSCORE_LIVE="1" if live else "0", CAREKV_K_CORRECTION_MODE=kmode,
             CAREKV_PREFILL_RESIDUAL_KIND=kind)
    read = dict(read_budget_mode=rmode)
    if rmode == "ratio":
        read["read_budget_ratio"] = rb
    else:
        read.update(read_abs_k=rb[0], read_abs_v=rb[1], read_budget_ratio=0.0)
    B = 2
    with env(**e):
        cfg = pkg.CacheConfig(num_layers=1, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, page_size=16,
                              max_pages=(T + steps) // 16 + 2, base_bits=bits, group_size=g, scale_quant="int8",
                              store_budget_mode="absolute", store_abs_k=sk, store_abs_v=sv, route_policy=policy,
                              sketch_dim=32, store_sketch=not live, **read)
        cache = pkg.CAREKVCache(cfg, torch.device("cuda"), batch=B)
        eng = pkg.DecodeEngine(cache)
        seqs = []
        for b in range(B):
            Tb = T - 7 * b                     # ragged batch
            K, V = _inputs(rng, Hkv, Tb, D, dt)
            eng.prefill_store(0, torch.from_numpy(K).cuda().to(TDT[dt])[None],
                              torch.from_numpy(V).cuda().to(TDT[dt])[None], seq_begin=b)
            oc = oracle_cache_for(cfg)
            for h in range(Hkv):
                oc.prefill_write(0, h, K[h], V[h], dt)
            seqs.append(oc)
        for step in range(steps):
            k = oracle.round_to(rng.standard_normal((B, Hkv, D)).astype(np.float32), dt)
            v = oracle.round_to(rng.standard_normal((B, Hkv, D)).astype(np.float32), dt)
            eng.append(0, torch.from_numpy(k).cuda().to(TDT[dt]), torch.from_numpy(v).cuda().to(TDT[dt]))
            for b, oc in enumerate(seqs):
                pos = int(oc.valid[0, 0, :oc.next_page[0, 0]].sum())
                for h in range(Hkv):
                    oc.append(0, h, k[b, h], v[b, h], dt, pos_abs=pos)
            q = rng.standard_normal((B, Hq, D)).astype(np.float32)
            _check_step(pkg, eng, None, cfg, q, dt, seqs)
        torch.cuda.synchronize()
        for b, oc in enumerate(seqs):
            compare_cache_state(cache, oc, b, 0, check_sketch=not live)
        cache.check_errors()


def test_empty_cache_and_read_budget_zero(pkg):
    with env(**PAPER_BEST_ENV):
        cfg = pkg.CacheConfig(num_layers=2, num_heads=8, num_kv_heads=2, head_dim=64, max_pages=8, base_bits=3,
                              group_size=32, scale_quant="int8", store_budget_mode="absolute", store_abs_k=2,
                              store_abs_v=2, read_budget_mode="absolute", read_abs_k=0, read_abs_v=0,
                              route_policy="joint")
        cache = pkg.CAREKVCache(cfg, torch.device("cuda"), batch=1)
        eng = pkg.DecodeEngine(cache)
        q = torch.randn(1, 8, 64, device="cuda")
        # no tokens yet: the reference returns zeros (attention.py:993-994)
        assert torch.count_nonzero(eng.attend(1, q, pages=1)) == 0
        K = torch.randn(1, 2, 45, 64, device="cuda")
        eng.prefill_store(0, K, torch.randn_like(K))
        # READ=0 is bit-identical to base attention (layer.py:366-370)
        a = eng.attend(0, q)
        b = eng.attend(0, q, correction=False)
        assert torch.equal(a, b)
        assert cache.read_counters() == (0, 0)


def test_cache_full_is_reported_on_the_host(pkg):
    cfg = pkg.CacheConfig(num_layers=1, num_heads=2, num_kv_heads=2, head_dim=64, max_pages=8, base_bits=3,
                          group_size=32, scale_quant="int8", store_budget_mode="absolute", store_abs_k=1,
                          store_abs_v=1)
    cache = pkg.CAREKVCache(cfg, torch.device("cuda"), batch=1)
    eng = pkg.DecodeEngine(cache)
    K = torch.randn(1, 2, 8 * 16, 64, device="cuda")
    eng.prefill_store(0, K, K.clone())
    with pytest.raises(pkg._lib.CacheFullError):
        eng.append(0, torch.randn(1, 2, 64, device="cuda"), torch.randn(1, 2, 64, device="cuda"))
    with pytest.raises(pkg._lib.CacheFullError):
        eng.prefill_store(0, K[:, :, :1], K[:, :, :1])
    cache.check_errors()


def test_full_context_sampled_against_oracle(pkg):
    """Config-3 shape (head_dim 128, MHA, 4096-token context, bf16, INT3 g32,
    3% store and read budgets) on a few sequences; sampled kv heads are
    replayed through the oracle."""
    B, H, D, N = 2, 32, 128, 4096
    with env(**PAPER_BEST_ENV):
        cfg = pkg.CacheConfig(num_layers=1, num_heads=H, num_kv_heads=H, head_dim=D, max_pages=N // 16 + 8,
                              base_bits=3, group_size=32, scale_quant="int8", packed_base=True,
                              store_budget_mode="absolute", store_abs_k=1, store_abs_v=1,
                              read_budget_mode="ratio", read_budget_ratio=0.03, route_policy="joint")
        cache = pkg.CAREKVCache(cfg, torch.device("cuda"), batch=B)
        eng = pkg.DecodeEngine(cache)
        g = torch.Generator(device="cuda").manual_seed(0)
        K = torch.randn(B, H, N, D, device="cuda", generator=g)
        K[..., :4] *= 20
        K = K.to(torch.bfloat16)
        V = torch.randn(B, H, N, D, device="cuda", generator=g).to(torch.bfloat16)
        eng.prefill_store(0, K, V)
        kn = torch.randn(B, H, D, device="cuda", generator=g).to(torch.bfloat16)
        vn = torch.randn(B, H, D, device="cuda", generator=g).to(torch.bfloat16)
        eng.append(0, kn, vn)
        q = torch.randn(B, H, D, device="cuda", generator=g).to(torch.bfloat16)
        pages = eng._pages(0, 0)
        out = eng.attend(0, q, pages=pages).float().cpu().numpy()
        sel = eng.last_selection(0, 0, B, pages)
        assert np.isfinite(out).all()
        rc = route_cfg_from(cfg)
        Kc, Vc, knc, vnc, qc = (t.float().cpu().numpy() for t in (K, V, kn, vn, q))
        for (b, h) in ((0, 0), (1, 17), (0, 31)):
            oc = oracle_cache_for(cfg, num_layers=1)
            oc.H = 1
            oc.__init__(1, 1, D, cfg.padded_max_pages, oc.cfg, scale_quant="int8")
            oc.prefill_write(0, 0, Kc[b, h], Vc[b, h], "bf16")
            oc.append(0, 0, knc[b, h], vnc[b, h], "bf16", pos_abs=N)
            O, info = oracle.decode_attention_kvh(oc, 0, 0, qc[b, h:h + 1], rc)
            np.testing.assert_allclose(out[b, h], oracle.round_to(O, "bf16")[0], rtol=1e-2, atol=1e-2)
            want = oracle_selection(info, 1)[0]
            got = sorted(sel[(b, h, 0)])
            if got != want:
                assert selection_margin(info, 0) < 1e-5, (b, h, got, want)
