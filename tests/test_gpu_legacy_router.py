"""The cached router (correction_impl "python" / "cached"): decode attention
with ResidualRouter.route (residual_router.py:88-452) and
apply_slot_corrections (attention.py:208-374) per query head, against the
oracle restatement (oracle/legacy_router.py, pinned to the reference by
tests/golden/legacy_router.npz): the joint / separate / k_first / adaptive
policies, the baseline_score ablations, the adaptive_score thresholds,
exact and linear corrections, ratio and absolute budgets.  Selections must
equal the oracle's except where the two best-excluded / worst-included
scores tie within 1e-5 (relative)."""

import zlib

import numpy as np
import pytest
import torch

import oracle
from oracle.legacy_router import legacy_correction, legacy_route
from conftest import load_pkg
from helpers import PAPER_BEST_ENV, env, oracle_cache_for

pytestmark = pytest.mark.gpu
TDT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}

CASES = [
    # name, D, Hq, Hkv, dt, T, store (k, v), read mode, rk, rv, ratio, policy, normalize, kmode, kind, baseline,
    # rel, abs, min_keep
    ("joint_norm_exact", 64, 4, 2, "fp32", 150, (2, 2), "absolute", 2, 2, 0.0, "joint", True, "exact", "both",
     "carekv", 0.0, 0.0, 0),
    ("separate_linear_d128", 128, 2, 2, "fp32", 130, (2, 2), "absolute", 2, 3, 0.0, "separate", False, "linear",
     "both", "carekv", 0.0, 0.0, 0),
    ("k_first_exact", 64, 4, 2, "fp32", 150, (2, 2), "absolute", 2, 3, 0.0, "k_first", True, "exact", "both",
     "carekv", 0.0, 0.0, 0),
    ("adaptive_exact", 64, 4, 2, "fp32", 150, (2, 2), "absolute", 3, 3, 0.0, "adaptive", True, "exact", "both",
     "carekv", 0.0, 0.0, 0),
    ("adaptive_score", 64, 4, 2, "fp32", 150, (2, 2), "adaptive_score", 3, 3, 0.0, "separate", True, "exact",
     "both", "carekv", 0.3, 0.0, 1),
    ("magnitude_only", 64, 4, 2, "fp32", 120, (2, 2), "absolute", 2, 2, 0.0, "joint", True, "exact", "both",
     "magnitude_only", 0.0, 0.0, 0),
    ("attention_only_linear", 64, 4, 2, "fp32", 120, (2, 2), "absolute", 2, 2, 0.0, "separate", False, "linear",
     "both", "attention_only", 0.0, 0.0, 0),
    ("oracle_proxy_bf16", 64, 4, 2, "bf16", 120, (2, 2), "absolute", 2, 2, 0.0, "joint", True, "exact", "both",
     "oracle_proxy", 0.0, 0.0, 0),
    ("ratio_joint_mha", 128, 2, 2, "fp32", 260, (1, 1), "ratio", 0, 0, 0.05, "joint", True, "exact", "both",
     "carekv", 0.0, 0.0, 0),
    ("kind_k_one_budget", 64, 4, 2, "fp32", 150, (2, 2), "absolute", 2, 0, 0.0, "joint", True, "exact", "k",
     "carekv", 0.0, 0.0, 0),
]


@pytest.fixture(scope="module")
def pkg():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_pkg()


def _same_up_to_ties(got, want, scores):
    if sorted(got) == sorted(want):
        return True
    diff = set(got) ^ set(want)
    vals = [scores.get((p, g)) for (_, p, g) in diff]
    if any(v is None for v in vals):
        return False
    lo, hi = min(vals), max(vals)
    return hi - lo <= 1e-5 * max(abs(hi), 1e-30)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_cached_router_decode_matches_oracle(pkg, case):
    (name, D, Hq, Hkv, dt, T, (sk, sv), rmode, rk, rv, ratio, policy, norm, kmode, kind, base, rel, ab,
     mk) = case
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    QN = Hq // Hkv
    e = dict(PAPER_BEST_ENV, CAREKV_SCORE_NORMALIZE="1" if norm else "0", CAREKV_K_CORRECTION_MODE=kmode,
             CAREKV_PREFILL_RESIDUAL_KIND=kind, CAREKV_KSCORE_LIVE="0", CAREKV_DECODE_ROUTER="cached")
    with env(**e):
        cfg = pkg.CacheConfig(num_layers=1, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, max_pages=T // 16 + 4,
                              base_bits=3, group_size=32, scale_quant="int8", store_budget_mode="absolute",
                              store_abs_k=sk, store_abs_v=sv, read_budget_mode=rmode, read_abs_k=rk, read_abs_v=rv,
                              read_budget_ratio=ratio, route_policy=policy, baseline_score=base,
                              read_relative_threshold=rel, read_absolute_threshold=ab, read_min_keep=mk,
                              sketch_dim=32, correction_impl="cached")
        assert cfg.store_sketch
        dev = torch.device("cuda")
        cache = pkg.CAREKVCache(cfg, dev, batch=1)
        eng = pkg.DecodeEngine(cache)
        K = rng.standard_normal((Hkv, T, D)).astype(np.float32)
        K[:, :, :4] *= 20.0
        V = rng.standard_normal((Hkv, T, D)).astype(np.float32)
        K, V = oracle.round_to(K, dt), oracle.round_to(V, dt)
        eng.prefill_store(0, torch.from_numpy(K).to(dev, TDT[dt])[None], torch.from_numpy(V).to(dev, TDT[dt])[None])
        oc = oracle_cache_for(cfg)
        for h in range(Hkv):
            oc.prefill_write(0, h, K[h], V[h], dt)
        rc = oracle.RouteConfig(head_dim=D, kind=kind, route_policy=policy, score_normalize=norm,
                                k_correction_mode=kmode, read_budget_mode=rmode, read_abs_k=rk, read_abs_v=rv,
                                read_budget_ratio=ratio)
        for step in range(3):
            k = oracle.round_to(rng.standard_normal((Hkv, D)).astype(np.float32), dt)
            v = oracle.round_to(rng.standard_normal((Hkv, D)).astype(np.float32), dt)
            eng.append(0, torch.from_numpy(k).to(dev, TDT[dt])[None], torch.from_numpy(v).to(dev, TDT[dt])[None])
            for h in range(Hkv):
                oc.append(0, h, k[h], v[h], dt, pos_abs=T + step)
            q = rng.standard_normal((Hq, D)).astype(np.float32)
            q[1] *= 3.0
            q = oracle.round_to(q, dt)
            pages = eng._pages(0, 0)
            out = eng.attend(0, torch.from_numpy(q).to(dev, TDT[dt])[None], pages=pages).float().cpu().numpy()[0]
            sel = eng.last_selection(0, 0, 1, pages)
            for h in range(Hkv):
                K_hat, V_hat, _ = oc.read_base_concat(0, h)
                for i in range(QN):
                    qi = q[h * QN + i]
                    S, A, O = oracle.base_attention(K_hat, V_hat, qi[None], D)
                    d, info = legacy_correction(oc, 0, h, qi, S[0], A[0], O[0], V_hat, rc, oc.sketch_P, kind=kind,
                                                score_normalize=norm, k_corr_scale=0.1, exact=kmode == "exact",
                                                baseline=base, rel_thr=rel, abs_thr=ab, min_keep=mk)
                    sc = legacy_route.last_scores if hasattr(legacy_route, "last_scores") else {"K": {}, "V": {}}
                    want_k = [("K", p, g) for p, g, _ in info["k_sel"]]
                    want_v = [("V", p, b) for p, b, _ in info["v_sel"]]
                    got = sel[(0, h, i)]
                    got_k = [x for x in got if x[0] == "K"]
                    got_v = [x for x in got if x[0] == "V"]
                    assert _same_up_to_ties(got_k, want_k, sc["K"]), (step, h, i, sorted(got_k), sorted(want_k))
                    assert _same_up_to_ties(got_v, want_v, sc["V"]), (step, h, i, sorted(got_v), sorted(want_v))
                    if sorted(got) == sorted(want_k + want_v):
                        tol = {"fp32": (1e-3, 2e-3), "bf16": (1e-2, 1e-2)}[dt]
                        np.testing.assert_allclose(out[h * QN + i], oracle.round_to(O[0] + d, dt), rtol=tol[0],
                                                   atol=tol[1], err_msg=f"step {step} kv head {h} query {i}")
        cache.check_errors()
