"""KIVI-style packed base (base_quantizer='kivi_style') on the GPU.

The reference keeps K_hat / V_hat of a KIVI base in an fp16 side buffer
(cache.py:487-499, 800-865): K quantized per channel over the whole
prefill, V per token (kivi_helpers.py:35-59), decode-appended K rows
quantized per channel over their single token (layer.py:1037-1085).  This
library stores packed codes with per-channel K / per-token V scales and a
bounded fp16 window for decode-appended K rows.  Checked here:

* the reference's goldens (tests/golden/kivi_store.npz): side buffers bit
  for bit as read back (read_base_hat_concat), slots, and base decode
  outputs over 20 steps;
* the oracle on seeded inputs with the paper-best correction on top,
  including a Mistral-7B-like INT2 GQA-4 shape with a ratio budget;
* the fp16 window capacity reported on the host.
"""

import json
import os
import zlib

import numpy as np
import pytest
import torch

import oracle
from conftest import load_pkg
from helpers import (PAPER_BEST_ENV, classify_selection, compare_kivi_state, env, oracle_cache_for,
                     oracle_selection, route_cfg_from)

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "kivi_store.npz")
TDT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}
RTOL, ATOL = 1e-3, 2e-3


@pytest.fixture(scope="module")
def pkg():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_pkg()


def _kivi_oracle(cfg):
    oc = oracle_cache_for(cfg)
    return oracle.OracleCache(oc.L, oc.H, oc.D, oc.P, oc.cfg, scale_quant="none", base="kivi")


@pytest.mark.parametrize("ci", range(4))
def test_kivi_store_and_decode_match_reference_goldens(pkg, ci):
    z = np.load(GOLD)
    c = json.loads(str(z["meta"]))[ci]
    key, dt = c["key"], c["dt"]
    Hq, Hkv, D = c["Hq"], c["Hkv"], c["D"]
    with env(**PAPER_BEST_ENV):
        cfg = pkg.CacheConfig(num_layers=1, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, max_pages=c["max_pages"],
                              base_bits=c["bits"], base_quantizer="kivi_style", store_budget_mode="absolute",
                              store_abs_k=c["store_abs_k"], store_abs_v=c["store_abs_v"], read_budget_ratio=0.0,
                              kivi_window_pages=4)
        cache = pkg.CAREKVCache(cfg, torch.device("cuda"), batch=1)
        eng = pkg.DecodeEngine(cache)
        dev = torch.device("cuda")
        eng.prefill_store(0, torch.from_numpy(z[key + "_K"]).to(dev, TDT[dt])[None],
                          torch.from_numpy(z[key + "_V"]).to(dev, TDT[dt])[None])

        def check_side_buffers(k):
            for h in range(Hkv):
                Kg, Vg, lens = cache.read_base_hat_concat(0, h)
                n = sum(lens)
                np.testing.assert_array_equal(Kg.float().cpu().numpy(),
                                              z[k + "_khat"][0, h].reshape(-1, D)[np.concatenate(
                                                  [np.arange(16 * p, 16 * p + m) for p, m in enumerate(lens)])],
                                              err_msg=f"K_hat head {h}")
                np.testing.assert_array_equal(Vg.float().cpu().numpy(),
                                              z[k + "_vhat"][0, h].reshape(-1, D)[np.concatenate(
                                                  [np.arange(16 * p, 16 * p + m) for p, m in enumerate(lens)])],
                                              err_msg=f"V_hat head {h}")
                assert n == int(z[k + "_valid"][0, h].sum())
            for m in json.loads(str(z[k + "_meta"])):
                gm = cache.page_meta(0, m["h"], m["p"])
                assert gm.k_residual_slots == m["k"] and gm.v_residual_slots == m["v"], m
        torch.cuda.synchronize()
        check_side_buffers(key)
        grp = Hq // Hkv
        for s in range(c["steps"]):
            eng.append(0, torch.from_numpy(z[key + "_dk"][s]).to(dev, TDT[dt])[None],
                       torch.from_numpy(z[key + "_dv"][s]).to(dev, TDT[dt])[None])
            out = eng.attend(0, torch.from_numpy(z[key + "_dq"][s]).to(dev, TDT[dt])[None], correction=False)
            tol = {"fp32": (RTOL, ATOL), "fp16": (3e-3, 3e-3), "bf16": (1e-2, 1e-2)}[dt]
            np.testing.assert_allclose(out[0].float().cpu().numpy(), z[key + "_dO"][s], rtol=tol[0], atol=tol[1],
                                       err_msg=f"step {s}")
        torch.cuda.synchronize()
        check_side_buffers(key + "d")
        cache.check_errors()


KIVI_CASES = [
    # name, D, bits, Hq, Hkv, dt, T, steps, store (k, v), read mode, read
    ("int2_d128_gqa4_bf16_ratio", 128, 2, 8, 2, "bf16", 300, 20, (1, 1), "ratio", 0.05),
    ("int2_d128_gqa4_fp32_abs", 128, 2, 4, 1, "fp32", 170, 18, (2, 2), "absolute", (2, 3)),
    ("int3_d64_mha_fp32", 64, 3, 2, 2, "fp32", 90, 12, (1, 2), "absolute", (2, 2)),
    ("int4_d64_gqa2_fp16", 64, 4, 4, 2, "fp16", 61, 9, (2, 2), "absolute", (1, 2)),
]


@pytest.mark.parametrize("case", KIVI_CASES, ids=[c[0] for c in KIVI_CASES])
def test_kivi_decode_with_correction_matches_oracle(pkg, case):
    name, D, bits, Hq, Hkv, dt, T, steps, (sk, sv), rmode, rb = case
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    read = dict(read_budget_mode=rmode)
    if rmode == "ratio":
        read["read_budget_ratio"] = rb
    else:
        read.update(read_abs_k=rb[0], read_abs_v=rb[1], read_budget_ratio=0.0)
    B = 2
    with env(**PAPER_BEST_ENV):
        cfg = pkg.CacheConfig(num_layers=1, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, page_size=16,
                              max_pages=(T + steps) // 16 + 2, base_bits=bits, base_quantizer="kivi_style",
                              store_budget_mode="absolute", store_abs_k=sk, store_abs_v=sv, route_policy="joint",
                              kivi_window_pages=3, **read)
        cache = pkg.CAREKVCache(cfg, torch.device("cuda"), batch=B)
        eng = pkg.DecodeEngine(cache)
        seqs = []
        for b in range(B):
            Tb = T - 9 * b
            K = rng.standard_normal((Hkv, Tb, D)).astype(np.float32)
            K[:, :, :4] *= 20.0
            V = rng.standard_normal((Hkv, Tb, D)).astype(np.float32)
            K, V = oracle.round_to(K, dt), oracle.round_to(V, dt)
            eng.prefill_store(0, torch.from_numpy(K).cuda().to(TDT[dt])[None],
                              torch.from_numpy(V).cuda().to(TDT[dt])[None], seq_begin=b)
            oc = _kivi_oracle(cfg)
            for h in range(Hkv):
                oc.prefill_write(0, h, K[h], V[h], dt)
            seqs.append(oc)
        rc = route_cfg_from(cfg)
        grp = Hq // Hkv
        counts = {"equal": 0, "tie": 0, "saturated": 0}
        for step in range(steps):
            k = oracle.round_to(rng.standard_normal((B, Hkv, D)).astype(np.float32), dt)
            v = oracle.round_to(rng.standard_normal((B, Hkv, D)).astype(np.float32), dt)
            eng.append(0, torch.from_numpy(k).cuda().to(TDT[dt]), torch.from_numpy(v).cuda().to(TDT[dt]))
            for b, oc in enumerate(seqs):
                pos = int(oc.valid[0, 0, :oc.next_page[0, 0]].sum())
                for h in range(Hkv):
                    oc.append(0, h, k[b, h], v[b, h], dt, pos_abs=pos)
            q = rng.standard_normal((B, Hq, D)).astype(np.float32)
            pages = max(eng._pages(b, 0) for b in range(B))
            out = eng.attend(0, torch.from_numpy(q).cuda().to(TDT[dt]), pages=pages).float().cpu().numpy()
            sel = eng.last_selection(0, 0, B, pages)
            for b, oc in enumerate(seqs):
                for h in range(Hkv):
                    qh = oracle.round_to(q[b, h * grp:(h + 1) * grp], dt)
                    O, info = oracle.decode_attention_kvh(oc, 0, h, qh, rc)
                    tol = {"fp32": (RTOL, ATOL), "fp16": (3e-3, 3e-3), "bf16": (1e-2, 1e-2)}[dt]
                    np.testing.assert_allclose(out[b, h * grp:(h + 1) * grp], oracle.round_to(O, dt), rtol=tol[0],
                                               atol=tol[1], err_msg=f"step {step} seq {b} kv head {h}")
                    if info is not None and "sel_k" in info:
                        want = oracle_selection(info, grp)
                        for i in range(grp):
                            cl = classify_selection(sel[(b, h, i)], want[i], info, i)
                            assert cl != "mismatch", (step, b, h, i, sorted(sel[(b, h, i)]), want[i])
                            counts[cl] += 1
        torch.cuda.synchronize()
        for b, oc in enumerate(seqs):
            compare_kivi_state(cache, oc, b, 0)
        cache.check_errors()
        print(name, counts)
        assert counts["saturated"] == 0


def test_kivi_window_capacity_is_reported_on_the_host(pkg):
    with env(**PAPER_BEST_ENV):
        cfg = pkg.CacheConfig(num_layers=1, num_heads=2, num_kv_heads=2, head_dim=64, max_pages=16, base_bits=2,
                              base_quantizer="kivi_style", store_budget_mode="absolute", store_abs_k=1,
                              store_abs_v=1, kivi_window_pages=1)
        cache = pkg.CAREKVCache(cfg, torch.device("cuda"), batch=1)
        eng = pkg.DecodeEngine(cache)
        K = torch.randn(1, 2, 40, 64, device="cuda")
        eng.prefill_store(0, K, K.clone())           # 40 tokens: the window starts at page 2 (row 8)
        for _ in range(8):                           # rows 8..15 of page 2 fill window page 0
            eng.append(0, torch.randn(1, 2, 64, device="cuda"), torch.randn(1, 2, 64, device="cuda"))
        with pytest.raises(pkg._lib.CacheFullError):
            eng.append(0, torch.randn(1, 2, 64, device="cuda"), torch.randn(1, 2, 64, device="cuda"))
        with pytest.raises(NotImplementedError):     # one prefill per sequence and layer
            eng.prefill_store(0, K, K.clone())
        cache.check_errors()
