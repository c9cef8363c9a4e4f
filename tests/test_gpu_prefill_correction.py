"""Stored-slot prefill correction (CAREKV_PREFILL_MODE=carekv_stored) against
the oracle: the reference's prefill attention (layer.py:936-972: fp32 logits
and softmax, weights cast to the activation dtype, base output in the
activation dtype, over K_hat / V_hat quantised with activation-dtype scales)
followed by vectorized_joint_correction per kv head over all of its
group x T queries (layer.py:525-550), compared with
DecodeEngine.prefill_correct and with CAREKVLayer.prefill end to end."""

import math

import zlib

import numpy as np
import pytest
import torch

import oracle
from conftest import load_pkg
from helpers import (PAPER_BEST_ENV, env, oracle_cache_for, oracle_selection, route_cfg_from, saturated_attention,
                     selection_margin)

pytestmark = pytest.mark.gpu

TDT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}
TOL = {"fp32": (1e-3, 2e-3), "fp16": (3e-3, 3e-3), "bf16": (1e-2, 1e-2)}


@pytest.fixture(scope="module")
def pkg():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_pkg()


def _inputs(rng, H, T, D, dt):
    K = rng.standard_normal((H, T, D)).astype(np.float32)
    K[:, :, :4] *= 20.0
    V = rng.standard_normal((H, T, D)).astype(np.float32)
    return oracle.round_to(K, dt), oracle.round_to(V, dt)


def reference_prefill(q, K, V, bits, g, dt):
    """The reference's carekv_stored inputs: K_hat / V_hat (activation-dtype
    scales), masked logits S, weights A (cast to dt) and base output O (dt).
    q [Hq, T, D], K / V [Hkv, T, D]."""
    Hq, T, D = q.shape
    QN = Hq // K.shape[0]
    Kh = oracle.dequantize(*oracle.quantize(K, bits, g, dt), g, dt)
    Vh = oracle.dequantize(*oracle.quantize(V, bits, g, dt), g, dt)
    Kq, Vq = np.repeat(Kh, QN, axis=0), np.repeat(Vh, QN, axis=0)
    S = np.einsum("hid,hjd->hij", q.astype(np.float32), Kq) / np.float32(math.sqrt(D))
    S = S + np.triu(np.full((T, T), np.finfo(np.float32).min, np.float32), 1)[None]
    m = S.max(-1, keepdims=True)
    e = np.exp(S - m)
    A = oracle.round_to((e / e.sum(-1, keepdims=True)).astype(np.float32), dt)
    O = oracle.round_to(np.einsum("hij,hjd->hid", A, Vq), dt)
    return Kh, Vh, S.astype(np.float32), A, O


CASES = [
    # name, D, bits, g, Hq, Hkv, dt, T, store(k,v), read mode, read(k,v)/ratio, policy, live, kmode, kind
    ("mha_int3_bf16_ratio", 128, 3, 32, 2, 2, "bf16", 70, (1, 1), "ratio", 0.03, "joint", True, "exact", "both"),
    ("gqa4_int3_fp16_abs", 64, 3, 32, 8, 2, "fp16", 53, (2, 4), "absolute", (2, 4), "joint", True, "exact", "both"),
    ("gqa2_int4_fp32_linear", 64, 4, 32, 4, 2, "fp32", 40, (2, 2), "absolute", (2, 2), "separate", True, "linear",
     "both"),
    ("gqa4_proxy_fp32", 64, 3, 32, 8, 2, "fp32", 48, (2, 2), "absolute", (2, 2), "joint", False, "exact", "both"),
    ("mha_int2_kind_v", 64, 2, 32, 2, 2, "fp32", 33, (1, 2), "absolute", (0, 2), "joint", True, "exact", "v"),
    ("gqa8_int3_bf16_ratio", 128, 3, 32, 16, 2, "bf16", 45, (1, 2), "ratio", 0.05, "joint", True, "exact", "both"),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_prefill_correction_matches_oracle(pkg, case):
    name, D, bits, g, Hq, Hkv, dt, T, (sk, sv), rmode, rb, policy, live, kmode, kind = case
    rng = np.random.default_rng(zlib.crc32(name.encode()))   # stable across processes
    QN = Hq // Hkv
    e = dict(PAPER_BEST_ENV, CAREKV_KSCORE_LIVE="1" if live else "0", CAREKV_K_CORRECTION_MODE=kmode,
             CAREKV_PREFILL_RESIDUAL_KIND=kind)
    read = dict(read_budget_mode=rmode)
    if rmode == "ratio":
        read["read_budget_ratio"] = rb
    else:
        read.update(read_abs_k=rb[0], read_abs_v=rb[1], read_budget_ratio=0.0)
    with env(**e):
        cfg = pkg.CacheConfig(num_layers=1, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, page_size=16,
                              max_pages=T // 16 + 2, base_bits=bits, group_size=g, scale_quant="int8",
                              store_budget_mode="absolute", store_abs_k=sk, store_abs_v=sv, route_policy=policy,
                              sketch_dim=32, store_sketch=not live, correction_impl="vectorized", **read)
        dev = torch.device("cuda")
        cache = pkg.CAREKVCache(cfg, dev, batch=1)
        eng = pkg.DecodeEngine(cache)
        K, V = _inputs(rng, Hkv, T, D, dt)
        eng.prefill_store(0, torch.from_numpy(K).to(dev, TDT[dt])[None], torch.from_numpy(V).to(dev, TDT[dt])[None])
        oc = oracle_cache_for(cfg)
        for h in range(Hkv):
            oc.prefill_write(0, h, K[h], V[h], dt)
        q = oracle.round_to(rng.standard_normal((Hq, T, D)).astype(np.float32), dt)
        Kh, Vh, S, A, O = reference_prefill(q, K, V, bits, g, dt)

        # oracle: vectorized_joint_correction per kv head over group x T queries
        rc = route_cfg_from(cfg)
        want = np.empty_like(O)
        infos = []
        for h in range(Hkv):
            hs = slice(h * QN, (h + 1) * QN)
            delta, info = oracle.vectorized_joint_correction(
                oc, 0, h, q[hs].reshape(-1, D), S[hs].reshape(-1, T), A[hs].reshape(-1, T), Vh[h],
                O[hs].reshape(-1, D), rc, sketch_P=oc.sketch_P)
            want[hs] = oracle.round_to(O[hs] + delta.reshape(QN, T, D), dt)
            infos.append(info)

        # device: rows (t, kv head) of QN queries
        P = eng._pages(0, 0)
        N = P * 16

        def rows(x, fill):
            y = np.full((Hq, T, N), fill, np.float32)
            y[..., :T] = x
            return torch.from_numpy(y.reshape(Hkv, QN, T, N).transpose(2, 0, 1, 3).copy()).to(dev)

        def per_row(x):
            return torch.from_numpy(np.ascontiguousarray(
                x.reshape(Hkv, QN, T, *x.shape[2:]).transpose(2, 0, 1, *range(3, x.ndim + 1)))).to(dev)
        v_rows = np.zeros((Hkv, N, D), np.float32)
        v_rows[:, :T] = Vh
        out = eng.prefill_correct(
            0, 0, torch.from_numpy(np.ascontiguousarray(q.transpose(1, 0, 2))).to(dev, TDT[dt]),
            attn=rows(A, 0.0), o_base=per_row(O.astype(np.float32)),
            o_exact=per_row(np.einsum("hij,hjd->hid", A, np.repeat(Vh, QN, axis=0)).astype(np.float32)),
            attn_sum=per_row(A.sum(-1).astype(np.float32)), logits=rows(S, np.finfo(np.float32).min),
            row_max=per_row(S.max(-1)), v_rows=torch.from_numpy(v_rows).to(dev),
            v_pnorm=torch.from_numpy(np.linalg.norm(v_rows.reshape(Hkv, P, -1), axis=-1).astype(np.float32)).to(dev))
        got = out.float().cpu().numpy().transpose(1, 0, 2)              # [Hq, T, D]
        rtol, atol = TOL[dt]
        np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)

        # selections: row (t, h) query i is the oracle's row i * T + t of kv head h
        sel = eng.last_selection(0, 0, T, P, cache_seq=0)
        for h, info in enumerate(infos):
            if info is None or "sel_k" not in info:
                continue
            ws = oracle_selection(info, QN * T)
            for i in range(QN):
                for t in range(T):
                    got_s = sorted(sel[(t, h, i)])
                    if got_s != ws[i * T + t]:
                        r = i * T + t
                        assert selection_margin(info, r) < 1e-5 or saturated_attention(info, r), \
                            (h, i, t, got_s, ws[r])
        cache.check_errors()


def test_layer_prefill_carekv_stored(pkg):
    """CAREKVLayer.prefill in carekv_stored mode: finite, different from
    base_quant when slots are read, equal to base_quant with a zero read
    budget (layer.py:817-829)."""
    Hq, Hkv, D, T, dm = 8, 2, 64, 75, 128
    g = torch.Generator().manual_seed(7)
    W = [torch.randn(o, dm, generator=g) * 0.08 for o in (Hq * D, Hkv * D, Hkv * D)] + \
        [torch.randn(dm, Hq * D, generator=g) * 0.05]
    hidden = torch.randn(2, T, dm, generator=g)
    dev = torch.device("cuda")

    def run(mode, read_abs):
        with env(**PAPER_BEST_ENV, CAREKV_PREFILL_MODE=mode):
            cfg = pkg.CacheConfig(num_layers=1, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, max_pages=8,
                                  base_bits=3, group_size=32, scale_quant="int8", store_budget_mode="absolute",
                                  store_abs_k=2, store_abs_v=2, read_budget_mode="absolute", read_abs_k=read_abs,
                                  read_abs_v=read_abs, read_budget_ratio=0.0, route_policy="joint")
            cache = pkg.CAREKVCache(cfg, dev, batch=2)
            layer = pkg.CAREKVLayer(cfg, 0, *(w.to(dev) for w in W), device=dev)
            return layer.prefill_batch(cache, hidden.to(dev)).float().cpu()

    base = run("base_quant", 2)
    stored = run("carekv_stored", 2)
    stored0 = run("carekv_stored", 0)
    assert torch.isfinite(stored).all()
    assert torch.equal(stored0, base)
    assert not torch.equal(stored, base)
    assert (stored - base).abs().max() < 0.5 * base.abs().max()
