"""Ill-conditioned exact corrections: the router's direct form.

When the selected K pages hold nearly all of a query's attention and their
corrections ds are strongly negative, the exact correction's new normaliser
sum_t A_t e^ds_t falls below 0.01 and the router sums the tokens outside the
selection explicitly (route_body.cuh, the direct form) instead of taking them
through the base output.  These cases build such queries on purpose: one
token per (sequence, kv head) whose first 32-channel group quantizes with a
large residual of negative dot product with the query, which aligns with it
(normalisers 3e-5 .. 2e-3 in the oracle, recorded here and required below
0.01), and compare outputs and selections with the oracle.  D = 64 runs the
direct form with the two half-warps on alternate rows, D = 128 with one row
per warp step."""

import numpy as np
import pytest
import torch

import oracle
import oracle.attention as oattn
from conftest import load_pkg
from helpers import (PAPER_BEST_ENV, env, oracle_cache_for, oracle_selection, route_cfg_from, saturated_attention,
                     selection_margin)

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 2e-3


@pytest.fixture(scope="module")
def pkg():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_pkg()


def _inputs(D, H, QG, T, B, sigma=6.0, s=1.0, seed=7):
    rng = np.random.default_rng(seed)
    K = rng.standard_normal((B, H, T, D)).astype(np.float32)
    V = rng.standard_normal((B, H, T, D)).astype(np.float32)
    q = (rng.standard_normal((B, H * QG, D)) * 0.3).astype(np.float32)
    for b in range(B):
        for h in range(H):
            t = 37 + 16 * ((b + h) % 5)
            K[b, h, t, 0] = 3 * sigma          # sets the group's scale
            K[b, h, t, 1:32] = 0.6 * sigma     # rounds up: residual -0.4 sigma per channel
            q[b, h * QG:(h + 1) * QG, :32] += s
    return K, V, q


@pytest.mark.parametrize("D,H,QG", [(64, 2, 8), (128, 2, 1)], ids=["d64_gqa8", "d128_mha"])
def test_direct_form_against_oracle(pkg, D, H, QG, monkeypatch):
    B, T = 2, 200
    K, V, q = _inputs(D, H, QG, T, B)
    rng = np.random.default_rng(11)
    kn = rng.standard_normal((B, H, D)).astype(np.float32)
    vn = rng.standard_normal((B, H, D)).astype(np.float32)
    norms = []
    exact = oattn.exact_softmax_correction

    def recording(A, ds, *args, **kw):
        norms.append((A * np.exp(ds)).sum(axis=1))
        return exact(A, ds, *args, **kw)

    monkeypatch.setattr(oattn, "exact_softmax_correction", recording)
    with env(**PAPER_BEST_ENV):
        cfg = pkg.CacheConfig(num_layers=1, num_heads=H * QG, num_kv_heads=H, head_dim=D, max_pages=T // 16 + 4,
                              base_bits=3, group_size=32, scale_quant="int8", packed_base=True,
                              store_budget_mode="absolute", store_abs_k=1, store_abs_v=1,
                              read_budget_mode="absolute", read_abs_k=2, read_abs_v=2, route_policy="joint",
                              correction_impl="vectorized")
        cache = pkg.CAREKVCache(cfg, torch.device("cuda"), batch=B)
        eng = pkg.DecodeEngine(cache)
        eng.prefill_store(0, torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda())
        eng.append(0, torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda())
        pages = max(eng._pages(b, 0) for b in range(B))
        out = eng.attend(0, torch.from_numpy(q).cuda(), pages=pages).cpu().numpy()
        sel = eng.last_selection(0, 0, B, pages)
        cache.check_errors()
        rc = route_cfg_from(cfg)
        for b in range(B):
            oc = oracle_cache_for(cfg)
            for h in range(H):
                oc.prefill_write(0, h, K[b, h], V[b, h], "fp32")
                oc.append(0, h, kn[b, h], vn[b, h], "fp32")
            for h in range(H):
                qs = slice(h * QG, (h + 1) * QG)
                O, info = oracle.decode_attention_kvh(oc, 0, h, q[b, qs], rc)
                np.testing.assert_allclose(out[b, qs], O, rtol=RTOL, atol=ATOL, err_msg=f"seq {b} kv head {h}")
                want = oracle_selection(info, QG)
                for i in range(QG):
                    got = sorted(sel[(b, h, i)])
                    if got != want[i]:
                        assert selection_margin(info, i) < 1e-5 or saturated_attention(info, i), (b, h, i, got, want[i])
    nn = np.concatenate(norms)
    # the construction makes the direct form run: most queries ill-conditioned
    assert (nn < 0.01).sum() >= nn.size // 2, nn
