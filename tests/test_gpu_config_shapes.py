"""Decode parity at the shapes of the benchmark configurations, at the fp32
tolerance (1e-3 relative / 2e-3 absolute), with every kv head compared and
the selection outcome of every query counted:

* config 1: 32 query / 4 kv heads, head_dim 64, 512-token context, INT3 g32,
  one K and one V slot stored per page, read ratio 0.03;
* config 3 (per sequence): 32 / 32 heads, head_dim 128, ~4096-token
  context, INT3 g32, 3 % budgets, over decode steps that fill a page and
  open the next one;
* long contexts (16384 and 32768 tokens) whose ratio budgets select more
  than 32 slots per query (60 and 122 at ratio 0.03).

Selections must equal the oracle's except at near-ties of the normalised
scores; the count of differences accepted on saturated queries must be 0."""

import collections

import numpy as np
import pytest
import torch

import oracle
from conftest import load_pkg
from helpers import PAPER_BEST_ENV, classify_selection, env, oracle_cache_for, oracle_selection, route_cfg_from

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 2e-3


@pytest.fixture(scope="module")
def pkg():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_pkg()


def _run(pkg, *, Hq, Hkv, D, T, steps, seed, policy="joint", ratio=0.03, outliers=True):
    """Prefill T tokens of one sequence, then `steps` decode steps; every
    step compares every kv head's output and every query's selection with
    the oracle.  Returns the selection outcome counts."""
    rng = np.random.default_rng(seed)
    counts = collections.Counter()
    with env(**PAPER_BEST_ENV):
        cfg = pkg.CacheConfig(num_layers=1, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, page_size=16,
                              max_pages=(T + steps) // 16 + 2, base_bits=3, group_size=32, scale_quant="int8",
                              packed_base=True, store_budget_mode="absolute", store_abs_k=1, store_abs_v=1,
                              read_budget_mode="ratio", read_budget_ratio=ratio, route_policy=policy)
        cache = pkg.CAREKVCache(cfg, torch.device("cuda"), batch=1)
        eng = pkg.DecodeEngine(cache)
        K = rng.standard_normal((Hkv, T, D)).astype(np.float32)
        if outliers:
            K[:, :, :4] *= 20.0
        V = rng.standard_normal((Hkv, T, D)).astype(np.float32)
        eng.prefill_store(0, torch.from_numpy(K).cuda()[None], torch.from_numpy(V).cuda()[None])
        oc = oracle_cache_for(cfg)
        for h in range(Hkv):
            oc.prefill_write(0, h, K[h], V[h], "fp32")
        rc = route_cfg_from(cfg)
        grp = Hq // Hkv
        for step in range(steps):
            k = rng.standard_normal((Hkv, D)).astype(np.float32)
            v = rng.standard_normal((Hkv, D)).astype(np.float32)
            eng.append(0, torch.from_numpy(k).cuda()[None], torch.from_numpy(v).cuda()[None])
            pos = T + step
            for h in range(Hkv):
                oc.append(0, h, k[h], v[h], "fp32", pos_abs=pos)
            q = rng.standard_normal((1, Hq, D)).astype(np.float32)
            pages = eng._pages(0, 0)
            out = eng.attend(0, torch.from_numpy(q).cuda(), pages=pages).cpu().numpy()
            sel = eng.last_selection(0, 0, 1, pages)
            for h in range(Hkv):
                O, info = oracle.decode_attention_kvh(oc, 0, h, q[0, h * grp:(h + 1) * grp], rc)
                np.testing.assert_allclose(out[0, h * grp:(h + 1) * grp], O, rtol=RTOL, atol=ATOL,
                                           err_msg=f"step {step} kv head {h}")
                want = oracle_selection(info, grp)
                for i in range(grp):
                    got = sel[(0, h, i)]
                    c = classify_selection(got, want[i], info, i)
                    assert c != "mismatch", (step, h, i, sorted(got), want[i])
                    counts[c] += 1
                    if c == "equal":
                        counts["selected"] += len(got)
                    counts["max_per_query"] = max(counts["max_per_query"], len(got))
        torch.cuda.synchronize()
        cache.check_errors()
    return counts


def test_config1_shape_selection_exact(pkg):
    c = _run(pkg, Hq=32, Hkv=4, D=64, T=512, steps=4, seed=101)
    print("config 1 selections:", dict(c))
    assert c["saturated"] == 0, dict(c)


def test_config3_shape_fp32_every_kv_head(pkg):
    # 4090 prefill tokens: the 6th decode step completes page 256 (page
    # store on decode), the 7th opens page 257
    c = _run(pkg, Hq=32, Hkv=32, D=128, T=4090, steps=8, seed=303)
    print("config 3 selections:", dict(c))
    assert c["saturated"] == 0, dict(c)


@pytest.mark.parametrize("T,Hq,Hkv,policy", [(16384, 2, 2, "joint"), (32768, 4, 1, "joint"),
                                             (16384, 1, 1, "separate")],
                         ids=["16k_mha_joint", "32k_gqa4_joint", "16k_separate"])
def test_long_context_ratio_budgets_beyond_32_slots(pkg, T, Hq, Hkv, policy):
    c = _run(pkg, Hq=Hq, Hkv=Hkv, D=128, T=T, steps=2, seed=T + Hq, policy=policy)
    print(f"{T} tokens selections:", dict(c))
    # ratio 0.03 over ~T/16 K and V slots: more than 32 per query
    assert c["max_per_query"] > 32, dict(c)
    assert c["saturated"] == 0, dict(c)
