"""The router's CTA size follows its grid: 4 warps when the (sequence, kv
head, query head) grid fills the GPU, 8 or 16 when it is small (route.cu).
Most GPU tests run small batches (16-warp CTAs); this one also runs batches
of 640 (4-warp CTAs) and 384 (8-warp CTAs) routing CTAs and checks, for
sampled sequences, the oracle and the same sequences routed alone in a
small batch."""

import numpy as np
import pytest
import torch

import oracle
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


@pytest.mark.parametrize("B", [20, 12], ids=["640_ctas_4_warps", "384_ctas_8_warps"])
def test_large_and_small_route_grids_agree(pkg, B):
    H, D, T = 32, 128, 200
    sample = [0, 7, B - 1]                 # routed alone: 96 CTAs, the 16-warp form
    rng = np.random.default_rng(20260)
    K = rng.standard_normal((B, H, T, D)).astype(np.float32)
    K[..., :4] *= 20.0
    V = rng.standard_normal((B, H, T, D)).astype(np.float32)
    with env(**PAPER_BEST_ENV):
        kw = dict(num_layers=1, num_heads=H, num_kv_heads=H, head_dim=D, max_pages=T // 16 + 4, base_bits=3,
                  group_size=32, scale_quant="int8", packed_base=True, store_budget_mode="absolute",
                  store_abs_k=1, store_abs_v=1, read_budget_mode="absolute", read_abs_k=2, read_abs_v=2,
                  route_policy="joint", correction_impl="vectorized")
        cfg = pkg.CacheConfig(**kw)
        big = pkg.CAREKVCache(cfg, torch.device("cuda"), batch=B)
        small = pkg.CAREKVCache(cfg, torch.device("cuda"), batch=len(sample))
        eb, es = pkg.DecodeEngine(big), pkg.DecodeEngine(small)
        eb.prefill_store(0, torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda())
        es.prefill_store(0, torch.from_numpy(K[sample]).cuda(), torch.from_numpy(V[sample]).cuda())
        ocs = []
        for b in sample:
            oc = oracle_cache_for(cfg)
            for h in range(H):
                oc.prefill_write(0, h, K[b, h], V[b, h], "fp32")
            ocs.append(oc)
        rc = route_cfg_from(cfg)
        for step in range(2):
            kn = rng.standard_normal((B, H, D)).astype(np.float32)
            vn = rng.standard_normal((B, H, D)).astype(np.float32)
            q = rng.standard_normal((B, H, D)).astype(np.float32)
            eb.append(0, torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda())
            es.append(0, torch.from_numpy(kn[sample]).cuda(), torch.from_numpy(vn[sample]).cuda())
            for oc, b in zip(ocs, sample):
                for h in range(H):
                    oc.append(0, h, kn[b, h], vn[b, h], "fp32")
            pb = max(eb._pages(b, 0) for b in range(B))
            ob = eb.attend(0, torch.from_numpy(q).cuda(), pages=pb).cpu().numpy()
            sb = eb.last_selection(0, 0, B, pb)
            ps = max(es._pages(b, 0) for b in range(len(sample)))
            os_ = es.attend(0, torch.from_numpy(q[sample]).cuda(), pages=ps).cpu().numpy()
            for k, (oc, b) in enumerate(zip(ocs, sample)):
                np.testing.assert_allclose(ob[b], os_[k], rtol=1e-5, atol=1e-6, err_msg=f"step {step} seq {b}")
                for h in range(H):
                    O, info = oracle.decode_attention_kvh(oc, 0, h, q[b, h:h + 1], rc)
                    np.testing.assert_allclose(ob[b, h:h + 1], O, rtol=RTOL, atol=ATOL,
                                               err_msg=f"step {step} seq {b} kv head {h}")
                    want = oracle_selection(info, 1)[0]
                    got = sorted(sb[(b, h, 0)])
                    if got != want:
                        assert selection_margin(info, 0) < 1e-5 or saturated_attention(info, 0), (b, h, got, want)
