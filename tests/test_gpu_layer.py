"""CAREKVLayer (prefill + decode_step) against the reference layer (GPU).

The fixture tests/golden/layer.npz holds the reference CAREKVLayer's
outputs (layer.py:643-1163) on seeded weights / hidden states / RoPE tables
regenerated here by tests/golden/layer_case.py.  The read budget is 0 in
these cases, so both sides run base decode after the append and page-full
store: the cases pin the layer plumbing (projections, RoPE, cache write,
decode attention, output projection).  The correction itself is pinned by
test_gpu_parity.py / test_gpu_decode.py.
"""

import json
import os
import sys

import numpy as np
import pytest
import torch

from conftest import load_pkg
from helpers import PAPER_BEST_ENV, env

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
from layer_case import LAYER_CASES, layer_cfg_kwargs, layer_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "layer.npz"))
META = json.loads(str(GOLD["meta"]))

PREFILL_TOL = {"fp": (1e-4, 1e-4), "base_quant": (1e-3, 2e-3)}
DECODE_RTOL, DECODE_ATOL = 1e-3, 2e-3


@pytest.mark.parametrize("case", META, ids=[c["name"] for c in META])
def test_layer_matches_reference(case):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    pkg = load_pkg()
    dev = torch.device("cuda", 0)
    Hq, Hkv, D, T, S = case["Hq"], case["Hkv"], case["D"], case["T"], case["steps"]
    L = T + S
    W_Q, W_K, W_V, W_O, hid, cos, sin = [torch.from_numpy(x).to(dev) for x in layer_inputs(Hq, Hkv, D, L, case["seed"])]
    with env(CAREKV_PREFILL_MODE=case["prefill_mode"], **PAPER_BEST_ENV):
        cfg = pkg.CacheConfig(**layer_cfg_kwargs(Hq, Hkv, D, L, case.get("base", "uniform")))
        cache = pkg.CAREKVCache(cfg, dev, batch=1)
        layer = pkg.CAREKVLayer(cfg, 0, W_Q, W_K, W_V, W_O, dev)
        pre = layer.prefill(cache, hid[:T], position_embeddings=(cos[:, :T], sin[:, :T]))
        rt, at = PREFILL_TOL[case["prefill_mode"]]
        np.testing.assert_allclose(pre.cpu().numpy(), GOLD[case["key"] + "_prefill"], rtol=rt, atol=at)
        dec = [layer.decode_step(cache, hid[T + j:T + j + 1],
                                 position_embeddings=(cos[:, T + j:T + j + 1], sin[:, T + j:T + j + 1]))
               for j in range(S)]
        got = torch.cat(dec).cpu().numpy()
        np.testing.assert_allclose(got, GOLD[case["key"] + "_decode"], rtol=DECODE_RTOL, atol=DECODE_ATOL)
        assert cache.total_valid_tokens(0, 0) == L
        cache.check_errors()


def test_layer_batch_equals_per_sequence():
    """decode_step_batch over an arena of 3 sequences equals three single-sequence layers."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    pkg = load_pkg()
    dev = torch.device("cuda", 0)
    name, Hq, Hkv, D, T, S, mode, seed = LAYER_CASES[0]
    L = T + S
    W_Q, W_K, W_V, W_O, hid, cos, sin = [torch.from_numpy(x).to(dev) for x in layer_inputs(Hq, Hkv, D, L, seed)]
    g = torch.Generator(device=dev).manual_seed(5)
    hids = torch.stack([hid, hid + 0.1 * torch.randn(hid.shape, device=dev, generator=g),
                        hid - 0.1 * torch.randn(hid.shape, device=dev, generator=g)])
    with env(CAREKV_PREFILL_MODE="fp", **PAPER_BEST_ENV):
        kw = layer_cfg_kwargs(Hq, Hkv, D, L)
        kw.update(read_budget_mode="absolute", read_abs_k=1, read_abs_v=1)
        cfg = pkg.CacheConfig(**kw)
        big = pkg.CAREKVCache(cfg, dev, batch=3)
        layer = pkg.CAREKVLayer(cfg, 0, W_Q, W_K, W_V, W_O, dev)
        pe = (cos[:, :T].expand(3, -1, -1), sin[:, :T].expand(3, -1, -1))
        pre_b = layer.prefill_batch(big, hids[:, :T], position_embeddings=pe)
        outs_b = [layer.decode_step_batch(big, hids[:, T + j], (cos[:, T + j], sin[:, T + j])) for j in range(S)]
        for b in range(3):
            one = pkg.CAREKVCache(cfg, dev, batch=1)
            pre = layer.prefill(one, hids[b, :T], position_embeddings=(cos[:, :T], sin[:, :T]))
            np.testing.assert_allclose(pre.cpu().numpy(), pre_b[b].cpu().numpy(), rtol=1e-5, atol=1e-5)
            for j in range(S):
                o = layer.decode_step(one, hids[b, T + j:T + j + 1], (cos[:, T + j:T + j + 1], sin[:, T + j:T + j + 1]))
                np.testing.assert_allclose(o[0].cpu().numpy(), outs_b[j][b].cpu().numpy(), rtol=1e-4, atol=1e-4,
                                           err_msg=f"seq {b} step {j}")
