"""Kv-head shards (the C ABI's _shard entry points): arenas that each hold a
contiguous range of a model's kv heads, fed the model's full activation
rows, reproduce the whole-model arena bit for bit -- cache state, decode
outputs and the step graph -- since every (sequence, kv head) is computed
independently (attention.py:576)."""

import numpy as np
import pytest
import torch

from conftest import load_pkg
from helpers import PAPER_BEST_ENV, env

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pkg():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_pkg()


def _cfg(pkg, H, Hq, **kw):
    return pkg.CacheConfig(num_layers=2, num_heads=Hq, num_kv_heads=H, head_dim=128, max_pages=24, base_bits=3,
                           group_size=32, scale_quant="int8", packed_base=True, store_budget_mode="absolute",
                           store_abs_k=1, store_abs_v=1, read_budget_mode="ratio", read_budget_ratio=0.05,
                           route_policy="joint", **kw)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_kv_head_shards_match_whole_arena(pkg, dt):
    H, QN, B, T, D = 4, 2, 3, 150, 128
    dev = torch.device("cuda")
    with env(**PAPER_BEST_ENV):
        whole = pkg.DecodeEngine(pkg.CAREKVCache(_cfg(pkg, H, H * QN), dev, batch=B))
        shards = []
        for r in range(2):
            b0, n = pkg.partition.kv_head_shard(H, 2, r)
            shards.append(pkg.DecodeEngine(pkg.CAREKVCache(_cfg(pkg, n, n * QN), dev, batch=B), shard=(b0, H)))
        g = torch.Generator(device=dev).manual_seed(11)
        for layer in range(2):
            K = torch.randn(B, H, T, D, device=dev, generator=g)
            K[..., :4] *= 20
            K, V = K.to(dt), torch.randn(B, H, T, D, device=dev, generator=g).to(dt)
            for e in [whole] + shards:
                e.prefill_store(layer, K, V)
        for step in range(20):          # crosses a page boundary (150 -> 170 tokens)
            layer = step % 2
            k = torch.randn(B, H, D, device=dev, generator=g).to(dt)
            v = torch.randn(B, H, D, device=dev, generator=g).to(dt)
            q = torch.randn(B, H * QN, D, device=dev, generator=g).to(dt)
            for e in [whole] + shards:
                e.append(layer, k, v)
            ref = whole.attend(layer, q)
            parts = [e.attend(layer, q) for e in shards]
            got = pkg.partition.reassemble_kv_heads(parts, QN)
            assert torch.equal(got, ref), f"step {step}"
        torch.cuda.synchronize()
        for r, e in enumerate(shards):
            b0, n = pkg.partition.kv_head_shard(H, 2, r)
            for name in ("k_codes", "v_codes", "k_scale", "v_scale", "k_master", "valid", "k_slot_data",
                         "v_slot_data", "k_slot_group", "v_slot_block"):
                a = whole.cache.view(name)[:, :, b0:b0 + n].cpu()
                b = e.cache.view(name).cpu()
                assert torch.equal(a, b), (r, name)
            e.cache.check_errors()
        whole.cache.check_errors()


def test_shard_step_graph_matches_whole_arena(pkg):
    H, QN, B, T, D, L = 4, 1, 2, 100, 128, 2
    dev = torch.device("cuda")
    with env(**PAPER_BEST_ENV):
        g = torch.Generator(device=dev).manual_seed(5)
        K = [torch.randn(B, H, T, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(L)]
        V = [torch.randn(B, H, T, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(L)]
        q = torch.randn(L, B, H * QN, D, device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn(L, B, H, D, device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn(L, B, H, D, device=dev, generator=g).to(torch.bfloat16)
        outs = []
        for shard in (None, (2, H)):
            n = H if shard is None else 2
            e = pkg.DecodeEngine(pkg.CAREKVCache(_cfg(pkg, n, n * QN), dev, batch=B), shard=shard)
            for l in range(L):
                e.prefill_store(l, K[l], V[l])
            out = torch.zeros_like(q)
            step = pkg.engine.DecodeStepGraph(e, q, k, v, out, 24)
            for _ in range(3):
                step.replay()
            torch.cuda.synchronize()
            e.cache.check_errors()
            outs.append(out.clone())
            del step
        assert torch.equal(outs[1][:, :, 2:4], outs[0][:, :, 2:4])
        assert torch.count_nonzero(outs[1][:, :, :2]) == 0


def test_invalid_shard_is_rejected(pkg):
    dev = torch.device("cuda")
    cache = pkg.CAREKVCache(_cfg(pkg, 2, 4), dev, batch=1)
    with pytest.raises(ValueError):
        pkg.DecodeEngine(cache, shard=(3, 4))
    e = pkg.DecodeEngine(cache, shard=(2, 4))
    with pytest.raises(ValueError):
        e.append(0, torch.randn(1, 2, 128, device=dev), torch.randn(1, 2, 128, device=dev))   # needs model rows
