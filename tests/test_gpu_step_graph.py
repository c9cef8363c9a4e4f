"""DecodeStepGraph: one decode step over every layer replayed as a CUDA graph,
against the eager DecodeEngine calls, and its host-I/O form (transfers in
the graph, overlapping other layers) against the plain graph."""

import ctypes
import os

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


def _setup(pkg, L, B, Hq, Hkv, D, T, max_pages, seed):
    cfg = pkg.CacheConfig(num_layers=L, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, max_pages=max_pages,
                          base_bits=3, group_size=32, scale_quant="int8", store_budget_mode="absolute",
                          store_abs_k=1, store_abs_v=2, read_budget_mode="absolute", read_abs_k=2, read_abs_v=2,
                          read_budget_ratio=0.0, route_policy="joint")
    dev = torch.device("cuda")
    cache = pkg.CAREKVCache(cfg, dev, batch=B)
    eng = pkg.DecodeEngine(cache)
    g = torch.Generator(device=dev).manual_seed(seed)
    for l in range(L):
        K = torch.randn(B, Hkv, T, D, device=dev, generator=g)
        K[..., :4] *= 20
        eng.prefill_store(l, K.to(torch.bfloat16), torch.randn(B, Hkv, T, D, device=dev, generator=g).to(torch.bfloat16))
    return cfg, cache, eng


def test_step_graph_matches_eager_and_host_io(pkg):
    L, B, Hq, Hkv, D, T, MP = 2, 3, 4, 2, 64, 30, 8
    with env(**PAPER_BEST_ENV):
        _, c_e, e_e = _setup(pkg, L, B, Hq, Hkv, D, T, MP, 5)
        _, c_g, e_g = _setup(pkg, L, B, Hq, Hkv, D, T, MP, 5)
        _, c_h, e_h = _setup(pkg, L, B, Hq, Hkv, D, T, MP, 5)
        dev = torch.device("cuda")
        q = torch.zeros(L, B, Hq, D, device=dev, dtype=torch.bfloat16)
        k = torch.zeros(L, B, Hkv, D, device=dev, dtype=torch.bfloat16)
        v = torch.zeros_like(k)
        out = torch.empty_like(q)
        step = pkg.engine.DecodeStepGraph(e_g, q, k, v, out, MP)
        qh, kh, vh = torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v)
        oh = torch.empty_like(out)
        io = tuple(torch.empty_like(t, device="cpu").pin_memory() for t in (q, k, v, out))
        step_io = pkg.engine.DecodeStepGraph(e_h, qh, kh, vh, oh, MP, host_io=io)
        g = torch.Generator(device=dev).manual_seed(11)
        fills = 0
        for s in range(5):                         # T = 30: the second step completes a page
            qs = torch.randn(L, B, Hq, D, device=dev, generator=g).to(torch.bfloat16)
            ks = torch.randn(L, B, Hkv, D, device=dev, generator=g).to(torch.bfloat16)
            vs = torch.randn(L, B, Hkv, D, device=dev, generator=g).to(torch.bfloat16)
            ref = torch.stack([_eager(e_e, l, qs[l], ks[l], vs[l], MP) for l in range(L)])
            q.copy_(qs); k.copy_(ks); v.copy_(vs)
            fill = step.next_fill()
            fills += fill
            # append (+ page store and id scan on a filling step) and two launches per batch chunk
            n_att = ctypes.c_int32(0)
            pkg._lib.check(pkg._lib.lib().carekv_decode_attention_launches(ctypes.byref(c_g.ccfg), B,
                                                                           ctypes.byref(n_att)), "launches")
            assert n_att.value == 2 * (int(os.environ.get("CAREKV_ATTEND_CHUNKS", "1")) if B > 1 else 1)
            assert step.replay() == step.launches[fill] == L * ((3 if fill else 1) + n_att.value)
            for h_, d_ in zip(io[:3], (qs, ks, vs)):
                h_.copy_(d_.cpu())
            step_io.replay()
            torch.cuda.synchronize()
            torch.testing.assert_close(out.float(), ref.float(), rtol=1e-2, atol=1e-2)
            assert torch.equal(io[3], out.cpu())     # same kernels and bounds: bit-identical
        assert fills == 1
        c_g.check_errors()
        c_h.check_errors()


def _eager(eng, l, q, k, v, max_pages):
    eng.append(l, k, v)
    return eng.attend(l, q, pages=max_pages)
