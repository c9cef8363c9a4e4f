"""carekv_decode_attention_noalloc against carekv_decode_attention (GPU).

The no-allocation entry point serves callers that cannot allocate device
memory while a decode step runs (an engine that owns all device memory in
its own pool, a host runtime binding the C ABI without a CUDA allocator, a
latency-bound loop that must not synchronise on an allocation).  It must
give the regular entry point's output, within the parity tolerance, on two
calls in a row (the second call reuses the library's scratch array as the
first left it) and on a ragged batch and a sub-range after them, hold the
benchmark's own shape, and refuse a shape whose scratch exceeds its fixed
maximum.

Kept in its own file, named to be collected last.
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import load_pkg
from helpers import PAPER_BEST_ENV, env

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 2e-3


def _noalloc(pkg, eng, layer, q, out, pages, seq_begin=0):
    c = eng.cache
    rp = pkg.resolve_route_params(eng.cfg, layer)
    return pkg._lib.lib().carekv_decode_attention_noalloc(
        ctypes.byref(c.ccfg), ctypes.byref(c.c), layer, q.data_ptr(), out.data_ptr(), pkg._lib.BF16, seq_begin,
        q.shape[0], pages, ctypes.byref(rp), None, torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_regular_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    pkg = load_pkg()
    with env(**PAPER_BEST_ENV):
        cfg = pkg.CacheConfig(num_layers=2, num_heads=16, num_kv_heads=4, head_dim=128, max_pages=40,
                              base_bits=3, group_size=32, scale_quant="int8", packed_base=True,
                              store_budget_mode="absolute", store_abs_k=2, store_abs_v=4,
                              read_budget_mode="absolute", read_abs_k=2, read_abs_v=4, route_policy="joint")
        cache = pkg.CAREKVCache(cfg, torch.device("cuda", 0), batch=3)
        eng = pkg.DecodeEngine(cache)
        g = torch.Generator(device="cuda").manual_seed(7)
        # ragged batch: the sequences hold 301, 204 and 107 tokens, so the
        # calls leave parts of the shared scratch unwritten that a call on
        # longer sequences wrote before
        for layer in range(2):
            for b, T in enumerate((301, 204, 107)):
                K = torch.randn(1, 4, T, 128, device="cuda", generator=g)
                K[..., :4] *= 20
                eng.prefill_store(layer, K.to(torch.bfloat16),
                                  torch.randn(1, 4, T, 128, device="cuda", generator=g).to(torch.bfloat16),
                                  seq_begin=b)
        # two calls in a row over the whole batch, then one over the two
        # shorter sequences only
        for call, (layer, s0, n) in enumerate(((1, 0, 3), (0, 0, 3), (1, 1, 2))):
            k = torch.randn(n, 4, 128, device="cuda", generator=g).to(torch.bfloat16)
            eng.append(layer, k, torch.randn_like(k), seq_begin=s0)
            q = torch.randn(n, 16, 128, device="cuda", generator=g).to(torch.bfloat16)
            pages = max(eng._pages(b, layer) for b in range(s0, s0 + n))
            ref = eng.attend(layer, q, pages=pages, seq_begin=s0)
            out = torch.full_like(q, float("nan"))
            st = _noalloc(pkg, eng, layer, q, out, pages, seq_begin=s0)
            assert st == 0, pkg._lib.lib().carekv_status_string(st)
            torch.cuda.synchronize()
            np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy(), rtol=RTOL, atol=ATOL,
                                       err_msg=f"call {call + 1}")
        cache.check_errors()


def test_noalloc_scratch_holds_the_benchmark_shape():
    """32 sequences x 32 kv heads x a 4096-token context (Llama-2-7B shape,
    one K and one V slot per page) fit the fixed scratch."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    pkg = load_pkg()
    with env(**PAPER_BEST_ENV):
        cfg = pkg.CacheConfig(num_layers=1, num_heads=32, num_kv_heads=32, head_dim=128, max_pages=272,
                              base_bits=3, group_size=32, scale_quant="int8", store_budget_mode="absolute",
                              store_abs_k=1, store_abs_v=1, read_budget_mode="ratio", read_budget_ratio=0.03)
        cache = pkg.CAREKVCache(cfg, torch.device("cuda", 0), batch=1)
        eng = pkg.DecodeEngine(cache)
        assert eng.workspace_bytes(32, 264) <= pkg._lib.NOALLOC_MAX_BYTES


def test_noalloc_rejects_scratch_beyond_its_maximum():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    pkg = load_pkg()
    with env(**PAPER_BEST_ENV):
        cfg = pkg.CacheConfig(num_layers=1, num_heads=32, num_kv_heads=32, head_dim=128, max_pages=2048,
                              base_bits=3, group_size=32, scale_quant="int8", store_budget_mode="absolute",
                              store_abs_k=1, store_abs_v=1, read_budget_mode="absolute", read_abs_k=1,
                              read_abs_v=1)
        cache = pkg.CAREKVCache(cfg, torch.device("cuda", 0), batch=8)
        eng = pkg.DecodeEngine(cache)
        pages = 2048
        assert eng.workspace_bytes(8, pages) > pkg._lib.NOALLOC_MAX_BYTES
        q = torch.zeros(8, 32, 128, device="cuda", dtype=torch.bfloat16)
        out = torch.zeros_like(q)
        assert _noalloc(pkg, eng, 0, q, out, pages) == pkg._lib.ERR_WORKSPACE
