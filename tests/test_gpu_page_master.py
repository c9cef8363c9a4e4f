"""CAREKV_DECODE_PAGE_MASTER: a page opened during decode keeps the
reference's int8 master 0 by default (cache.py:689-695: its appended rows
read back as zero); with the flag, its first appended row sets the master
the way write_base does for a prefill page (cache.py:592-606: largest scale,
clamped, / 127) and the rows read back quantized."""

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


def _decode_page(pkg, flag):
    D, H, G = 128, 2, 4
    with env(**PAPER_BEST_ENV, CAREKV_DECODE_PAGE_MASTER=flag):
        cfg = pkg.CacheConfig(num_layers=1, num_heads=H, num_kv_heads=H, head_dim=D, max_pages=4, base_bits=3,
                              group_size=32, scale_quant="int8", store_budget_mode="absolute", store_abs_k=1,
                              store_abs_v=1, read_budget_mode="absolute", read_abs_k=1, read_abs_v=1,
                              read_budget_ratio=0.0, route_policy="joint")
        dev = torch.device("cuda")
        cache = pkg.CAREKVCache(cfg, dev, batch=1)
        eng = pkg.DecodeEngine(cache)
        g = torch.Generator(device=dev).manual_seed(3)
        eng.prefill_store(0, torch.randn(1, H, 16, D, device=dev, generator=g),
                          torch.randn(1, H, 16, D, device=dev, generator=g))   # one full page
        # row 1 is smaller than row 0, row 2 an outlier 8x larger
        rows = [(torch.randn(1, H, D, device=dev, generator=g) * f, torch.randn(1, H, D, device=dev, generator=g) * f)
                for f in (1.0, 0.5, 8.0)]
        for k, v in rows:                        # the first append opens page 1
            eng.append(0, k, v)
        out = eng.attend(0, torch.randn(1, H, D, device=dev, generator=g))
        torch.cuda.synchronize()
        cache.check_errors()
        assert torch.isfinite(out.float()).all()
        res = []
        for h in range(H):
            Kc, Ks, Vc, Vs, lens = cache.read_base_concat(0, h, [1])
            assert lens == [3]
            kh = Kc.float() * Ks.float().repeat_interleave(D // G, dim=1)
            vh = Vc.float() * Vs.float().repeat_interleave(D // G, dim=1)
            k_in = torch.stack([r[0][0, h] for r in rows]).float()
            v_in = torch.stack([r[1][0, h] for r in rows]).float()
            km = cache.view("k_master")[0, 0, h, 1].float().item()
            vm = cache.view("v_master")[0, 0, h, 1].float().item()
            res.append((kh, vh, k_in, v_in, km, vm))
        return res


def test_decode_opened_page_reads_zero_by_default(pkg):
    for kh, vh, *_ in _decode_page(pkg, "0"):
        assert torch.count_nonzero(kh) == 0 and torch.count_nonzero(vh) == 0


def test_decode_page_master_flag(pkg):
    for kh, vh, k_in, v_in, km, vm in _decode_page(pkg, "1"):
        for got, want, m in ((kh, k_in, km), (vh, v_in, vm)):
            assert m > 0
            assert torch.count_nonzero(got, dim=1).min() > 0
            # rows 0 and 1 fit the master set by row 0: INT3 group
            # quantization error only
            for r in (0, 1):
                rel = (got[r] - want[r]).norm() / want[r].norm()
                assert rel < 0.4, (r, rel)
            # row 2's group scales exceed 127 x master: its int8 scale codes
            # saturate at 127, so it reads back clipped to 3 x 127 x master
            lim = 3 * 127 * m * (1 + 2e-3)
            assert got[2].abs().max().item() <= lim
            assert want[2].abs().max().item() > lim
            rel2 = (got[2] - want[2]).norm() / want[2].norm()
            assert rel2 > 0.4, rel2
