"""CAREKVCache: the paged, packed, KV-head-indexed cache arena in HBM.

One arena holds ``batch`` sequences with the reference's per-sequence layout
(cache.py:430-536) as its inner dimensions: for sequence b,
``k_codes[b]`` is the reference's ``base_K_codes[L, Hkv, P, T, rowB]`` in its
exact packed row format, ``k_scale[b]`` its int8 (or raw) scale buffer,
``k_master[b]`` its fp16 page masters and ``valid[b]`` its valid_tokens.
Residual slots live next to their page (capacity = the store budget) instead
of in one global arena; each slot also records the id the reference's
sequential free-list allocator would have given it, so ``page_meta`` can
rebuild the reference's PageMeta exactly.

All buffers are torch device tensors (plumbing only); every computation on
them goes through libcarekv_b200.so.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import torch

from . import _lib
from .config import CacheConfig


@dataclass
class PageMeta:
    """Per-page metadata view (cache.py:391-409)."""
    page_id: int
    layer_id: int
    kv_head: int
    token_start: int
    num_tokens: int
    k_residual_slots: List[int] = field(default_factory=list)
    v_residual_slots: List[int] = field(default_factory=list)
    k_error_norm: Optional[torch.Tensor] = None
    v_error_norm: Optional[torch.Tensor] = None
    k_sketch: Optional[torch.Tensor] = None
    prior_score: float = 0.0


def _stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class CAREKVCache:
    """Arena for ``batch`` sequences of ``cfg`` on a CUDA device."""

    def __init__(self, cfg: CacheConfig, device: torch.device = None, batch: int = 1):
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("CAREKVCache lives in GPU memory; the B200 build has no CPU path")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.cfg = cfg
        self.device = device
        self.batch = int(batch)
        self.ccfg = cfg.c_config()
        lib = _lib.lib()
        sizes = (ctypes.c_size_t * _lib.NUM_BUFFERS)()
        _lib.check(lib.carekv_cache_layout(ctypes.byref(self.ccfg), self.batch, sizes), "carekv_cache_layout")
        self.sizes = list(sizes)
        self.buffers = {}
        for name, n in zip(_lib.CACHE_PTR_FIELDS, self.sizes):
            self.buffers[name] = torch.empty(max(int(n), 0), dtype=torch.uint8, device=device) if n else None
        if not cfg.store_sketch:
            self.buffers["k_sketch"] = None
        self.c = _lib.Cache()
        self.c.batch = self.batch
        for name in _lib.CACHE_PTR_FIELDS:
            t = self.buffers[name]
            setattr(self.c, name, t.data_ptr() if t is not None else None)
        self._sketch_P = None
        self.lengths = [[0] * cfg.num_layers for _ in range(self.batch)]  # host mirror of token counts
        self.reset()

    # ── lifecycle ─────────────────────────────────────────────────────
    def reset(self):
        """Empty every sequence (the reference builds a fresh cache)."""
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().carekv_cache_init(ctypes.byref(self.ccfg), ctypes.byref(self.c),
                                                    _stream_ptr(self.device)), "carekv_cache_init")
        self.lengths = [[0] * self.cfg.num_layers for _ in range(self.batch)]
        self._page_state = {}   # (seq, layer) -> (pages, valid rows of the last page)

    def memory_bytes(self) -> int:
        return sum(int(t.numel()) for t in self.buffers.values() if t is not None)

    def sketch_proj(self) -> torch.Tensor:
        """Fixed random projection (residual_store.py:206-214) on the device."""
        if self._sketch_P is None:
            import math
            gen = torch.Generator(device="cpu").manual_seed(42)
            P = torch.randn(self.cfg.k_channel_group, self.cfg.sketch_dim, generator=gen) / math.sqrt(self.cfg.sketch_dim)
            self._sketch_P = P.to(self.device).contiguous()
        return self._sketch_P

    def check_errors(self):
        flags = _lib.i32(0)
        _lib.check(_lib.lib().carekv_check_device_errors(ctypes.byref(self.c), ctypes.byref(flags),
                                                         _stream_ptr(self.device)), "device check")

    # ── typed views (inspection / parity) ─────────────────────────────
    def _view(self, name, dtype, shape):
        t = self.buffers[name]
        if t is None:
            return None
        return t.view(dtype).view(*shape)

    @property
    def dims(self):
        c = self.ccfg
        B, L, H, P, T = self.batch, c.num_layers, c.num_kv_heads, c.max_pages, c.page_size
        D = c.head_dim
        rowB = {2: D // 4, 3: D * 3 // 8, 4: D // 2}[c.base_bits]
        return B, L, H, P, T, D, rowB, D // c.group_size

    def view(self, name):
        B, L, H, P, T, D, R, G = self.dims
        c = self.ccfg
        C, NV = D // c.k_channel_group, T // c.v_token_block
        scale_dt = {_lib.SCALE_INT8: torch.int8, _lib.SCALE_F16: torch.float16,
                    _lib.SCALE_BF16: torch.bfloat16, _lib.SCALE_F32: torch.float32}[c.scale_mode]
        spec = {
            "k_codes": (torch.uint8, (B, L, H, P, T, R)), "v_codes": (torch.uint8, (B, L, H, P, T, R)),
            "k_scale": (scale_dt, (B, L, H, P, T, G)), "v_scale": (scale_dt, (B, L, H, P, T, G)),
            "k_master": (torch.float16, (B, L, H, P)), "v_master": (torch.float16, (B, L, H, P)),
            "valid": (torch.int32, (B, L, H, P)), "num_pages": (torch.int32, (B, L, H)),
            "v_norm2": (torch.float32, (B, L, H, P)),
            "k_slot_group": (torch.int8, (B, L, H, P, c.k_slots_per_page)),
            "k_slot_data": (torch.uint8, (B, L, H, P, c.k_slots_per_page, T * c.k_channel_group // 2)),
            "k_slot_scale": (torch.float16, (B, L, H, P, c.k_slots_per_page)),
            "k_slot_id": (torch.int32, (B, L, H, P, c.k_slots_per_page)),
            "v_slot_block": (torch.int8, (B, L, H, P, c.v_slots_per_page)),
            "v_slot_data": (torch.uint8, (B, L, H, P, c.v_slots_per_page, c.v_token_block * D // 2)),
            "v_slot_scale": (torch.float16, (B, L, H, P, c.v_slots_per_page)),
            "v_slot_id": (torch.int32, (B, L, H, P, c.v_slots_per_page)),
            "k_err": (torch.float16, (B, L, H, P, C)), "v_err": (torch.float16, (B, L, H, P, NV)),
            "k_sketch": (torch.float16, (B, L, H, P, C, max(c.sketch_dim, 1))),
            "slot_counter": (torch.int32, (B, 2)), "read_counter": (torch.int64, (L, H, 2)),
            "error_flag": (torch.int32, (1,)),
            "k_chan_scale": (torch.float32, (B, L, H, D)),
            "k_window": (torch.float16, (B, L, H, max(c.kivi_window_pages, 1), T, D)),
            "prefill_tokens": (torch.int32, (B, L, H)),
        }[name]
        return self._view(name, *spec)

    # ── reference-compatible accessors ─────────────────────────────────
    def num_pages(self, layer: int, kv_head: int, seq: int = 0) -> int:
        return int(self.view("num_pages")[seq, layer, kv_head].item())

    def all_page_ids(self, layer: int, kv_head: int, seq: int = 0) -> List[int]:
        return list(range(self.num_pages(layer, kv_head, seq)))

    def total_valid_tokens(self, layer: int, kv_head: int, seq: int = 0) -> int:
        np_ = self.num_pages(layer, kv_head, seq)
        return int(self.view("valid")[seq, layer, kv_head, :np_].sum().item()) if np_ else 0

    def num_stored_residual_slots(self, seq: int = 0) -> Tuple[int, int]:
        sc = self.view("slot_counter")[seq]
        return int(sc[0].item()), int(sc[1].item())

    def page_meta(self, layer: int, kv_head: int, page_id: int, seq: int = 0) -> PageMeta:
        """The reference's PageMeta for a page, rebuilt from the device tables."""
        c = self.ccfg
        C, NV = c.head_dim // c.k_channel_group, c.page_size // c.v_token_block
        def _row(name):
            t = self.view(name)
            return [] if t is None else t[seq, layer, kv_head, page_id].tolist()
        kg, ki = _row("k_slot_group"), _row("k_slot_id")
        vb, vi = _row("v_slot_block"), _row("v_slot_id")
        ks = [-1] * C
        vs = [-1] * NV
        for g, i in zip(kg, ki):
            if g >= 0:
                ks[g] = i
        for g, i in zip(vb, vi):
            if g >= 0:
                vs[g] = i
        sk = self.view("k_sketch")
        return PageMeta(
            page_id=page_id, layer_id=layer, kv_head=kv_head,
            token_start=page_id * c.page_size,
            num_tokens=int(self.view("valid")[seq, layer, kv_head, page_id].item()),
            k_residual_slots=ks, v_residual_slots=vs,
            k_error_norm=self.view("k_err")[seq, layer, kv_head, page_id].clone(),
            v_error_norm=self.view("v_err")[seq, layer, kv_head, page_id].clone(),
            k_sketch=None if sk is None else sk[seq, layer, kv_head, page_id].clone())

    def read_base_concat(self, layer: int, kv_head: int, page_ids: Optional[List[int]] = None, seq: int = 0):
        """cache.py:720-772: valid rows' codes (unpacked on the GPU) and fp16 scales."""
        from .quantizer import unpack_codes_2d
        c = self.ccfg
        if page_ids is None:
            page_ids = self.all_page_ids(layer, kv_head, seq)
        valid = self.view("valid")[seq, layer, kv_head]
        lens = [int(valid[p].item()) for p in page_ids]
        Kc, Ks, Vc, Vs = [], [], [], []
        for p, n in zip(page_ids, lens):
            if n == 0:
                continue
            Kc.append(unpack_codes_2d(self.view("k_codes")[seq, layer, kv_head, p, :n].contiguous(), c.base_bits, c.head_dim))
            Vc.append(unpack_codes_2d(self.view("v_codes")[seq, layer, kv_head, p, :n].contiguous(), c.base_bits, c.head_dim))
            Ks.append(self._read_scale("k", seq, layer, kv_head, p, n))
            Vs.append(self._read_scale("v", seq, layer, kv_head, p, n))
        D, G = c.head_dim, c.head_dim // c.group_size
        if not Kc:
            e8 = torch.zeros(0, D, dtype=torch.int8, device=self.device)
            ef = torch.zeros(0, G, dtype=torch.float16, device=self.device)
            return e8, ef, e8, ef, lens
        return torch.cat(Kc), torch.cat(Ks), torch.cat(Vc), torch.cat(Vs), lens

    def _read_scale(self, which, seq, layer, h, p, n):
        s = self.view(f"{which}_scale")[seq, layer, h, p, :n]
        if self.ccfg.scale_mode == _lib.SCALE_INT8:
            m = self.view(f"{which}_master")[seq, layer, h, p]
            return (s.float() * m.float()).to(torch.float16)
        return s.to(torch.float16)

    def read_base_hat_concat(self, layer: int, kv_head: int, page_ids: Optional[List[int]] = None, seq: int = 0):
        """KIVI base: the valid K_hat / V_hat rows of the pages in fp16, as the
        reference's side buffer returns them (cache.py:845-865), rebuilt from
        the packed codes, the per-channel K / per-token V scales and the fp16
        window of decode-appended K rows.  Returns (K_hat, V_hat, valid_lens)."""
        c = self.ccfg
        if c.base_kind != _lib.BASE_KIVI:
            raise AssertionError("read_base_hat_concat requires a KIVI-style base_quantizer")
        from .quantizer import unpack_codes_2d
        D, T = c.head_dim, c.page_size
        if page_ids is None:
            page_ids = self.all_page_ids(layer, kv_head, seq)
        dt = getattr(self, "kivi_dtype", torch.float32)
        pf = int(self.view("prefill_tokens")[seq, layer, kv_head].item())
        cs = self.view("k_chan_scale")[seq, layer, kv_head]
        kw = self.view("k_window")[seq, layer, kv_head]
        Ks, Vs, lens = [], [], []
        for p in page_ids:
            n = int(self.view("valid")[seq, layer, kv_head, p].item())
            lens.append(n)
            if n == 0:
                continue
            kc = unpack_codes_2d(self.view("k_codes")[seq, layer, kv_head, p, :n].contiguous(), c.base_bits, D)
            vc = unpack_codes_2d(self.view("v_codes")[seq, layer, kv_head, p, :n].contiguous(), c.base_bits, D)
            vs = self.view("v_scale")[seq, layer, kv_head, p, :n]                       # [n, 1]
            kh = (kc.float() * cs.unsqueeze(0)).to(dt).to(torch.float16)
            npk = max(0, min(n, pf - p * T))
            if npk < n:
                kh[npk:] = kw[p - pf // T, npk:n]
            Ks.append(kh)
            Vs.append((vc.float() * vs).to(dt).to(torch.float16))
        if not Ks:
            z = torch.zeros(0, D, dtype=torch.float16, device=self.device)
            return z, z, lens
        return torch.cat(Ks), torch.cat(Vs), lens

    def read_counters(self):
        rc = self.view("read_counter")
        return int(rc[..., 0].sum().item()), int(rc[..., 1].sum().item())
