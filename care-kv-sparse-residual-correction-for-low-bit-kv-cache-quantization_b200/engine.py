"""DecodeEngine: host driver of the cache path over the C ABI.

It owns nothing but the decode workspace; the cache arena is a CAREKVCache.
Per layer and step the engine issues at most three kernel launches:
carekv_append (plus the page-full store on steps where a page completes),
and carekv_decode_attention (split-K pass + route/correct).  Host-side token
counts (``cache.lengths``) decide capacity, the workspace page stride and
whether a page can complete, so no call reads device memory back.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence, Tuple

import torch

from . import _lib
from .cache import CAREKVCache
from .config import legacy_router, resolve_route_params, resolve_store_params


def decode_router(router: Optional[str] = None) -> str:
    """The decode router: "vectorized" (default) or "cached"."""
    r = (router or os.environ.get("CAREKV_DECODE_ROUTER", "vectorized")).lower()
    if r not in ("vectorized", "cached"):
        raise ValueError(f"decode router {r!r}: vectorized or cached")
    return r

_DT = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


class DecodeEngine:
    """shard = (kvh_begin, kvh_total): the cache holds kv heads [kvh_begin,
    kvh_begin + cfg.num_kv_heads) of a model with kvh_total kv heads, and the
    engine takes the model's full activation rows (k / v [n, kvh_total, D],
    q / out [n, kvh_total * QN, D]), touching only its own heads (the C
    ABI's _shard entry points).  None: the cache holds every kv head."""

    def __init__(self, cache: CAREKVCache, shard: Optional[Tuple[int, int]] = None):
        self.cache = cache
        self.cfg = cache.cfg
        self._ws = None
        self._ws_bytes = 0
        H = self.cfg.num_kv_heads
        if shard is None:
            shard = (0, H)
        b0, tot = int(shard[0]), int(shard[1])
        if b0 < 0 or b0 + H > tot:
            raise ValueError(f"shard {shard}: kv heads [{b0}, {b0 + H}) do not fit {tot}")
        self.shard = _lib.Shard(b0, tot)
        self.kvh_total = tot
        self.qn = self.cfg.num_heads // H

    # ── helpers ───────────────────────────────────────────────────────
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.cache.device).cuda_stream

    def _check_tensor(self, t: torch.Tensor, shape, what):
        if not t.is_cuda or t.device != self.cache.device:
            raise RuntimeError(f"{what}: expected a tensor on {self.cache.device}, got {t.device}")
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"{what}: expected shape {tuple(shape)}, got {tuple(t.shape)}")
        if t.dtype not in _DT:
            raise ValueError(f"{what}: unsupported dtype {t.dtype}")
        return t.contiguous()

    def pages_used(self, layer: int, seq_begin: int, seq_count: int, extra_tokens: int = 0) -> int:
        T = self.cfg.page_size
        n = max((self.cache.lengths[b][layer] + extra_tokens for b in range(seq_begin, seq_begin + seq_count)),
                default=0)
        return (n + T - 1) // T

    def workspace(self, nbytes: int) -> torch.Tensor:
        if self._ws is None or self._ws_bytes < nbytes:
            self._ws = torch.empty(nbytes, dtype=torch.uint8, device=self.cache.device)
            self._ws_bytes = nbytes
        return self._ws

    def workspace_bytes(self, seq_count: int, pages: int) -> int:
        n = ctypes.c_size_t(0)
        _lib.check(_lib.lib().carekv_decode_workspace_bytes(ctypes.byref(self.cache.ccfg), seq_count, pages,
                                                            ctypes.byref(n)), "carekv_decode_workspace_bytes")
        return int(n.value)

    def _sketch_ptr(self):
        return self.cache.sketch_proj().data_ptr() if self.cfg.store_sketch else None

    # ── prefill store ─────────────────────────────────────────────────
    def prefill_store(self, layer: int, K: torch.Tensor, V: torch.Tensor, seq_begin: int = 0,
                      token_start: int = 0, sink_tokens: int = 4):
        """Write T rows per (sequence, kv head): K, V [seq_count, Hkv, T, D]."""
        cfg = self.cfg
        n, H, T, D = K.shape
        K = self._check_tensor(K, (n, self.kvh_total, T, cfg.head_dim), "prefill K")
        V = self._check_tensor(V, (n, self.kvh_total, T, cfg.head_dim), "prefill V")
        if K.dtype != V.dtype:
            raise ValueError("K and V must share a dtype")
        n_new = (T + cfg.page_size - 1) // cfg.page_size
        for b in range(seq_begin, seq_begin + n):
            if self._pages(b, layer) + n_new > cfg.max_pages:
                raise _lib.CacheFullError(_lib.ERR_CACHE_FULL, "prefill_store")
            if cfg.is_kivi and self._pages(b, layer) > 0:
                # the per-channel K scales span one prefill (kivi_helpers.py:35-47)
                raise NotImplementedError("KIVI base: one prefill per sequence and layer, before any append")
        if cfg.is_kivi:
            self.cache.kivi_dtype = K.dtype
        sp = resolve_store_params(cfg, layer, _DT[K.dtype], token_start, sink_tokens)
        _lib.check(_lib.lib().carekv_prefill_store_shard(
            ctypes.byref(self.cache.ccfg), ctypes.byref(self.cache.c), layer, K.data_ptr(), V.data_ptr(), T,
            seq_begin, n, ctypes.byref(sp), self._sketch_ptr(), ctypes.byref(self.shard), self._stream()),
            "carekv_prefill_store")
        if T > 0:
            last = T % cfg.page_size or cfg.page_size
            for b in range(seq_begin, seq_begin + n):
                self._state()[(b, layer)] = (self._pages(b, layer) + n_new, last)
                self.cache.lengths[b][layer] += T
                if cfg.is_kivi:
                    self._kivi_prefill()[(b, layer)] = T

    # ── decode ────────────────────────────────────────────────────────
    def append(self, layer: int, k: torch.Tensor, v: torch.Tensor, seq_begin: int = 0):
        """Append one token per sequence: k, v [seq_count, Hkv, D]."""
        cfg = self.cfg
        n = k.shape[0]
        k = self._check_tensor(k, (n, self.kvh_total, cfg.head_dim), "append k")
        v = self._check_tensor(v, (n, self.kvh_total, cfg.head_dim), "append v")
        T = cfg.page_size
        may_fill = 0
        for b in range(seq_begin, seq_begin + n):
            pages, last = self._state().get((b, layer), (0, 0))
            if pages == 0 or last >= T:
                if pages + 1 > cfg.max_pages:
                    raise _lib.CacheFullError(_lib.ERR_CACHE_FULL, "append")
                last = 0
                pages += 1
            if not self.kivi_window_ok(b, layer, pages - 1):
                raise _lib.CacheFullError(_lib.ERR_CACHE_FULL, "append (KIVI fp16 K window)")
            if last + 1 == T:
                may_fill = 1       # this append completes a page: run the page store
        sp = resolve_store_params(cfg, layer, _DT[k.dtype])
        _lib.check(_lib.lib().carekv_append_shard(ctypes.byref(self.cache.ccfg), ctypes.byref(self.cache.c), layer,
                                                  k.data_ptr(), v.data_ptr(), seq_begin, n, ctypes.byref(sp),
                                                  self._sketch_ptr(), may_fill, ctypes.byref(self.shard),
                                                  self._stream()), "carekv_append")
        for b in range(seq_begin, seq_begin + n):
            self._advance(b, layer)

    def attend(self, layer: int, q: torch.Tensor, out: Optional[torch.Tensor] = None, seq_begin: int = 0,
               kind: Optional[str] = None, correction: bool = True, score_normalize=None, k_corr_scale=None,
               pages: Optional[int] = None, router: Optional[str] = None) -> torch.Tensor:
        """Decode attention for [seq_count, Hq, D] queries against the cache.
        router: "vectorized" (vectorized_joint_correction per kv head, the
        default) or "cached" (the reference decode step's ResidualRouter.route
        + apply_slot_corrections per query head); None reads
        CAREKV_DECODE_ROUTER."""
        cfg = self.cfg
        n = q.shape[0]
        q = self._check_tensor(q, (n, self.kvh_total * self.qn, cfg.head_dim), "decode q")
        if out is None:
            out = torch.empty_like(q) if self.kvh_total == cfg.num_kv_heads else torch.zeros_like(q)
        if pages is None:
            pages = max(1, max((self._pages(b, layer) for b in range(seq_begin, seq_begin + n)), default=1))
        rp = resolve_route_params(cfg, layer, kind=kind, score_normalize=score_normalize,
                                  k_corr_scale=k_corr_scale, legacy=decode_router(router) == "cached")
        if not correction:
            rp.kind = _lib.KIND_NONE
        nbytes = self.workspace_bytes(n, pages)
        ws = self.workspace(nbytes)
        _lib.check(_lib.lib().carekv_decode_attention_shard(
            ctypes.byref(self.cache.ccfg), ctypes.byref(self.cache.c), layer, q.data_ptr(), out.data_ptr(),
            _DT[q.dtype], seq_begin, n, pages, ctypes.byref(rp), self._sketch_ptr(), ws.data_ptr(), ws.numel(),
            ctypes.byref(self.shard), self._stream()), "carekv_decode_attention")
        return out

    def prefill_correct(self, layer: int, seq: int, q: torch.Tensor, attn: torch.Tensor, o_base: torch.Tensor,
                        o_exact: Optional[torch.Tensor] = None, attn_sum: Optional[torch.Tensor] = None,
                        logits: Optional[torch.Tensor] = None, row_max: Optional[torch.Tensor] = None,
                        v_rows: Optional[torch.Tensor] = None, v_pnorm: Optional[torch.Tensor] = None,
                        out: Optional[torch.Tensor] = None, kind: Optional[str] = None, score_normalize=None,
                        k_corr_scale=None, legacy: Optional[bool] = None) -> torch.Tensor:
        """Stored-slot correction of a prefill (layer.py:458-637): one route /
        correct pass per (prefill position, kv head) over the slots of
        sequence `seq`.  With P = the sequence's pages and QN = Hq / Hkv:
        q [T, Hq, D]; attn, logits [T, Hkv, QN, P*16] fp32; attn_sum, row_max
        [T, Hkv, QN] fp32; o_base, o_exact [T, Hkv, QN, D] fp32; v_rows
        [Hkv, P*16, D] fp32; v_pnorm [Hkv, P] fp32.  Returns [T, Hq, D].
        legacy: the cached router (ResidualRouter.route per query, the
        reference's prefill correction unless correction_impl is
        "vectorized", layer.py:522-630); None follows cfg.correction_impl."""
        cfg = self.cfg
        T = q.shape[0]
        H, QN, D = cfg.num_kv_heads, cfg.num_heads // cfg.num_kv_heads, cfg.head_dim
        P = self._pages(seq, layer)
        if P == 0:
            raise ValueError("prefill_correct: the sequence holds no pages")
        q = self._check_tensor(q, (T, cfg.num_heads, D), "prefill q")

        def f32(t, shape, what, optional=True):
            if t is None:
                if optional:
                    return None
                raise ValueError(f"{what} is required")
            if t.dtype != torch.float32:
                raise ValueError(f"{what}: expected float32, got {t.dtype}")
            return self._check_tensor(t, shape, what)
        attn = f32(attn, (T, H, QN, P * cfg.page_size), "attn", optional=False)
        o_base = f32(o_base, (T, H, QN, D), "o_base", optional=False)
        o_exact = f32(o_exact, (T, H, QN, D), "o_exact")
        attn_sum = f32(attn_sum, (T, H, QN), "attn_sum")
        logits = f32(logits, (T, H, QN, P * cfg.page_size), "logits")
        row_max = f32(row_max, (T, H, QN), "row_max")
        v_rows = f32(v_rows, (H, P * cfg.page_size, D), "v_rows")
        v_pnorm = f32(v_pnorm, (H, P), "v_pnorm")
        if out is None:
            out = torch.empty_like(q)
        if legacy is None:
            legacy = legacy_router(cfg)
        rp = resolve_route_params(cfg, layer, kind=kind, score_normalize=score_normalize, k_corr_scale=k_corr_scale,
                                  legacy=legacy)
        n = ctypes.c_size_t(0)
        _lib.check(_lib.lib().carekv_prefill_workspace_bytes(ctypes.byref(self.cache.ccfg), T, P, ctypes.byref(n)),
                   "carekv_prefill_workspace_bytes")
        ws = self.workspace(int(n.value))

        def ptr(t):
            return t.data_ptr() if t is not None else None
        _lib.check(_lib.lib().carekv_prefill_correction(
            ctypes.byref(self.cache.ccfg), ctypes.byref(self.cache.c), layer, seq, T, P, q.data_ptr(), ptr(logits),
            ptr(row_max), attn.data_ptr(), ptr(attn_sum), o_base.data_ptr(), ptr(o_exact), ptr(v_rows),
            ptr(v_pnorm), out.data_ptr(), _DT[q.dtype], ctypes.byref(rp), self._sketch_ptr(), ws.data_ptr(),
            ws.numel(), self._stream()), "carekv_prefill_correction")
        return out

    # ── host mirror of the page state ─────────────────────────────────
    # The device keeps num_pages / valid; the host mirrors them per
    # (sequence, layer) as (pages, valid rows of the last page).
    def _state(self):
        st = getattr(self.cache, "_page_state", None)
        if st is None:
            st = {}
            self.cache._page_state = st
        return st

    def _pages(self, b, layer):
        return self._state().get((b, layer), (0, 0))[0]

    def _kivi_prefill(self):
        st = getattr(self.cache, "_kivi_pf", None)
        if st is None:
            st = {}
            self.cache._kivi_pf = st
        return st

    def kivi_window_ok(self, b, layer, page) -> bool:
        """KIVI base: a decode-appended row of `page` has a place in the fp16
        K window (pages prefill_tokens // page_size + w, w < kivi_window_pages)."""
        if not self.cfg.is_kivi:
            return True
        wp = page - self._kivi_prefill().get((b, layer), 0) // self.cfg.page_size
        return 0 <= wp < self.cfg.kivi_window_pages

    def _last_page_valid(self, b, layer):
        return self._state().get((b, layer), (0, 0))[1]

    def _advance(self, b, layer):
        T = self.cfg.page_size
        pages, last = self._state().get((b, layer), (0, 0))
        if pages == 0 or last >= T:
            pages, last = pages + 1, 1
        else:
            last += 1
        self._state()[(b, layer)] = (pages, last)
        self.cache.lengths[b][layer] += 1

    # ── parity readback (tests) ───────────────────────────────────────
    def _sel_stride(self, pages: int) -> int:
        cfg = self.cache.ccfg
        return 1 + pages * (cfg.k_slots_per_page + cfg.v_slots_per_page)

    def last_selection(self, layer: int, seq_begin: int, seq_count: int, pages: int, cache_seq: Optional[int] = None):
        """Selected slots of the last attend(): {(seq, kv_head, query): [(kind, page, group), ...]}.

        Reads the workspace region the route kernel publishes and maps grid
        indices back to (\"K\", page, channel group) / (\"V\", page, token block)
        through the cache's slot tables.  Synchronizes the device.  After
        prefill_correct, pass seq_count = the prefill positions and cache_seq =
        the sequence: rows are then (position, kv_head, query).
        """
        cfg = self.cache.ccfg
        qn = cfg.num_heads // cfg.num_kv_heads
        n_bh = seq_count * cfg.num_kv_heads
        stride = self._sel_stride(pages)
        sel = self._ws[: n_bh * qn * stride * 4].view(torch.int32).view(n_bh, qn, stride)
        sel = sel.cpu()
        SK, SV = cfg.k_slots_per_page, cfg.v_slots_per_page
        KG = pages * SK
        kg = self.cache.view("k_slot_group").cpu() if SK else None
        vb = self.cache.view("v_slot_block").cpu() if SV else None
        out = {}
        for bh in range(n_bh):
            s, h = divmod(bh, cfg.num_kv_heads)
            b = seq_begin + s if cache_seq is None else cache_seq
            for i in range(qn):
                n = int(sel[bh, i, 0])
                items = []
                for e in sel[bh, i, 1:1 + n].tolist():
                    if e < KG:
                        p, j = divmod(e, SK)
                        items.append(("K", p, int(kg[b, layer, h, p, j])))
                    else:
                        p, j = divmod(e - KG, SV)
                        items.append(("V", p, int(vb[b, layer, h, p, j])))
                out[(seq_begin + s, h, i)] = items
        return out

    def last_scores(self, seq_count: int, pages: int):
        """Normalised scores of the last attend(): [seq_count*Hkv, qn, pages*(SK+SV)] (-1 = no slot)."""
        cfg = self.cache.ccfg
        qn = cfg.num_heads // cfg.num_kv_heads
        n_bh = seq_count * cfg.num_kv_heads
        off = (n_bh * qn * self._sel_stride(pages) * 4 + 255) // 256 * 256   # regions are 256-byte aligned
        ng = pages * (cfg.k_slots_per_page + cfg.v_slots_per_page)
        return self._ws[off: off + n_bh * qn * ng * 4].view(torch.float32).view(n_bh, qn, ng).clone()


class DecodeStepGraph:
    """One decode step over every layer, captured as CUDA graphs.

    Per layer the step appends the new K/V rows and runs decode attention
    (on the engine's kv-head shard: q / k / v / out are the model's rows)
    (three kernel launches; five on steps where a page completes).  Kernels
    read page counts from device memory, so one graph replays for every
    step; a second graph adds the page-full store and is replayed on the
    steps where the host page mirror says a page completes.  Step inputs
    live in fixed device buffers (q [L,B,Hq,D], k/v [L,B,Hkv,D]) and outputs
    land in out [L,B,Hq,D].

    host_io = (hq, hk, hv, ho), pinned host tensors shaped like q, k, v,
    out, puts the host transfers in the graph: layer l's inputs are copied in
    on a copy stream while earlier layers compute, and its output is copied
    back on a third stream as soon as the layer is done, so only the first
    layer's inputs and the last layer's output are exposed.
    """

    def __init__(self, engine: DecodeEngine, q, k, v, out, max_pages: int, correction: bool = True,
                 host_io=None):
        self.engine = engine
        self.cache = engine.cache
        self.cfg = engine.cfg
        self.q, self.k, self.v, self.out = q, k, v, out
        self.L, self.B = q.shape[0], q.shape[1]
        self.max_pages = max_pages
        self.correction = correction
        lib = _lib.lib()
        cache = self.cache
        dt = _DT[q.dtype]
        self.store_params = [resolve_store_params(self.cfg, l, dt) for l in range(self.L)]
        self.route_params = []
        for l in range(self.L):
            rp = resolve_route_params(self.cfg, l, legacy=decode_router() == "cached")
            if not correction:
                rp.kind = _lib.KIND_NONE
            self.route_params.append(rp)
        nbytes = engine.workspace_bytes(self.B, max_pages)
        self.ws = engine.workspace(nbytes)
        self.sketch = engine._sketch_ptr()
        self.host_io = host_io
        if host_io is not None:
            for h, d_ in zip(host_io, (q, k, v, out)):
                if h.device.type != "cpu" or not h.is_pinned() or h.shape != d_.shape or h.dtype != d_.dtype:
                    raise ValueError("host_io: pinned host tensors shaped like q, k, v, out")
        n = ctypes.c_int32(0)
        _lib.check(lib.carekv_decode_attention_launches(ctypes.byref(cache.ccfg), self.B, ctypes.byref(n)),
                   "carekv_decode_attention_launches")
        attend_launches = int(n.value)
        self.graphs = {}
        self.launches = {}
        stream = torch.cuda.Stream(cache.device)
        for fill in (0, 1):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                self._issue(fill, torch.cuda.current_stream(cache.device))
            self.graphs[fill] = g
            self.launches[fill] = self.L * ((3 if fill else 1) + attend_launches)

    def _issue(self, fill, stream):
        lib = _lib.lib()
        cache = self.cache
        st = stream.cuda_stream
        io = self.host_io
        if io is not None:
            hq, hk, hv, ho = io
            dev = cache.device
            copy_in, copy_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
            fork = torch.cuda.Event()
            fork.record(stream)
            copy_in.wait_event(fork)
            copy_out.wait_event(fork)
            ready = []
            with torch.cuda.stream(copy_in):
                for l in range(self.L):
                    self.q[l].copy_(hq[l], non_blocking=True)
                    self.k[l].copy_(hk[l], non_blocking=True)
                    self.v[l].copy_(hv[l], non_blocking=True)
                    e = torch.cuda.Event()
                    e.record(copy_in)
                    ready.append(e)
        for l in range(self.L):
            if io is not None:
                stream.wait_event(ready[l])
            shard = ctypes.byref(self.engine.shard)
            _lib.check(lib.carekv_append_shard(ctypes.byref(cache.ccfg), ctypes.byref(cache.c), l,
                                               self.k[l].data_ptr(), self.v[l].data_ptr(), 0, self.B,
                                               ctypes.byref(self.store_params[l]), self.sketch, fill, shard, st),
                       "carekv_append")
            _lib.check(lib.carekv_decode_attention_shard(
                ctypes.byref(cache.ccfg), ctypes.byref(cache.c), l, self.q[l].data_ptr(), self.out[l].data_ptr(),
                _DT[self.q.dtype], 0, self.B, self.max_pages, ctypes.byref(self.route_params[l]), self.sketch,
                self.ws.data_ptr(), self.ws.numel(), shard, st), "carekv_decode_attention")
            if io is not None:
                done = torch.cuda.Event()
                done.record(stream)
                copy_out.wait_event(done)
                with torch.cuda.stream(copy_out):
                    ho[l].copy_(self.out[l], non_blocking=True)
        if io is not None:
            for s_ in (copy_in, copy_out):
                j = torch.cuda.Event()
                j.record(s_)
                stream.wait_event(j)

    def next_fill(self) -> int:
        T = self.cfg.page_size
        for b in range(self.B):
            for l in range(self.L):
                pages, last = self.engine._state().get((b, l), (0, 0))
                if pages == 0 or last >= T:
                    if pages + 1 > min(self.cfg.max_pages, self.max_pages):
                        raise _lib.CacheFullError(_lib.ERR_CACHE_FULL, "decode step")
                    last = 0
                    pages += 1
                if not self.engine.kivi_window_ok(b, l, pages - 1):
                    raise _lib.CacheFullError(_lib.ERR_CACHE_FULL, "decode step (KIVI fp16 K window)")
                if last + 1 == T:
                    return 1
        return 0

    def replay(self) -> int:
        """Run one step; returns the number of kernel launches it issued."""
        fill = self.next_fill()
        self.graphs[fill].replay()
        for b in range(self.B):
            for l in range(self.L):
                self.engine._advance(b, l)
        return self.launches[fill]
