"""Paged packed cache for one sequence (cache.py:416-904, layer.py:204-334, 1028-1146).

Holds the reference's logical state in numpy: packed base code rows, base
scales (int8 codes + one fp16 master per page, or raw fp16/bf16/fp32),
valid-token counts, per-page metadata (slot ids per channel group / token
block, error norms, sketches) and the two residual slot arenas with their
sequential free lists.
"""

import math

import numpy as np

from .numerics import round_to, F16, F32, BF16
from .quant import (quantize, dequantize, pack_codes_2d, unpack_codes_2d,
                    packed_row_bytes, int8_scale_write, int8_scale_read,
                    int8_scale_append, kivi_quant_dequant)
from .store import StoreConfig, process_page, sketch_projection


class OracleCache:
    def __init__(self, num_layers, num_kv_heads, head_dim, max_pages, store_cfg: StoreConfig,
                 page_size=16, scale_quant="int8", scale_dtype=F16, layer_sensitivity=None, base="uniform"):
        self.L, self.H, self.D, self.P, self.T = num_layers, num_kv_heads, head_dim, max_pages, page_size
        self.cfg = store_cfg
        self.bits = store_cfg.base_bits
        self.g = store_cfg.group_size
        self.G = head_dim // self.g
        self.rowB = packed_row_bytes(head_dim, self.bits)
        self.scale_quant = scale_quant
        self.scale_dtype = scale_dtype
        shp = (self.L, self.H, self.P)
        self.k_codes = np.zeros(shp + (self.T, self.rowB), np.uint8)
        self.v_codes = np.zeros(shp + (self.T, self.rowB), np.uint8)
        if scale_quant == "int8":
            self.k_scale = np.zeros(shp + (self.T, self.G), np.int8)
            self.v_scale = np.zeros(shp + (self.T, self.G), np.int8)
            self.k_master = np.zeros(shp, np.float32)
            self.v_master = np.zeros(shp, np.float32)
        else:
            self.k_scale = np.zeros(shp + (self.T, self.G), np.float32)
            self.v_scale = np.zeros(shp + (self.T, self.G), np.float32)
            self.k_master = self.v_master = None
        self.valid = np.zeros(shp, np.int32)
        self.next_page = np.zeros((self.L, self.H), np.int32)
        self.meta = [[[None] * self.P for _ in range(self.H)] for _ in range(self.L)]
        self.k_slots = {}      # slot id -> (packed uint8, fp16 scale)
        self.v_slots = {}
        self.next_k_slot = 0
        self.next_v_slot = 0
        self.sens = list(layer_sensitivity) if layer_sensitivity else [1.0] * self.L
        self.sketch_P = sketch_projection(head_dim, store_cfg.k_channel_group, store_cfg.sketch_dim)
        # KIVI-style base (kivi_style / kvquant_style): the reference keeps
        # K_hat / V_hat in an fp16 side buffer (cache.py:487-499, 800-865)
        self.base = base
        if base == "kivi":
            self.k_hat16 = np.zeros(shp + (self.T, head_dim), np.float32)
            self.v_hat16 = np.zeros(shp + (self.T, head_dim), np.float32)

    # ── base writes ─────────────────────────────────────────────────
    def _write_scale(self, which, l, h, p, scale_in, dt):
        """_write_scale_page (cache.py:592-606)."""
        buf = self.k_scale if which == "K" else self.v_scale
        if self.scale_quant == "int8":
            codes, master = int8_scale_write(scale_in, dt)
            buf[l, h, p] = codes
            (self.k_master if which == "K" else self.v_master)[l, h, p] = master
        else:
            buf[l, h, p] = round_to(scale_in, self.scale_dtype)

    def read_scale(self, which, l, h, p, rows=None):
        """_maybe_dequant_scale (cache.py:713-718): fp16 scales as float32."""
        buf = self.k_scale if which == "K" else self.v_scale
        s = buf[l, h, p] if rows is None else buf[l, h, p, :rows]
        if self.scale_quant == "int8":
            m = (self.k_master if which == "K" else self.v_master)[l, h, p]
            return int8_scale_read(s, m)
        return round_to(s, F16)

    def prefill_write(self, l, h, K, V, dt, token_start_abs=0, sink_tokens=4):
        """_write_pages_for_kv_head, uniform base (layer.py:204-334)."""
        if self.base == "kivi":
            return self._prefill_write_kivi(l, h, K, V, dt, token_start_abs, sink_tokens)
        T_all, D = K.shape
        ps = self.T
        num_pages = math.ceil(T_all / ps)
        cfg = self.cfg
        cfg.sensitivity = self.sens[l]
        out = []
        for p in range(num_pages):
            t0, t1 = p * ps, min((p + 1) * ps, T_all)
            nv = t1 - t0
            Kp = np.zeros((ps, D), np.float32)
            Vp = np.zeros((ps, D), np.float32)
            Kp[:nv] = K[t0:t1]
            Vp[:nv] = V[t0:t1]
            pid = int(self.next_page[l, h])
            assert pid < self.P, "KV cache is full"
            self.next_page[l, h] += 1
            is_sink = (token_start_abs + t0) < sink_tokens
            is_recent = p >= num_pages - 4
            Kc, Ks = quantize(Kp, self.bits, self.g, dt)
            Vc, Vs = quantize(Vp, self.bits, self.g, dt)
            self.k_codes[l, h, pid] = pack_codes_2d(Kc, self.bits)
            self.v_codes[l, h, pid] = pack_codes_2d(Vc, self.bits)
            self._write_scale("K", l, h, pid, Ks, dt)
            self._write_scale("V", l, h, pid, Vs, dt)
            self.valid[l, h, pid] = nv
            res = process_page(cfg, Kp, Vp, Kc, Ks, Vc, Vs, nv, dt,
                               is_recent=is_recent, is_sink=is_sink, sketch_P=self.sketch_P)
            self._commit_meta(l, h, pid, token_start_abs + t0, nv, res)
            out.append(res)
        return out

    def _prefill_write_kivi(self, l, h, K, V, dt, token_start_abs, sink_tokens):
        """_write_pages_for_kv_head, KIVI-style base (layer.py:230-297): K_hat
        per channel over the whole prefill, V_hat per token, both in dt
        (kivi_helpers.py:35-59); pages store fp16(K_hat) / fp16(V_hat) and the
        store runs against them (K_hat_override, residual_store.py:272-274)."""
        T_all, D = K.shape
        ps = self.T
        num_pages = math.ceil(T_all / ps)
        cfg = self.cfg
        cfg.sensitivity = self.sens[l]
        K = round_to(np.asarray(K, np.float32), dt)
        V = round_to(np.asarray(V, np.float32), dt)
        K_hat = kivi_quant_dequant(K, self.bits, dt, axis=-2)
        V_hat = kivi_quant_dequant(V, self.bits, dt, axis=-1)
        out = []
        for p in range(num_pages):
            t0, t1 = p * ps, min((p + 1) * ps, T_all)
            nv = t1 - t0
            Kp = np.zeros((ps, D), np.float32)
            Vp = np.zeros((ps, D), np.float32)
            Khp = np.zeros((ps, D), np.float32)
            Vhp = np.zeros((ps, D), np.float32)
            Kp[:nv], Vp[:nv] = K[t0:t1], V[t0:t1]
            Khp[:nv], Vhp[:nv] = K_hat[t0:t1], V_hat[t0:t1]
            pid = int(self.next_page[l, h])
            assert pid < self.P, "KV cache is full"
            self.next_page[l, h] += 1
            self.k_hat16[l, h, pid] = round_to(Khp, F16)
            self.v_hat16[l, h, pid] = round_to(Vhp, F16)
            self.valid[l, h, pid] = nv
            res = process_page(cfg, Kp, Vp, None, None, None, None, nv, dt,
                               is_recent=p >= num_pages - 4, is_sink=(token_start_abs + t0) < sink_tokens,
                               K_hat_override=Khp, V_hat_override=Vhp, sketch_P=self.sketch_P)
            self._commit_meta(l, h, pid, token_start_abs + t0, nv, res)
            out.append(res)
        return out

    def _commit_meta(self, l, h, pid, token_start, nv, res):
        """Slot allocation from the head of each free list (cache.py:548-560)."""
        num_cg = self.D // self.cfg.k_channel_group
        num_vb = math.ceil(self.T / self.cfg.v_token_block)
        k_ids = [-1] * num_cg
        v_ids = [-1] * num_vb
        for c in res["selected"]:
            if c["kind"] == "K":
                sid = self.next_k_slot
                self.next_k_slot += 1
                self.k_slots[sid] = (c["packed"], c["scale"])
                k_ids[c["idx"]] = sid
            else:
                sid = self.next_v_slot
                self.next_v_slot += 1
                self.v_slots[sid] = (c["packed"], c["scale"])
                v_ids[c["idx"]] = sid
        self.meta[l][h][pid] = dict(
            token_start=token_start, num_tokens=nv, k_slots=k_ids, v_slots=v_ids,
            k_err=res["k_err"], v_err=res["v_err"], k_sketch=res["k_sketch"])

    def append(self, l, h, k_row, v_row, dt, pos_abs=None):
        """decode_step append for one KV head (layer.py:1028-1146).

        Quantizes one row, appends it to the open page (a fresh page gets
        valid=0 and, under int8 scales, keeps master 0), and when the page
        fills re-runs the store with K_orig := K_hat (so every residual is 0
        and the page ends with no slots).
        """
        ps = self.T
        npg = int(self.next_page[l, h])
        if npg > 0 and self.valid[l, h, npg - 1] < ps:
            pid = npg - 1
        else:
            pid = npg
            assert pid < self.P, "KV cache is full"
            self.next_page[l, h] += 1
            self.valid[l, h, pid] = 0
        if self.base == "kivi":
            return self._append_kivi(l, h, pid, k_row, v_row, dt, pos_abs)
        kc, ks = quantize(np.asarray(k_row, np.float32)[None], self.bits, self.g, dt)
        vc, vs = quantize(np.asarray(v_row, np.float32)[None], self.bits, self.g, dt)
        off = int(self.valid[l, h, pid])
        assert off < ps, "page already full"
        self.k_codes[l, h, pid, off] = pack_codes_2d(kc, self.bits)[0]
        self.v_codes[l, h, pid, off] = pack_codes_2d(vc, self.bits)[0]
        if self.scale_quant == "int8":
            self.k_scale[l, h, pid, off] = int8_scale_append(ks[0], self.k_master[l, h, pid])
            self.v_scale[l, h, pid, off] = int8_scale_append(vs[0], self.v_master[l, h, pid])
        else:
            self.k_scale[l, h, pid, off] = round_to(ks[0], self.scale_dtype)
            self.v_scale[l, h, pid, off] = round_to(vs[0], self.scale_dtype)
        self.valid[l, h, pid] = off + 1
        if off + 1 == ps:
            # page full: process_page(K_orig=K_hat) -> all residuals exactly 0
            D = self.D
            Kc = unpack_codes_2d(self.k_codes[l, h, pid], self.bits, D)
            Vc = unpack_codes_2d(self.v_codes[l, h, pid], self.bits, D)
            Ks = self.read_scale("K", l, h, pid)
            Vs = self.read_scale("V", l, h, pid)
            K_hat = dequantize(Kc, Ks, self.g, F16)
            V_hat = dequantize(Vc, Vs, self.g, F16)
            cfg = self.cfg
            cfg.sensitivity = self.sens[l]
            if pos_abs is None:
                pos_abs = int(self.valid[l, 0, :self.next_page[l, 0]].sum()) - 1
            ts = pos_abs + 1 - ps
            sub = F16 if dt == F16 else F32
            res = process_page(cfg, round_to(K_hat, dt), round_to(V_hat, dt), Kc, Ks, Vc, Vs,
                               ps, dt, is_recent=True, is_sink=ts < 4, sketch_P=self.sketch_P,
                               hat_dt=F16, sub_dt=sub)
            self._commit_meta(l, h, pid, ts, ps, res)
        return pid, off

    def _append_kivi(self, l, h, pid, k_row, v_row, dt, pos_abs):
        """KIVI decode append (layer.py:1037-1101): the row's K quantized per
        channel over its one token, V per token, stored fp16; a page filled
        by decode is re-stored with K_orig := K_hat (every residual 0)."""
        ps = self.T
        k = round_to(np.asarray(k_row, np.float32)[None], dt)
        v = round_to(np.asarray(v_row, np.float32)[None], dt)
        off = int(self.valid[l, h, pid])
        assert off < ps, "page already full"
        self.k_hat16[l, h, pid, off] = round_to(kivi_quant_dequant(k, self.bits, dt, axis=-2)[0], F16)
        self.v_hat16[l, h, pid, off] = round_to(kivi_quant_dequant(v, self.bits, dt, axis=-1)[0], F16)
        self.valid[l, h, pid] = off + 1
        if off + 1 == ps:
            Kh = round_to(self.k_hat16[l, h, pid], dt)
            Vh = round_to(self.v_hat16[l, h, pid], dt)
            cfg = self.cfg
            cfg.sensitivity = self.sens[l]
            if pos_abs is None:
                pos_abs = int(self.valid[l, 0, :self.next_page[l, 0]].sum()) - 1
            ts = pos_abs + 1 - ps
            res = process_page(cfg, Kh, Vh, None, None, None, None, ps, dt, is_recent=True, is_sink=ts < 4,
                               K_hat_override=Kh, V_hat_override=Vh, sketch_P=self.sketch_P)
            self._commit_meta(l, h, pid, ts, ps, res)
        return pid, off

    # ── reads ───────────────────────────────────────────────────────
    def page_ids(self, l, h):
        return list(range(int(self.next_page[l, h])))

    def read_base_concat(self, l, h):
        """read_base_concat + dequantize (cache.py:720-772, attention.py:1009-1016).

        Returns K_hat, V_hat (N, D) float32 (fp16-exact values) and the
        per-page valid lengths.
        """
        Ks_all, Vs_all, lens = [], [], []
        for p in self.page_ids(l, h):
            n = int(self.valid[l, h, p])
            lens.append(n)
            if n == 0:
                continue
            if self.base == "kivi":   # read_base_hat_concat (cache.py:845-865)
                Ks_all.append(self.k_hat16[l, h, p, :n].copy())
                Vs_all.append(self.v_hat16[l, h, p, :n].copy())
                continue
            Kc = unpack_codes_2d(self.k_codes[l, h, p, :n], self.bits, self.D)
            Vc = unpack_codes_2d(self.v_codes[l, h, p, :n], self.bits, self.D)
            Ks = self.read_scale("K", l, h, p, rows=n)
            Vs = self.read_scale("V", l, h, p, rows=n)
            Ks_all.append(dequantize(Kc, Ks, self.g, F16))
            Vs_all.append(dequantize(Vc, Vs, self.g, F16))
        if not Ks_all:
            z = np.zeros((0, self.D), np.float32)
            return z, z, lens
        return np.concatenate(Ks_all), np.concatenate(Vs_all), lens

    def read_k_slot(self, sid):
        return self.k_slots[sid]

    def read_v_slot(self, sid):
        return self.v_slots[sid]
