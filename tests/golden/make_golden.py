"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference CARE-KV package itself (pure PyTorch, CPU) on small
seeded inputs and writes ``tests/golden/*.npz``.  It needs the reference
source tree, so it runs only where that tree exists:

    python tests/golden/make_golden.py --reference /path/to/reference

The tree is imported as ``CARE_KV.care_kv`` through a temporary symlink
(the package uses relative imports and expects that name).  The fixtures
are committed; tests never import the reference.
"""

import argparse
import json
import math
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def import_reference(ref_root):
    tmp = tempfile.mkdtemp(prefix="carekv_ref_")
    os.makedirs(os.path.join(tmp, "CARE_KV"))
    open(os.path.join(tmp, "CARE_KV", "__init__.py"), "w").close()
    os.symlink(os.path.abspath(ref_root), os.path.join(tmp, "CARE_KV", "care_kv"))
    sys.dont_write_bytecode = True
    sys.path.insert(0, tmp)
    import CARE_KV.care_kv as ck  # noqa: F401
    return tmp


TORCH_DT = None


def tdt(name):
    import torch
    return {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}[name]


def as_np(t):
    import torch
    if t.dtype == torch.bfloat16 or t.dtype == torch.float16:
        t = t.float()
    return t.detach().cpu().numpy().copy()


# ───────────────────────────── quantizer ─────────────────────────────
def gen_quant(out):
    import torch
    from CARE_KV.care_kv.quantizer import (QuantConfig, quantize, dequantize,
                                          quantize_and_residual, pack_codes_2d)
    from CARE_KV.care_kv.residual_store import pack_4bit
    from CARE_KV.care_kv.cache import CacheConfig, CAREKVCache
    g = torch.Generator().manual_seed(1234)
    cases = []
    arrays = {}
    ci = 0
    for dt in ("fp32", "fp16", "bf16"):
        for bits in (2, 3, 4):
            for D, gs in ((64, 32), (128, 32), (128, 64)):
                x = torch.randn(16, D, generator=g) * 3.0
                x[:, 0] *= 20.0                      # outlier channel
                x[13:] = 0.0                         # zero padded rows
                x[5, gs:2 * gs] = 1e-3               # tiny group
                xt = x.to(tdt(dt))
                qc = QuantConfig(bits=bits, group_size=gs)
                codes, scale, resid, _ = quantize_and_residual(xt, qc)
                x_hat = dequantize(codes, scale, xt.shape, qc)
                packed = pack_codes_2d(codes, bits)
                # int8 page scales through the cache's own writer
                cfg = CacheConfig(num_layers=1, num_heads=1, num_kv_heads=1, head_dim=D,
                                  max_pages=1, base_bits=bits, group_size=gs,
                                  packed_base=True, scale_quant="int8")
                cache = CAREKVCache(cfg)
                cache.write_base(0, 0, 0, codes, scale, codes, scale, num_valid=13)
                # 4-bit residual slot of a block of the residual
                rp, rs = pack_4bit(resid.float()[:, :32])
                key = f"c{ci}"
                arrays[key + "_x"] = as_np(xt)
                arrays[key + "_codes"] = codes.numpy().copy()
                arrays[key + "_scale"] = as_np(scale)
                arrays[key + "_xhat"] = as_np(x_hat)
                arrays[key + "_resid"] = as_np(resid)
                arrays[key + "_packed"] = packed.numpy().view(np.uint8).copy()
                arrays[key + "_s8"] = cache.base_K_scale[0, 0, 0].numpy().copy()
                arrays[key + "_master"] = np.float32(cache.base_K_scale_master[0, 0, 0].float().item())
                arrays[key + "_r4"] = rp.numpy().view(np.uint8).copy()
                arrays[key + "_r4s"] = np.float32(rs.float().item())
                cases.append(dict(key=key, dt=dt, bits=bits, D=D, group_size=gs))
                ci += 1
    arrays["meta"] = np.array(json.dumps(cases))
    np.savez_compressed(os.path.join(out, "quant.npz"), **arrays)
    print("quant.npz", len(cases), "cases")


# ─────────────────────── prefill store + decode ───────────────────────
STORE_CASES = [
    # name, dt, D, bits, gs, T, scale_quant, store mode, sk, sv, ratio, policy, kind
    ("int3_d64_abs11", "fp32", 64, 3, 32, 40, "int8", "absolute", 1, 1, 0.0, "residual_kind_aware", "both"),
    ("int3_d128_abs24_f16", "fp16", 128, 3, 32, 40, "int8", "absolute", 2, 4, 0.0, "residual_kind_aware", "both"),
    ("int3_d64_abs24_bf16", "bf16", 64, 3, 32, 37, "int8", "absolute", 2, 4, 0.0, "residual_kind_aware", "both"),
    ("int2_d128_ratio", "fp16", 128, 2, 32, 48, "int8", "ratio", 0, 0, 0.1, "residual_kind_aware", "both"),
    ("int4_d128_g64_none", "fp32", 128, 4, 64, 33, "none", "absolute", 1, 2, 0.0, "residual_kind_aware", "both"),
    ("int3_d64_joint", "fp32", 64, 3, 32, 32, "int8", "ratio", 0, 0, 0.25, "joint", "both"),
    ("int3_d64_kind_v", "fp16", 64, 3, 32, 32, "int8", "absolute", 2, 2, 0.0, "residual_kind_aware", "v"),
]


def make_layer(cfg, Hq, Hkv, D, dt, seed):
    import torch
    from CARE_KV.care_kv.layer import CAREKVLayer
    g = torch.Generator().manual_seed(seed)
    dm = Hkv * D
    W_Q = (torch.randn(Hq * D, dm, generator=g) / math.sqrt(dm)).to(tdt(dt))
    W_K = torch.eye(dm).to(tdt(dt))
    W_V = (torch.randn(dm, dm, generator=g) / math.sqrt(dm)).to(tdt(dt))
    W_O = torch.eye(Hq * D, Hq * D).to(tdt(dt))
    return CAREKVLayer(cfg, 0, W_Q, W_K, W_V, W_O)


def dump_cache(cache, arrays, key):
    arrays[key + "_kcodes"] = cache.base_K_codes.numpy().view(np.uint8).copy()
    arrays[key + "_vcodes"] = cache.base_V_codes.numpy().view(np.uint8).copy()
    arrays[key + "_kscale"] = as_np(cache.base_K_scale)
    arrays[key + "_vscale"] = as_np(cache.base_V_scale)
    if cache.base_K_scale_master is not None:
        arrays[key + "_kmaster"] = as_np(cache.base_K_scale_master)
        arrays[key + "_vmaster"] = as_np(cache.base_V_scale_master)
    arrays[key + "_valid"] = cache.valid_tokens.numpy().copy()
    L, H, P = cache.valid_tokens.shape
    metas = []
    for l in range(L):
        for h in range(H):
            for p in range(cache.next_page[l][h]):
                m = cache.meta_table[l][h][p]
                if m is None:
                    continue
                metas.append(dict(l=l, h=h, p=p, k=list(m.k_residual_slots),
                                  v=list(m.v_residual_slots)))
                arrays[f"{key}_kerr_{l}_{h}_{p}"] = as_np(m.k_error_norm)
                arrays[f"{key}_verr_{l}_{h}_{p}"] = as_np(m.v_error_norm)
                arrays[f"{key}_ksk_{l}_{h}_{p}"] = as_np(m.k_sketch)
    arrays[key + "_meta"] = np.array(json.dumps(metas))
    nk = cache.num_stored_residual_slots()
    arrays[key + "_kbuf"] = cache.k_residual_buf[:nk[0]].numpy().view(np.uint8).copy()
    arrays[key + "_kbufs"] = as_np(cache.k_residual_scale[:nk[0], 0])
    arrays[key + "_vbuf"] = cache.v_residual_buf[:nk[1]].numpy().view(np.uint8).copy()
    arrays[key + "_vbufs"] = as_np(cache.v_residual_scale[:nk[1], 0])
    arrays[key + "_npages"] = np.array(cache.next_page, np.int32)


def gen_store(out):
    import torch
    from CARE_KV.care_kv.cache import CacheConfig, CAREKVCache
    arrays = {}
    cases = []
    os.environ["CAREKV_PREFILL_RESIDUAL_KIND"] = "both"
    for ci, (name, dt, D, bits, gs, T, sq, mode, sk, sv, ratio, policy, kind) in enumerate(STORE_CASES):
        os.environ["CAREKV_STORE_POLICY"] = policy
        os.environ["CAREKV_PREFILL_RESIDUAL_KIND"] = kind
        Hq, Hkv = 4, 2
        cfg = CacheConfig(num_layers=1, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, page_size=16,
                          max_pages=8, base_bits=bits, group_size=gs, k_channel_group=32,
                          v_token_block=4, sketch_dim=32, packed_base=True, scale_quant=sq,
                          store_budget_mode=mode, store_abs_k=sk, store_abs_v=sv,
                          store_budget_ratio=ratio, read_budget_ratio=0.0)
        layer = make_layer(cfg, Hq, Hkv, D, dt, 100 + ci)
        cache = CAREKVCache(cfg)
        g = torch.Generator().manual_seed(200 + ci)
        K = torch.randn(Hkv, T, D, generator=g)
        K[:, :, :4] *= 20.0
        V = torch.randn(Hkv, T, D, generator=g)
        Kt, Vt = K.to(tdt(dt)), V.to(tdt(dt))
        for h in range(Hkv):
            layer._write_pages_for_kv_head(cache, h, Kt[h], Vt[h], token_start_abs=0, sink_tokens=4)
        key = f"s{ci}"
        arrays[key + "_K"] = as_np(Kt)
        arrays[key + "_V"] = as_np(Vt)
        dump_cache(cache, arrays, key)
        # decode: append 20 tokens (crosses the partial page and fills a fresh one)
        steps = 20
        dm = Hkv * D
        hs = (torch.randn(steps, dm, generator=g)).to(tdt(dt))
        outs, qs, ks, vs = [], [], [], []
        rec = {}
        orig = layer.attn.forward

        def fwd(*a, **kw):
            r = orig(*a, **kw)
            rec["O"] = r
            return r
        layer.attn.forward = fwd
        for s in range(steps):
            h1 = hs[s:s + 1]
            q = (h1[0] @ layer.W_Q.T).reshape(Hq, D)
            k = (h1[0] @ layer.W_K.T).reshape(Hkv, D)
            v = (h1[0] @ layer.W_V.T).reshape(Hkv, D)
            layer.decode_step(cache, h1, position_embeddings=None)
            qs.append(as_np(q)); ks.append(as_np(k)); vs.append(as_np(v))
            outs.append(as_np(rec["O"]))
        arrays[key + "_dq"] = np.stack(qs)
        arrays[key + "_dk"] = np.stack(ks)
        arrays[key + "_dv"] = np.stack(vs)
        arrays[key + "_dO"] = np.stack(outs)
        dump_cache(cache, arrays, key + "d")
        cases.append(dict(key=key, name=name, dt=dt, D=D, bits=bits, group_size=gs, T=T,
                          scale_quant=sq, store_budget_mode=mode, store_abs_k=sk, store_abs_v=sv,
                          store_budget_ratio=ratio, store_policy=policy, kind=kind,
                          Hq=Hq, Hkv=Hkv, max_pages=8, steps=steps))
    os.environ["CAREKV_STORE_POLICY"] = "residual_kind_aware"
    os.environ["CAREKV_PREFILL_RESIDUAL_KIND"] = "both"
    arrays["meta"] = np.array(json.dumps(cases))
    np.savez_compressed(os.path.join(out, "store_decode.npz"), **arrays)
    print("store_decode.npz", len(cases), "cases")


# ───────────────────────────── correction ─────────────────────────────
CORR_CASES = [
    # name, D, Hq, Hkv, N, sk, sv, read mode, rk, rv, ratio, kind, policy, norm, live, kmode
    ("paper_best_cfg1", 64, 32, 4, 512, 1, 1, "ratio", 0, 0, 0.03, "both", "joint", True, True, "exact"),
    ("paper_best_abs", 128, 8, 2, 160, 2, 4, "absolute", 2, 4, 0.0, "both", "joint", True, True, "exact"),
    ("linear_live", 64, 8, 2, 96, 2, 2, "absolute", 2, 2, 0.0, "both", "joint", True, True, "linear"),
    ("proxy_exact", 64, 8, 2, 96, 2, 2, "absolute", 2, 2, 0.0, "both", "joint", True, False, "exact"),
    ("separate", 64, 8, 2, 96, 2, 2, "absolute", 1, 2, 0.0, "both", "separate", False, True, "exact"),
    ("kind_v", 64, 8, 2, 96, 2, 2, "absolute", 2, 2, 0.0, "v", "joint", True, True, "exact"),
    ("kind_k", 64, 8, 2, 96, 2, 2, "absolute", 2, 2, 0.0, "k", "joint", True, True, "exact"),
    ("read0", 64, 8, 2, 96, 2, 2, "absolute", 0, 0, 0.0, "both", "joint", True, True, "exact"),
    ("partial_pages", 64, 4, 1, 70, 2, 4, "absolute", 3, 3, 0.0, "both", "joint", True, True, "exact"),
]


def gen_correction(out):
    import torch
    import torch.nn.functional as F
    from CARE_KV.care_kv.cache import CacheConfig, CAREKVCache
    from CARE_KV.care_kv.quantizer import QuantConfig, dequantize
    from CARE_KV.care_kv.residual_router import ResidualRouter
    from CARE_KV.care_kv import attention as att
    arrays = {}
    cases = []
    for ci, (name, D, Hq, Hkv, N, sk, sv, rmode, rk, rv, ratio, kind, policy, norm, live, kmode) in enumerate(CORR_CASES):
        os.environ["CAREKV_KSCORE_LIVE"] = "1" if live else "0"
        os.environ["CAREKV_K_CORRECTION_MODE"] = kmode
        os.environ["CAREKV_STORE_POLICY"] = "residual_kind_aware"
        os.environ["CAREKV_PREFILL_RESIDUAL_KIND"] = "both"
        cfg = CacheConfig(num_layers=1, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, page_size=16,
                          max_pages=(N + 15) // 16 + 1, base_bits=3, group_size=32,
                          k_channel_group=32, v_token_block=4, sketch_dim=32, packed_base=True,
                          scale_quant="int8", store_budget_mode="absolute", store_abs_k=sk,
                          store_abs_v=sv, read_budget_mode=rmode, read_abs_k=rk, read_abs_v=rv,
                          read_budget_ratio=ratio, route_policy=policy)
        layer = make_layer(cfg, Hq, Hkv, D, "fp32", 300 + ci)
        cache = CAREKVCache(cfg)
        g = torch.Generator().manual_seed(ci)
        Q = torch.randn(Hq, D, generator=g)
        K = torch.randn(Hkv, N, D, generator=g)
        K[:, :, :4] *= 20.0
        V = torch.randn(Hkv, N, D, generator=g)
        for h in range(Hkv):
            layer._write_pages_for_kv_head(cache, h, K[h], V[h], token_start_abs=0, sink_tokens=4)
        router = ResidualRouter(cfg, 0, torch.device("cpu"))
        qc = QuantConfig(bits=3, group_size=32)
        key = f"r{ci}"
        grp = Hq // Hkv
        deltas, O_all = [], []
        for h in range(Hkv):
            pids = cache.all_page_ids(0, h)
            Kc, Ks, Vc, Vs, _ = cache.read_base_concat(0, h, pids)
            Nv = Kc.shape[0]
            Kb = dequantize(Kc, Ks, (Nv, D), qc).float()
            Vb = dequantize(Vc, Vs, (Nv, D), qc).float()
            Qq = Q[h * grp:(h + 1) * grp].float()
            S = (Kb @ Qq.T).T * (1.0 / math.sqrt(D))
            A = F.softmax(S, dim=-1)
            O = A @ Vb
            rec = []
            att.set_chunk_recorder(rec)
            stats = {}
            delta = att.vectorized_joint_correction(
                cache, cfg, router, 0, h, pids, Q_q=Qq, S=S, A=A, V_base=Vb, O_base=O,
                kind=kind, k_corr_scale=0.1, score_normalize=norm, debug_stats=stats)
            att.set_chunk_recorder(None)
            r = rec[-1] if rec else {}
            arrays[f"{key}_S_{h}"] = S.numpy()
            arrays[f"{key}_A_{h}"] = A.numpy()
            arrays[f"{key}_O_{h}"] = O.numpy()
            arrays[f"{key}_delta_{h}"] = delta.numpy()
            for nm in ("score_K", "score_V", "sel_k", "sel_v"):
                v = r.get(nm)
                if v is not None:
                    arrays[f"{key}_{nm}_{h}"] = v.numpy()
            arrays[f"{key}_reads_{h}"] = np.array([stats.get("k_slots_read", 0),
                                                   stats.get("v_slots_read", 0)], np.int64)
        arrays[key + "_Q"] = Q.numpy()
        arrays[key + "_K"] = K.numpy()
        arrays[key + "_V"] = V.numpy()
        cases.append(dict(key=key, name=name, D=D, Hq=Hq, Hkv=Hkv, N=N, store_abs_k=sk,
                          store_abs_v=sv, read_budget_mode=rmode, read_abs_k=rk, read_abs_v=rv,
                          read_budget_ratio=ratio, kind=kind, route_policy=policy,
                          score_normalize=norm, kscore_live=live, k_correction_mode=kmode,
                          max_pages=cfg.max_pages))
    for k in ("CAREKV_KSCORE_LIVE", "CAREKV_K_CORRECTION_MODE"):
        os.environ.pop(k, None)
    arrays["meta"] = np.array(json.dumps(cases))
    np.savez_compressed(os.path.join(out, "correction.npz"), **arrays)
    print("correction.npz", len(cases), "cases")


# ───────────────────────────── KIVI helpers ─────────────────────────────
def gen_kivi(out):
    """quant_dequant_kivi_k / _v (kivi_helpers.py:35-59) on seeded (B, H, T, D)."""
    import torch
    from CARE_KV.care_kv.kivi_helpers import quant_dequant_kivi_k, quant_dequant_kivi_v
    g = torch.Generator().manual_seed(77)
    arrays, cases = {}, []
    ci = 0
    for dt in ("fp32", "fp16", "bf16"):
        for bits in (2, 3, 4):
            for shape, special in (((1, 2, 19, 64), False), ((1, 2, 9, 128), True)):
                x = torch.randn(*shape, generator=g) * 3.0
                x[..., :2] *= 25.0
                if special:
                    x[0, 0, :, 5] = 0.0        # an all-zero channel (K scale)
                    x[0, 1, 3, :] = 0.0        # an all-zero token (V scale)
                x = x.to(tdt(dt))
                key = f"k{ci}"
                arrays[key + "_x"] = as_np(x)
                arrays[key + "_k"] = as_np(quant_dequant_kivi_k(x, bits))
                arrays[key + "_v"] = as_np(quant_dequant_kivi_v(x, bits))
                cases.append(dict(key=key, dtype=dt, bits=bits, shape=list(shape)))
                ci += 1
    arrays["meta"] = np.array(json.dumps(cases))
    np.savez_compressed(os.path.join(out, "kivi.npz"), **arrays)
    print("kivi.npz", len(cases), "cases")


# ───────────────────────────── KIVI-style base ─────────────────────────────
KIVI_STORE_CASES = [
    # name, dt, D, bits, T, store k, store v, steps
    ("kivi_int2_d128_bf16", "bf16", 128, 2, 70, 1, 1, 20),
    ("kivi_int2_d64_fp16", "fp16", 64, 2, 45, 2, 2, 20),
    ("kivi_int3_d64_fp32", "fp32", 64, 3, 50, 1, 2, 20),
    ("kivi_int4_d128_bf16", "bf16", 128, 4, 33, 2, 1, 20),
]


def dump_kivi(cache, arrays, key):
    """The fp16 side buffers (cache.py:487-499), valid counts and slots."""
    arrays[key + "_khat"] = as_np(cache.base_K_hat_fp16)
    arrays[key + "_vhat"] = as_np(cache.base_V_hat_fp16)
    arrays[key + "_valid"] = cache.valid_tokens.numpy().copy()
    L, H, P = cache.valid_tokens.shape
    metas = []
    for l in range(L):
        for h in range(H):
            for p in range(cache.next_page[l][h]):
                m = cache.meta_table[l][h][p]
                if m is None:
                    continue
                metas.append(dict(l=l, h=h, p=p, k=list(m.k_residual_slots), v=list(m.v_residual_slots)))
                arrays[f"{key}_kerr_{l}_{h}_{p}"] = as_np(m.k_error_norm)
                arrays[f"{key}_verr_{l}_{h}_{p}"] = as_np(m.v_error_norm)
    arrays[key + "_meta"] = np.array(json.dumps(metas))
    nk = cache.num_stored_residual_slots()
    arrays[key + "_kbuf"] = cache.k_residual_buf[:nk[0]].numpy().view(np.uint8).copy()
    arrays[key + "_kbufs"] = as_np(cache.k_residual_scale[:nk[0], 0])
    arrays[key + "_vbuf"] = cache.v_residual_buf[:nk[1]].numpy().view(np.uint8).copy()
    arrays[key + "_vbufs"] = as_np(cache.v_residual_scale[:nk[1], 0])
    arrays[key + "_npages"] = np.array(cache.next_page, np.int32)


def gen_kivi_store(out):
    """KIVI-style base (base_quantizer='kivi_style'): the prefill store
    (layer.py:230-297), then decode appends through CAREKVLayer.decode_step
    (layer.py:1037-1101) with their base attention outputs."""
    import torch
    from CARE_KV.care_kv.cache import CacheConfig, CAREKVCache
    arrays, cases = {}, []
    os.environ["CAREKV_STORE_POLICY"] = "residual_kind_aware"
    os.environ["CAREKV_PREFILL_RESIDUAL_KIND"] = "both"
    for ci, (name, dt, D, bits, T, sk, sv, steps) in enumerate(KIVI_STORE_CASES):
        Hq, Hkv = 4, 2
        cfg = CacheConfig(num_layers=1, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, page_size=16,
                          max_pages=8, base_bits=bits, group_size=32, k_channel_group=32, v_token_block=4,
                          sketch_dim=32, packed_base=True, scale_quant="none", store_budget_mode="absolute",
                          store_abs_k=sk, store_abs_v=sv, read_budget_ratio=0.0, base_quantizer="kivi_style")
        layer = make_layer(cfg, Hq, Hkv, D, dt, 400 + ci)
        cache = CAREKVCache(cfg)
        g = torch.Generator().manual_seed(500 + ci)
        K = torch.randn(Hkv, T, D, generator=g)
        K[:, :, :4] *= 20.0
        V = torch.randn(Hkv, T, D, generator=g)
        Kt, Vt = K.to(tdt(dt)), V.to(tdt(dt))
        for h in range(Hkv):
            layer._write_pages_for_kv_head(cache, h, Kt[h], Vt[h], token_start_abs=0, sink_tokens=4)
        key = f"k{ci}"
        arrays[key + "_K"] = as_np(Kt)
        arrays[key + "_V"] = as_np(Vt)
        dump_kivi(cache, arrays, key)
        dm = Hkv * D
        hs = torch.randn(steps, dm, generator=g).to(tdt(dt))
        outs, qs, ks, vs = [], [], [], []
        rec = {}
        orig = layer.attn.forward

        def fwd(*a, **kw):
            r = orig(*a, **kw)
            rec["O"] = r
            return r
        layer.attn.forward = fwd
        for s_ in range(steps):
            h1 = hs[s_:s_ + 1]
            qs.append(as_np((h1[0] @ layer.W_Q.T).reshape(Hq, D)))
            ks.append(as_np((h1[0] @ layer.W_K.T).reshape(Hkv, D)))
            vs.append(as_np((h1[0] @ layer.W_V.T).reshape(Hkv, D)))
            layer.decode_step(cache, h1, position_embeddings=None)
            outs.append(as_np(rec["O"]))
        arrays[key + "_dq"] = np.stack(qs)
        arrays[key + "_dk"] = np.stack(ks)
        arrays[key + "_dv"] = np.stack(vs)
        arrays[key + "_dO"] = np.stack(outs)
        dump_kivi(cache, arrays, key + "d")
        cases.append(dict(key=key, name=name, dt=dt, D=D, bits=bits, T=T, store_abs_k=sk, store_abs_v=sv,
                          Hq=Hq, Hkv=Hkv, max_pages=8, steps=steps))
    arrays["meta"] = np.array(json.dumps(cases))
    np.savez_compressed(os.path.join(out, "kivi_store.npz"), **arrays)
    print("kivi_store.npz", len(cases), "cases")


# ───────────────────────────── legacy cached router ─────────────────────────────
LEGACY_CASES = [
    # name, D, Hkv, T, store (k, v), read mode, rk, rv, ratio, policy, normalize, kmode, kind, baseline,
    # rel, abs, min_keep
    ("joint_norm_exact", 64, 2, 150, (2, 2), "absolute", 2, 2, 0.03, "joint", True, "exact", "both", "carekv", 0, 0, 0),
    ("separate_linear", 64, 2, 150, (2, 2), "absolute", 2, 3, 0.03, "separate", False, "linear", "both", "carekv",
     0, 0, 0),
    ("k_first_exact", 64, 2, 150, (2, 2), "absolute", 2, 3, 0.03, "k_first", True, "exact", "both", "carekv", 0, 0, 0),
    ("adaptive_exact", 64, 2, 150, (2, 2), "absolute", 3, 3, 0.03, "adaptive", True, "exact", "both", "carekv",
     0, 0, 0),
    ("ratio_joint_d128", 128, 1, 260, (1, 1), "ratio", 0, 0, 0.05, "joint", True, "exact", "both", "carekv", 0, 0, 0),
    ("adaptive_score", 64, 2, 150, (2, 2), "adaptive_score", 3, 3, 0.03, "separate", True, "exact", "both", "carekv",
     0.3, 0.0, 1),
    ("magnitude_only", 64, 2, 150, (2, 2), "absolute", 2, 2, 0.03, "joint", True, "exact", "both", "magnitude_only",
     0, 0, 0),
    ("attention_only", 64, 2, 150, (2, 2), "absolute", 2, 2, 0.03, "separate", False, "linear", "both",
     "attention_only", 0, 0, 0),
    ("oracle_proxy", 64, 2, 150, (2, 2), "absolute", 2, 2, 0.03, "joint", True, "exact", "both", "oracle_proxy",
     0, 0, 0),
    ("kind_v", 64, 2, 150, (2, 2), "absolute", 2, 2, 0.03, "joint", False, "exact", "v", "carekv", 0, 0, 0),
    ("kind_k_joint_one_budget", 64, 2, 150, (2, 2), "absolute", 2, 0, 0.03, "joint", True, "exact", "k", "carekv",
     0, 0, 0),
]


def gen_legacy(out):
    """ResidualRouter.route + apply_slot_corrections through the reference's
    per-query-head CAREKVAttention.forward (attention.py:979-1039) on a
    prefilled cache with sketches, several queries per kv head."""
    import torch
    from CARE_KV.care_kv.cache import CacheConfig, CAREKVCache
    from CARE_KV.care_kv.attention import CAREKVAttention
    arrays, cases = {}, []
    os.environ["CAREKV_STORE_POLICY"] = "residual_kind_aware"
    os.environ["CAREKV_PREFILL_RESIDUAL_KIND"] = "both"
    for ci, (name, D, Hkv, T, (sk, sv), rmode, rk, rv, ratio, policy, norm, kmode, kind, base, rel, ab,
             mk) in enumerate(LEGACY_CASES):
        os.environ["CAREKV_K_CORRECTION_MODE"] = kmode
        Hq = Hkv * 2
        cfg = CacheConfig(num_layers=1, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, page_size=16, max_pages=24,
                          base_bits=3, group_size=32, k_channel_group=32, v_token_block=4, sketch_dim=32,
                          packed_base=True, scale_quant="int8", store_budget_mode="absolute", store_abs_k=sk,
                          store_abs_v=sv, read_budget_mode=rmode, read_abs_k=rk, read_abs_v=rv,
                          read_budget_ratio=ratio, route_policy=policy, baseline_score=base,
                          read_relative_threshold=float(rel), read_absolute_threshold=float(ab), read_min_keep=mk)
        layer = make_layer(cfg, Hq, Hkv, D, "fp32", 700 + ci)
        cache = CAREKVCache(cfg)
        g = torch.Generator().manual_seed(800 + ci)
        K = torch.randn(Hkv, T, D, generator=g)
        K[:, :, :4] *= 20.0
        V = torch.randn(Hkv, T, D, generator=g)
        for h in range(Hkv):
            layer._write_pages_for_kv_head(cache, h, K[h], V[h], token_start_abs=0, sink_tokens=4)
        att = CAREKVAttention(cfg, 0, torch.device("cpu"))
        rec = {}
        orig = att.router.route

        def route(*a, **kw):
            r = orig(*a, **kw)
            rec["sel"] = r
            return r
        att.router.route = route
        key = f"g{ci}"
        arrays[key + "_K"] = as_np(K)
        arrays[key + "_V"] = as_np(V)
        Q = torch.randn(Hkv, 4, D, generator=g)
        Q[:, 1] *= 3.0                   # sharper attention for the second query of each head
        arrays[key + "_Q"] = as_np(Q)
        outs, sels = [], []
        for h in range(Hkv):
            for j in range(4):
                rec.clear()
                o = att.forward(cache, h, Q[h, j], kind=kind, k_corr_scale=0.1, score_normalize=norm)
                outs.append(as_np(o))
                ksel, vsel = rec.get("sel", ([], []))
                sels.append(dict(k=[list(map(int, x)) for x in ksel], v=[list(map(int, x)) for x in vsel]))
        arrays[key + "_O"] = np.stack(outs)
        arrays[key + "_sel"] = np.array(json.dumps(sels))
        cases.append(dict(key=key, name=name, D=D, Hkv=Hkv, T=T, store_abs_k=sk, store_abs_v=sv, read_mode=rmode,
                          read_abs_k=rk, read_abs_v=rv, ratio=ratio, policy=policy, normalize=norm, kmode=kmode,
                          kind=kind, baseline=base, rel=rel, abs=ab, min_keep=mk, k_corr_scale=0.1))
    os.environ["CAREKV_K_CORRECTION_MODE"] = "exact"
    arrays["meta"] = np.array(json.dumps(cases))
    np.savez_compressed(os.path.join(out, "legacy_router.npz"), **arrays)
    print("legacy_router.npz", len(cases), "cases")


# ───────────────────────────── layer ─────────────────────────────
def gen_layer(out):
    """CAREKVLayer.prefill + decode_step of the reference (layer.py:643-1163)."""
    import torch
    sys.path.insert(0, HERE)
    from layer_case import LAYER_CASES, KIVI_LAYER_CASES, layer_inputs, layer_cfg_kwargs
    from CARE_KV.care_kv.cache import CacheConfig, CAREKVCache
    from CARE_KV.care_kv.layer import CAREKVLayer
    env = dict(CAREKV_K_CORRECTION_MODE="exact", CAREKV_KSCORE_LIVE="1", CAREKV_SCORE_NORMALIZE="1",
               CAREKV_PREFILL_RESIDUAL_KIND="both", CAREKV_STORE_POLICY="residual_kind_aware")
    arrays, cases = {}, []
    for ci, (name, Hq, Hkv, D, T, S, mode, seed, *base) in enumerate(LAYER_CASES + KIVI_LAYER_CASES):
        os.environ.update(env)
        os.environ["CAREKV_PREFILL_MODE"] = mode
        L = T + S
        W_Q, W_K, W_V, W_O, hid, cos, sin = [torch.from_numpy(x) for x in layer_inputs(Hq, Hkv, D, L, seed)]
        cfg = CacheConfig(**layer_cfg_kwargs(Hq, Hkv, D, L, *base))
        layer = CAREKVLayer(cfg, 0, W_Q, W_K, W_V, W_O)
        cache = CAREKVCache(cfg)
        pre = layer.prefill(cache, hid[:T], position_embeddings=(cos[:, :T], sin[:, :T]))
        dec = [layer.decode_step(cache, hid[T + j:T + j + 1], position_embeddings=(cos[:, T + j:T + j + 1],
                                                                               sin[:, T + j:T + j + 1]))
               for j in range(S)]
        key = f"l{ci}"
        arrays[key + "_prefill"] = as_np(pre)
        arrays[key + "_decode"] = as_np(torch.cat(dec, dim=0))
        cases.append(dict(key=key, name=name, Hq=Hq, Hkv=Hkv, D=D, T=T, steps=S, prefill_mode=mode, seed=seed,
                          base=base[0] if base else "uniform"))
    for k in list(env) + ["CAREKV_PREFILL_MODE"]:
        os.environ.pop(k, None)
    arrays["meta"] = np.array(json.dumps(cases))
    np.savez_compressed(os.path.join(out, "layer.npz"), **arrays)
    print("layer.npz", len(cases), "cases")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("CAREKV_REFERENCE"),
                    help="root of the reference project checkout (or set CAREKV_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", default="", help="comma list of quant,store,correction,layer,kivi,kivi_store,legacy")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give --reference (or CAREKV_REFERENCE): the reference checkout the fixtures come from")
    import_reference(a.reference)
    import torch
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    only = set(x for x in a.only.split(",") if x)
    for nm, fn in (("quant", gen_quant), ("store", gen_store), ("correction", gen_correction), ("layer", gen_layer),
                   ("kivi", gen_kivi), ("kivi_store", gen_kivi_store), ("legacy", gen_legacy)):
        if not only or nm in only:
            fn(a.out)


if __name__ == "__main__":
    main()
