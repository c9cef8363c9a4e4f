"""Legacy cached router (test infrastructure: the oracle of the GPU path).

Restates, per query head, ResidualRouter.route (residual_router.py:88-452)
and apply_slot_corrections (attention.py:208-374), the path the reference
takes whenever correction_impl is not "vectorized" (its decode step,
attention.py:1025-1038, and its cached prefill correction, layer.py:570-630):

* K slots are scored from their fp16 sketches: page attention mass x
  |q_sketch . k_sketch| x boundary risk x V difference x sensitivity (the
  "carekv" baseline score; magnitude_only / attention_only / oracle_proxy
  ablations, residual_router.py:185-212);
* V slots by block attention mass x error norm x sensitivity;
* budgets as _resolve_read_budgets, optional per-kind mean normalisation,
  the joint / separate / k_first / adaptive policies and the adaptive_score
  thresholds;
* the selected slots' correction: linear (V term + k_corr_scale x K
  Jacobian term) or the exact softmax renormalisation.

Ties keep Python's stable sort: candidates in page order, K before V.
"""

import math

import numpy as np

from .attention import exact_softmax_correction, resolve_read_budgets
from .quant import unpack_4bit

EPS = 1e-6


def _stable_desc(cands):
    return sorted(cands, key=lambda c: c[0], reverse=True)


def legacy_route(cache, l, h, q, s, a, O, V, rc, sketch_P, kind="both", score_normalize=False,
                 baseline="carekv", rel_thr=0.0, abs_thr=0.0, min_keep=0):
    """ResidualRouter.route for one query: returns (k_selected, v_selected)
    as lists of (page, group / block, slot id), plus the budgets."""
    q = np.asarray(q, np.float32)
    if a.size == 0:
        return [], [], (0, 0)
    s_top = np.float32(s.max())
    kcg = rc.k_channel_group
    num_cg = rc.head_dim // kcg
    q_sk = [q[cg * kcg:(cg + 1) * kcg] @ sketch_P for cg in range(num_cg)]
    sens = np.float32(rc.sensitivity)
    k_c, v_c = [], []
    off = 0
    for pid in cache.page_ids(l, h):
        meta = cache.meta[l][h][pid]
        n = int(cache.valid[l, h, pid])
        if n == 0 or meta is None:
            continue                      # the route's cursor skips such pages (residual_router.py:170-172)
        pa, ps_, pV = a[off:off + n], s[off:off + n], V[off:off + n]
        mass = np.float32(pa.sum(dtype=np.float32))
        margins = np.maximum(s_top - ps_, np.float32(EPS))
        bnd = np.float32((pa * (np.float32(1.0) / margins)).sum(dtype=np.float32))
        vdiff = np.float32((pa * np.linalg.norm(pV - O[None], axis=-1).astype(np.float32)).sum(dtype=np.float32))
        if kind in ("k", "both") and meta.get("k_sketch") is not None:
            for cg, slot in enumerate(meta["k_slots"]):
                if slot < 0:
                    continue
                qd = np.float32(abs(float((q_sk[cg] * meta["k_sketch"][cg]).sum(dtype=np.float32))))
                sc = {"carekv": mass * qd * bnd * vdiff * sens, "magnitude_only": qd, "attention_only": mass,
                      "oracle_proxy": qd * mass}[baseline]
                k_c.append((float(np.float32(sc)), pid, cg, slot))
        if kind not in ("v", "both"):
            off += n
            continue
        vtb = rc.v_token_block
        for vb, slot in enumerate(meta["v_slots"]):
            if slot < 0:
                continue
            t0, t1 = vb * vtb, min(vb * vtb + vtb, n)
            if t1 <= t0:
                continue
            bm = np.float32(pa[t0:t1].sum(dtype=np.float32))
            err = np.float32(meta["v_err"][vb])
            sc = {"carekv": bm * err * sens, "magnitude_only": err, "attention_only": bm,
                  "oracle_proxy": bm * err}[baseline]
            v_c.append((float(np.float32(sc)), pid, vb, slot))
        off += n
    tk, tv = len(k_c), len(v_c)
    if tk + tv == 0:
        return [], [], (0, 0)
    rk = rc.__class__(**{**rc.__dict__, "kind": kind})
    bk, bv = resolve_read_budgets(rk, tk, tv)
    if bk == 0 and bv == 0:
        return [], [], (bk, bv)

    def norm(c):
        if not c:
            return c
        m = sum(abs(x[0]) for x in c) / len(c)
        m = m if m > EPS else EPS
        return [(x[0] / m, *x[1:]) for x in c]
    if score_normalize and kind == "both":
        kr, vr = norm(k_c), norm(v_c)
    else:
        kr, vr = k_c, v_c
    pol = rc.route_policy
    if pol == "joint":
        mb = bk + bv if (bk > 0 and bv > 0) else max(bk, bv)
        allc = [("K", *c) for c in kr] + [("V", *c) for c in vr]
        sel = sorted(allc, key=lambda x: x[1], reverse=True)[:mb]
    elif pol == "k_first":
        kp = _stable_desc(kr)[:bk]
        rem = max(0, bk + bv - len(kp))
        vs = _stable_desc(vr)
        if vs and rem > 0:
            vmean = sum(c[0] for c in vs) / len(vs)
            vp = [c for c in vs if c[0] >= vmean][:rem]
        else:
            vp = []
        sel = [("K", *c) for c in kp] + [("V", *c) for c in vp]
    elif pol == "adaptive":
        tot = bk + bv
        if tot <= 0:
            sel = []
        else:
            ac = np.maximum(a.astype(np.float32), np.float32(EPS))
            ent = float(-(ac * np.log(ac)).sum(dtype=np.float32))
            max_ent = math.log(max(a.size, 2))
            vf = max(0.0, min(1.0, ent / max_ent))
            va = max(0, int(round(tot * vf)))
            ka = max(0, tot - va)
            sel = [("K", *c) for c in _stable_desc(kr)[:ka]] + [("V", *c) for c in _stable_desc(vr)[:va]]
    else:
        sel = [("K", *c) for c in _stable_desc(kr)[:bk]] + [("V", *c) for c in _stable_desc(vr)[:bv]]
    if rc.read_budget_mode == "adaptive_score":
        def filt(lst):
            if not lst:
                return lst
            top = abs(lst[0][1])
            kept = [c for c in lst if (rel_thr <= 0 or abs(c[1]) >= rel_thr * top) and
                    (abs_thr <= 0 or abs(c[1]) >= abs_thr)]
            if min_keep > 0 and len(kept) < min_keep:
                kept = lst[:min(min_keep, len(lst))]
            return kept
        sk_ = sorted([c for c in sel if c[0] == "K"], key=lambda c: c[1], reverse=True)
        sv_ = sorted([c for c in sel if c[0] == "V"], key=lambda c: c[1], reverse=True)
        sel = filt(sk_) + filt(sv_)
    ks = [(c[2], c[3], c[4]) for c in sel if c[0] == "K"]
    vs_ = [(c[2], c[3], c[4]) for c in sel if c[0] == "V"]
    legacy_route.last_scores = dict(K={(c[1], c[2]): c[0] for c in kr}, V={(c[1], c[2]): c[0] for c in vr})
    return ks, vs_, (bk, bv)


def legacy_correction(cache, l, h, q, s, a, O, V, rc, sketch_P, kind="both", score_normalize=False,
                      k_corr_scale=1.0, exact=True, **route_kw):
    """apply_slot_corrections for one query: dO (D,) and the selection."""
    ks, vs_, budgets = legacy_route(cache, l, h, q, s, a, O, V, rc, sketch_P, kind, score_normalize, **route_kw)
    D = rc.head_dim
    N = a.shape[0]
    offs = {}
    cur = 0
    for pid in cache.page_ids(l, h):
        n = int(cache.valid[l, h, pid])
        if n > 0:
            offs[pid] = (cur, cur + n)
        cur += n
    dV = np.zeros(D, np.float32)
    dK = np.zeros(D, np.float32)
    ds = np.zeros(N, np.float32)
    RV = np.zeros((N, D), np.float32)
    selv = np.zeros(N, bool)
    vtb = rc.v_token_block
    for pid, vb, slot in vs_:
        if pid not in offs:
            continue
        p0, p1 = offs[pid]
        t0, t1 = vb * vtb, min(vb * vtb + vtb, p1 - p0)
        if t1 <= t0:
            continue
        packed, sc = cache.read_v_slot(slot)
        R = unpack_4bit(packed, sc, vtb * D).reshape(vtb, D)[:t1 - t0]
        dV += (a[p0 + t0:p0 + t1, None] * R).sum(0, dtype=np.float32)
        RV[p0 + t0:p0 + t1] = R
        selv[p0 + t0:p0 + t1] = True
    nk = 0
    kcg = rc.k_channel_group
    for pid, cg, slot in ks:
        if pid not in offs:
            continue
        p0, p1 = offs[pid]
        packed, sc = cache.read_k_slot(slot)
        R = unpack_4bit(packed, sc, rc.page_size * kcg).reshape(rc.page_size, kcg)[:p1 - p0]
        qd = (R * q[None, cg * kcg:(cg + 1) * kcg]).sum(-1, dtype=np.float32)
        dK += ((a[p0:p1] * qd)[:, None] * (V[p0:p1] - O[None])).sum(0, dtype=np.float32)
        ds[p0:p1] += qd
        nk += 1
    if exact and nk > 0:
        d = exact_softmax_correction(a[None], ds[None] / np.float32(math.sqrt(D)), V, O[None], RV, selv[None])[0]
    else:
        d = dV + np.float32(k_corr_scale) * dK
    return d.astype(np.float32), dict(k_sel=ks, v_sel=vs_, budgets=budgets)
