"""Decode attention over the packed cache plus the CARE-KV correction.

Restates, for one (layer, kv_head) and the Qn query heads that share it:
  * base attention (attention.py:1009-1022): s = K_hat q * fp32(1/sqrt(D)),
    a = softmax(s), O = a V_hat, all fp32 over fp16-exact K_hat / V_hat;
  * vectorized_joint_correction (attention.py:540-957) with the slot index
    builders, read-budget resolution (residual_router.py:37-76), the
    combined_kvscore K score (attention.py:167-184) or the sketch proxy
    (attention.py:718-725), per-query normalisation, joint / separate top-k
    and the exact softmax correction (attention.py:96-118) or the linear
    Jacobian form.
Top-k ties are broken by larger score, then lower candidate index.
"""

import math
from dataclasses import dataclass
from typing import Optional

import numpy as np

from .quant import unpack_4bit

EPS = 1e-6


@dataclass
class RouteConfig:
    head_dim: int = 64
    page_size: int = 16
    k_channel_group: int = 32
    v_token_block: int = 4
    sketch_dim: int = 32
    kind: str = "both"                 # v | k | both
    route_policy: str = "joint"        # joint | separate | k_first | adaptive (non-joint = separate)
    score_normalize: bool = True
    kscore_live: bool = True
    k_correction_mode: str = "exact"   # exact | linear
    k_corr_scale: float = 0.1
    read_budget_mode: str = "ratio"    # ratio | absolute | adaptive_score
    read_abs_k: int = 0
    read_abs_v: int = 0
    read_budget_ratio: float = 0.03
    read_budget_ratio_k: Optional[float] = None
    read_budget_ratio_v: Optional[float] = None
    layer_multiplier: float = 1.0
    sensitivity: float = 1.0
    lambda_k: float = 1.0
    lambda_v: float = 1.0


def resolve_read_budgets(rc: RouteConfig, total_k, total_v):
    """_resolve_read_budgets (residual_router.py:37-76)."""
    lm = rc.layer_multiplier
    if rc.read_budget_mode in ("absolute", "adaptive_score"):
        bk = int(round(max(0, int(rc.read_abs_k)) * lm))
        bv = int(round(max(0, int(rc.read_abs_v)) * lm))
    else:
        def _r(o, fb):
            return fb if (o is None or o < 0) else o
        rk = _r(rc.read_budget_ratio_k, rc.read_budget_ratio) * lm
        rv = _r(rc.read_budget_ratio_v, rc.read_budget_ratio) * lm
        bk = max(1, int(total_k * rk)) if rk > 0 and total_k > 0 else 0
        bv = max(1, int(total_v * rv)) if rv > 0 and total_v > 0 else 0
    if rc.kind == "v":
        bk = 0
    elif rc.kind == "k":
        bv = 0
    return min(bk, total_k), min(bv, total_v)


def topk_indices(scores, k):
    """Per row, the k largest entries; ties -> lower index first."""
    Qn, n = scores.shape
    out = np.zeros((Qn, k), np.int64)
    idx = np.arange(n)
    for q in range(Qn):
        order = np.lexsort((idx, -scores[q].astype(np.float64)))
        out[q] = order[:k]
    return out


def base_attention(K_hat, V_hat, Q, head_dim):
    """CAREKVAttention base math per query head (attention.py:1015-1022)."""
    sf = np.float32(1.0 / math.sqrt(head_dim))
    S = (Q.astype(np.float32) @ K_hat.T.astype(np.float32)) * sf
    m = S.max(axis=1, keepdims=True)
    e = np.exp(S - m)
    A = e / e.sum(axis=1, keepdims=True)
    O = A @ V_hat.astype(np.float32)
    return S.astype(np.float32), A.astype(np.float32), O.astype(np.float32)


def exact_softmax_correction(A, ds, V_base, O_base, RV_full=None, sel_tok=None):
    """attention.py:96-118 in fp32."""
    w = np.exp(ds - ds.max(axis=1, keepdims=True))
    a_new = A * w
    a_new = a_new / np.maximum(a_new.sum(axis=1, keepdims=True), np.float32(1e-30))
    O_new = a_new @ V_base
    if RV_full is not None and sel_tok is not None:
        O_new = O_new + (a_new * sel_tok.astype(np.float32)) @ RV_full
    return (O_new - O_base).astype(np.float32)


def _k_slot_index(cache, l, h, rc):
    """_build_k_slot_index (attention.py:540-573)."""
    ps = rc.page_size
    kcg = rc.k_channel_group
    out = []
    cursor = 0
    for pid in cache.page_ids(l, h):
        meta = cache.meta[l][h][pid]
        n_valid = int(cache.valid[l, h, pid])
        if n_valid == 0 or meta is None:
            cursor += n_valid
            continue
        for cg, slot in enumerate(meta["k_slots"]):
            if slot < 0:
                continue
            packed, scale = cache.read_k_slot(slot)
            r = unpack_4bit(packed, scale, ps * kcg).reshape(ps, kcg)
            out.append(dict(R=r[:n_valid], cg=cg, pstart=cursor, nvalid=n_valid,
                            sketch=meta["k_sketch"][cg], page=pid, slot=slot))
        cursor += n_valid
    return out


def _v_slot_index(cache, l, h, rc):
    """_build_v_slot_index (attention.py:386-441), including its cursor rule
    (a page with no metadata does not advance the token cursor)."""
    vtb = rc.v_token_block
    D = rc.head_dim
    out = []
    cursor = 0
    for pid in cache.page_ids(l, h):
        meta = cache.meta[l][h][pid]
        n_valid = int(cache.valid[l, h, pid])
        if n_valid == 0 or meta is None:
            continue
        for vb, slot in enumerate(meta["v_slots"]):
            if slot < 0:
                continue
            t0 = vb * vtb
            t1 = min(t0 + vtb, n_valid)
            if t1 <= t0:
                continue
            packed, scale = cache.read_v_slot(slot)
            r = unpack_4bit(packed, scale, vtb * D).reshape(vtb, D)
            out.append(dict(R=r, start=cursor + t0, len=t1 - t0,
                            err=float(meta["v_err"][vb]) * rc.sensitivity,
                            page=pid, vb=vb, slot=slot))
        cursor += n_valid
    return out


def vectorized_joint_correction(cache, l, h, Q, S, A, V_base, O_base, rc: RouteConfig,
                                sketch_P=None):
    """Batched ΔO (Qn, D) for the queries of one kv head (attention.py:576-957).

    Returns (delta, info) where info holds scores, selections, budgets and
    read counts for parity checks.
    """
    Qn, D = Q.shape
    N = A.shape[1]
    A = A.astype(np.float32)
    S = S.astype(np.float32)
    V_base = V_base.astype(np.float32)
    O_base = O_base.astype(np.float32)
    Q = Q.astype(np.float32)
    delta = np.zeros((Qn, D), np.float32)
    info = dict(n_k=0, n_v=0, budget_k=0, budget_v=0, score_K=None, score_V=None,
                sel_k=None, sel_v=None, k_reads=0, v_reads=0, k_index=[], v_index=[])
    if N == 0:
        return delta, info
    kidx = _k_slot_index(cache, l, h, rc)
    vidx = _v_slot_index(cache, l, h, rc)
    n_k, n_v = len(kidx), len(vidx)
    info.update(n_k=n_k, n_v=n_v, k_index=kidx, v_index=vidx, A=A)
    want_k = rc.kind in ("k", "both") and n_k > 0
    want_v = rc.kind in ("v", "both") and n_v > 0
    if not want_k and not want_v:
        return delta, info
    bk, bv = resolve_read_budgets(rc, n_k if want_k else 0, n_v if want_v else 0)
    info.update(budget_k=bk, budget_v=bv)
    if bk == 0 and bv == 0:
        return delta, info
    sens = np.float32(rc.sensitivity)
    kcg = rc.k_channel_group
    sqrtD = np.float32(math.sqrt(max(D, 1)))

    score_K = None
    if want_k and bk > 0:
        score_K = np.zeros((Qn, n_k), np.float32)
        if not rc.kscore_live:
            s_top = S.max(axis=1, keepdims=True)
            inv_margin = np.float32(1.0) / np.maximum(s_top - S, np.float32(EPS))
            vdiff = np.sqrt(((V_base[None, :, :] - O_base[:, None, :]) ** 2).sum(-1, dtype=np.float32))
            if sketch_P is None:
                from .store import sketch_projection
                sketch_P = sketch_projection(D, kcg, rc.sketch_dim)
        for si, e in enumerate(kidx):
            c0, c1 = e["cg"] * kcg, (e["cg"] + 1) * kcg
            ps, nv = e["pstart"], e["nvalid"]
            if rc.kscore_live:
                dS = (Q[:, c0:c1] @ e["R"].T) / sqrtD
                Aw = A[:, ps:ps + nv]
                sn = Aw * (np.float32(1.0) - Aw)
                kp = np.sqrt(((dS * sn) ** 2).sum(axis=1, dtype=np.float32))
                vc = np.sqrt((V_base[ps:ps + nv] ** 2).sum(dtype=np.float32))
                ks = np.nan_to_num(kp * vc, nan=0.0, posinf=0.0, neginf=0.0)
                score_K[:, si] = np.maximum(ks, 0) * sens
            else:
                pa = A[:, ps:ps + nv]
                mass = pa.sum(axis=1)
                boundary = (pa * inv_margin[:, ps:ps + nv]).sum(axis=1)
                pvd = (pa * vdiff[:, ps:ps + nv]).sum(axis=1)
                qs = Q[:, c0:c1] @ sketch_P
                qdotr = np.abs((qs * e["sketch"][None, :]).sum(axis=1))
                score_K[:, si] = mass * qdotr * boundary * pvd * sens

    score_V = None
    if want_v and bv > 0:
        mask = np.zeros((n_v, N), np.float32)
        for j, e in enumerate(vidx):
            mask[j, e["start"]:e["start"] + e["len"]] = 1.0
        err = np.array([e["err"] for e in vidx], np.float32)
        score_V = ((A @ mask.T) * err[None, :]) * sens

    if rc.score_normalize and rc.kind == "both" and score_K is not None and score_V is not None:
        nk = np.maximum(np.abs(score_K).mean(axis=1, keepdims=True), np.float32(EPS))
        nvv = np.maximum(np.abs(score_V).mean(axis=1, keepdims=True), np.float32(EPS))
        sK = score_K / nk
        sV = score_V / nvv
        if rc.kscore_live:
            sK = sK * np.float32(rc.lambda_k)
            sV = sV * np.float32(rc.lambda_v)
    else:
        sK, sV = score_K, score_V
    info.update(score_K=score_K, score_V=score_V, score_K_r=sK, score_V_r=sV)

    sel_k = np.zeros((Qn, n_k), bool) if score_K is not None else None
    sel_v = np.zeros((Qn, n_v), bool) if score_V is not None else None
    if rc.route_policy == "joint" and rc.kind == "both" and sK is not None and sV is not None:
        mb = (bk + bv) if (bk > 0 and bv > 0) else max(bk, bv)
        merged = np.concatenate([sK, sV], axis=1)
        mb = min(mb, merged.shape[1])
        top = topk_indices(merged, mb)
        selm = np.zeros((Qn, n_k + n_v), bool)
        np.put_along_axis(selm, top, True, axis=1)
        sel_k, sel_v = selm[:, :n_k], selm[:, n_k:]
    else:
        if sK is not None and bk > 0:
            np.put_along_axis(sel_k, topk_indices(sK, min(bk, n_k)), True, axis=1)
        if sV is not None and bv > 0:
            np.put_along_axis(sel_v, topk_indices(sV, min(bv, n_v)), True, axis=1)
    info.update(sel_k=sel_k, sel_v=sel_v)

    wK = None
    if sel_k is not None and sel_k.any():
        wK = np.zeros((Qn, N), np.float32)
        for si, e in enumerate(kidx):
            c0, c1 = e["cg"] * kcg, (e["cg"] + 1) * kcg
            ps, nv = e["pstart"], e["nvalid"]
            qd = Q[:, c0:c1] @ e["R"].T
            wK[:, ps:ps + nv] += sel_k[:, si].astype(np.float32)[:, None] * qd
        info["k_reads"] = int(sel_k.sum())

    RV_full = None
    sel_tok = None
    if sel_v is not None and sel_v.any():
        RV_full = np.zeros((N, D), np.float32)
        sel_tok = np.zeros((Qn, N), bool)
        for j, e in enumerate(vidx):
            s0, ln = e["start"], e["len"]
            RV_full[s0:s0 + ln] = e["R"][:ln]
            sel_tok[:, s0:s0 + ln] |= sel_v[:, j][:, None]
        info["v_reads"] = int(sel_v.sum())

    if rc.k_correction_mode == "exact" and wK is not None:
        delta = exact_softmax_correction(A, wK / sqrtD, V_base, O_base, RV_full, sel_tok)
    else:
        if wK is not None:
            AwK = A * wK
            dK = AwK @ V_base - AwK.sum(axis=1, keepdims=True) * O_base
            delta = delta + np.float32(rc.k_corr_scale) * dK
        if sel_tok is not None:
            delta = delta + (A * sel_tok.astype(np.float32)) @ RV_full
    return delta.astype(np.float32), info


def decode_attention_kvh(cache, l, h, Q, rc: RouteConfig, correction=True, sketch_P=None):
    """O (Qn, D) for the query heads of kv head h: base attention + ΔO."""
    K_hat, V_hat, _ = cache.read_base_concat(l, h)
    Qn, D = Q.shape
    if K_hat.shape[0] == 0:
        return np.zeros((Qn, D), np.float32), None
    S, A, O = base_attention(K_hat, V_hat, Q, D)
    if not correction:
        return O, dict(S=S, A=A, O_base=O)
    delta, info = vectorized_joint_correction(cache, l, h, Q, S, A, V_hat, O, rc, sketch_P=sketch_P)
    info.update(S=S, A=A, O_base=O, delta=delta)
    return (O + delta).astype(np.float32), info
