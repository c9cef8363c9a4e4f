"""Per-page residual enumeration and slot selection (residual_store.py:239-464).

For one page of ``page_size`` rows (``num_valid`` real tokens, the rest zero
padding) this computes R = X - X_hat, one K candidate per k_channel_group
block and one V candidate per v_token_block block, scores them, keeps the
per-kind budget, packs every kept candidate into a 4-bit slot and records
error norms and sketches.
"""

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from .numerics import round_to
from .quant import dequantize, pack_4bit


@dataclass
class StoreConfig:
    head_dim: int = 64
    page_size: int = 16
    base_bits: int = 3
    group_size: int = 32
    k_channel_group: int = 32
    v_token_block: int = 4
    sketch_dim: int = 32
    residual_bits: int = 4
    store_budget_mode: str = "absolute"      # "absolute" | "ratio"
    store_abs_k: int = 1
    store_abs_v: int = 1
    store_budget_ratio: float = 0.0
    store_budget_ratio_k: Optional[float] = None
    store_budget_ratio_v: Optional[float] = None
    store_policy: str = "residual_kind_aware"  # joint | per_kind | residual_kind_aware
    residual_kind: str = "both"                # v | k | both
    min_per_kind: int = 1
    k_fraction: float = 1.0
    v_fraction: float = 1.0
    layer_multiplier: float = 1.0
    sensitivity: float = 1.0


def sketch_projection(head_dim, k_channel_group, sketch_dim):
    """get_sketch_proj (residual_store.py:206-214): randn(seed 42)/sqrt(sd).

    The matrix is defined by torch's CPU normal generator, so it is drawn
    with torch here too (a constant table, not arithmetic under test).
    """
    import torch
    gen = torch.Generator(device="cpu").manual_seed(42)
    P = torch.randn(k_channel_group, sketch_dim, generator=gen) / math.sqrt(sketch_dim)
    return P.numpy().astype(np.float32)


def store_budgets(cfg: StoreConfig, num_k_cand: int, num_v_cand: int):
    """Per-kind store budgets (residual_store.py:383-409)."""
    use_k = not (cfg.store_policy == "residual_kind_aware" and cfg.residual_kind == "v")
    use_v = not (cfg.store_policy == "residual_kind_aware" and cfg.residual_kind == "k")
    lm = cfg.layer_multiplier
    if cfg.store_budget_mode == "absolute":
        base_k = int(round(max(0, int(cfg.store_abs_k)) * lm))
        base_v = int(round(max(0, int(cfg.store_abs_v)) * lm))
        kb = max(0, base_k) if use_k else 0
        vb = max(0, base_v) if use_v else 0
        joint = kb + vb
    else:
        def _res(o, fb):
            return fb if (o is None or o < 0) else o
        rk = _res(cfg.store_budget_ratio_k, cfg.store_budget_ratio) * cfg.k_fraction * lm
        rv = _res(cfg.store_budget_ratio_v, cfg.store_budget_ratio) * cfg.v_fraction * lm
        kt = max(1, num_k_cand)
        vt = max(1, num_v_cand)
        kb = max(cfg.min_per_kind, int(kt * rk)) if (use_k and rk > 0) else 0
        vb = max(cfg.min_per_kind, int(vt * rv)) if (use_v and rv > 0) else 0
        joint = max(1, int((kt + vt) * cfg.store_budget_ratio * lm))
    store_nothing = (cfg.store_budget_ratio <= 0 and cfg.store_budget_mode != "absolute"
                     and (cfg.store_budget_ratio_k or 0) <= 0
                     and (cfg.store_budget_ratio_v or 0) <= 0)
    return kb, vb, joint, store_nothing


def _err_norm(block):
    """mean over rows of the row L2 norm, fp32 (rk.norm(dim=-1).mean())."""
    if block.shape[0] == 0:
        return 0.0
    n = np.sqrt((block.astype(np.float32) ** 2).sum(axis=-1, dtype=np.float32))
    return float(np.float32(n.mean(dtype=np.float32)))


def process_page(cfg: StoreConfig, K_page, V_page, K_codes, K_scale, V_codes, V_scale,
                 num_valid, dt, is_recent=True, is_sink=False,
                 K_hat_override=None, V_hat_override=None, sketch_P=None,
                 hat_dt=None, sub_dt=None):
    """Score, select and pack the residual slots of one page.

    K_page/V_page: (T, D) in ``dt`` (zero rows past num_valid); K/V codes and
    the UNQUANTIZED scales from the base quantizer (the store path uses the
    pre-int8 scales, layer.py:312-329).  Returns a dict with the K / V
    candidates selected in allocation order (score order, K before V) plus
    per-candidate error norms and sketches.

    ``hat_dt`` is the dtype of the scales (so of X_hat) and ``sub_dt`` the
    torch promotion of the page dtype with it; both default to ``dt``.  The
    decode page-full store passes fp16 scales with a model-dtype page
    (layer.py:1134-1146): fp16 and fp32 pages give R = 0 exactly, a bf16 page
    gives R = bf16(x_hat) - x_hat computed in fp32.
    """
    T, D = K_page.shape
    hat_dt = hat_dt or dt
    sub_dt = sub_dt or dt
    if K_hat_override is not None:
        K_hat = round_to(K_hat_override, hat_dt)
        V_hat = round_to(V_hat_override, hat_dt)
    else:
        K_hat = dequantize(K_codes, K_scale, cfg.group_size, hat_dt)
        V_hat = dequantize(V_codes, V_scale, cfg.group_size, hat_dt)
    R_K = round_to(np.asarray(K_page, np.float32) - K_hat, sub_dt).astype(np.float32)
    R_V = round_to(np.asarray(V_page, np.float32) - V_hat, sub_dt).astype(np.float32)
    if num_valid < T:
        R_K[num_valid:] = 0
        R_V[num_valid:] = 0

    struct = 1.0
    if is_recent:
        struct *= 1.5
    if is_sink:
        struct *= 2.0
    sens = cfg.sensitivity
    kcg = cfg.k_channel_group
    num_cg = D // kcg
    if sketch_P is None:
        sketch_P = sketch_projection(D, kcg, cfg.sketch_dim)

    k_cands = []
    k_err = []
    for cg in range(num_cg):
        c0, c1 = cg * kcg, (cg + 1) * kcg
        if num_valid > 0:
            blk = R_K[:num_valid, c0:c1]
            err = _err_norm(blk)
            rk_mean = blk.mean(axis=0, dtype=np.float32)
        else:
            err = 0.0
            rk_mean = np.zeros(kcg, np.float32)
        k_err.append(err)
        sketch = (rk_mean.astype(np.float32) @ sketch_P).astype(np.float32)
        sketch = sketch.astype(np.float16).astype(np.float32)
        prior = err * sens * struct
        packed, scale, _ = pack_4bit(R_K[:, c0:c1])
        k_cands.append(dict(kind="K", idx=cg, prior=prior, packed=packed,
                            scale=scale, sketch=sketch))

    vtb = cfg.v_token_block
    num_vb = math.ceil(cfg.page_size / vtb)
    v_cands = []
    v_err = []
    for vb in range(num_vb):
        t0 = vb * vtb
        t1v = min(t0 + vtb, num_valid)
        err = _err_norm(R_V[t0:t1v]) if t1v > t0 else 0.0
        v_err.append(err)
        prior = err * sens * struct
        blk = R_V[t0:t0 + vtb]
        if blk.shape[0] < vtb:
            blk = np.concatenate([blk, np.zeros((vtb - blk.shape[0], D), np.float32)])
        packed, scale, _ = pack_4bit(blk)
        v_cands.append(dict(kind="V", idx=vb, prior=prior, packed=packed, scale=scale))

    kb, vb_, joint, nothing = store_budgets(cfg, len(k_cands), len(v_cands))
    k_scored = sorted([c for c in k_cands if c["prior"] > 0], key=lambda c: c["prior"], reverse=True)
    v_scored = sorted([c for c in v_cands if c["prior"] > 0], key=lambda c: c["prior"], reverse=True)
    if nothing:
        selected = []
    elif cfg.store_policy == "joint":
        selected = sorted(k_scored + v_scored, key=lambda c: c["prior"], reverse=True)[:joint]
    else:
        selected = k_scored[:kb] + v_scored[:vb_]

    return dict(
        R_K=R_K, R_V=R_V, K_hat=K_hat, V_hat=V_hat,
        selected=selected, k_cands=k_cands, v_cands=v_cands,
        k_err=np.array(k_err, np.float32).astype(np.float16).astype(np.float32),
        v_err=np.array(v_err, np.float32).astype(np.float16).astype(np.float32),
        k_err_f32=np.array(k_err, np.float32), v_err_f32=np.array(v_err, np.float32),
        k_sketch=np.stack([c["sketch"] for c in k_cands]),
    )
