"""CAREKVLayer: the reference's drop-in attention layer over the B200 cache path.

Mirrors ``CAREKVLayer`` (layer.py:147-1163): the constructor takes the Q/K/V/O
projection weights, ``prefill`` writes a prompt into the cache and returns
the attention output, ``decode_step`` appends one token and attends over the
cache with the residual correction.  Projections, RoPE and the output
projection are PyTorch; the cache write (quantize, pack, residual store,
slot enumeration) and decode attention with the correction run in the CUDA
library through ``DecodeEngine``.

One arena holds every sequence of a batch: ``seq`` picks the sequence of a
single-sequence call (the reference keeps one cache per sequence), and the
``*_batch`` methods run all sequences of the arena with one launch per
kernel.

Prefill attention follows ``CAREKV_PREFILL_MODE`` (layer.py:129-141, default
``fp``): ``fp`` attends over the full-precision post-RoPE K / V, ``base_quant``
over their per-group quantize-dequantize (scales in the activation dtype),
and ``carekv_stored`` adds the stored-slot correction
(_apply_sparse_prefill_correction_stored, layer.py:458-637, with the
vectorized router) to that base attention: the attention weights, logits and
base output come from PyTorch, the routing and correction of every prefill
position run in the CUDA route kernel over the slots the prefill just
stored.  ``carekv_eval`` (the in-memory residual upper bound,
layer.py:363-453) is not built and raises NotImplementedError.
"""

from __future__ import annotations

import math
import os
from typing import Any, Dict, Optional, Tuple

import torch
from torch import Tensor, nn

from .cache import CAREKVCache
from .config import CacheConfig, any_read_budget
from .engine import DecodeEngine
from .quantizer import QuantConfig, dequantize, quantize

try:  # RoPE as the reference applies it (layer.py:66)
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
except Exception:  # pragma: no cover - transformers is optional
    apply_rotary_pos_emb = None


def resolve_prefill_mode() -> str:
    """CAREKV_PREFILL_MODE as the reference resolves it (layer.py:129-141)."""
    raw = os.environ.get("CAREKV_PREFILL_MODE", "fp").lower()
    if raw == "carekv":
        return "carekv_eval"
    if raw in {"quant", "int"}:
        return "base_quant"
    return raw


def engine_for(cache: CAREKVCache) -> DecodeEngine:
    """The DecodeEngine bound to a cache arena (created on first use)."""
    eng = getattr(cache, "_engine", None)
    if eng is None:
        eng = DecodeEngine(cache)
        cache._engine = eng
    return eng


def _rope(q: Tensor, k: Tensor, position_embeddings) -> Tuple[Tensor, Tensor]:
    """q [B, Hq, T, D], k [B, Hkv, T, D] -> post-RoPE (HF apply_rotary_pos_emb)."""
    if position_embeddings is None or apply_rotary_pos_emb is None:
        return q, k
    cos, sin = position_embeddings
    cos = cos.to(device=q.device, dtype=q.dtype)
    sin = sin.to(device=q.device, dtype=q.dtype)
    if cos.dim() == 2:          # [T, D] -> [1, T, D]
        cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
    return apply_rotary_pos_emb(q, k, cos, sin)


def causal_attention(Q: Tensor, K: Tensor, V: Tensor, attention_mask: Optional[Tensor]) -> Tensor:
    """O = softmax(Q K^T / sqrt(D) + mask) V with scores and softmax in fp32
    (layer.py:936-973).  Q [B, Hq, T, D], K / V [B, Hq, T, D]; the additive
    mask is [T, T] or broadcastable to [B, 1, T, T]; None -> causal."""
    D = Q.shape[-1]
    T = Q.shape[-2]
    scores = torch.matmul(Q.float(), K.float().transpose(-1, -2)) / math.sqrt(D)
    if attention_mask is not None:
        am = attention_mask.to(device=scores.device, dtype=scores.dtype)
        if am.dim() == 2:
            am = am.unsqueeze(0).unsqueeze(0)
        elif am.dim() == 3:
            am = am.unsqueeze(1)
        scores = scores + am[..., :T, :T]
    else:
        causal = torch.full((T, T), torch.finfo(scores.dtype).min, device=scores.device, dtype=scores.dtype)
        scores = scores + torch.triu(causal, diagonal=1)
    w = torch.softmax(scores, dim=-1, dtype=torch.float32).to(Q.dtype)
    return torch.matmul(w, V)


class CAREKVLayer(nn.Module):
    """Drop-in attention layer (layer.py:147-179): projections + CARE-KV cache."""

    def __init__(self, cfg: CacheConfig, layer_id: int, W_Q: Tensor, W_K: Tensor, W_V: Tensor, W_O: Tensor,
                 device: torch.device = torch.device("cpu")):
        super().__init__()
        self.cfg = cfg
        self.layer_id = layer_id
        self.device = torch.device(device)
        self.W_Q = nn.Parameter(W_Q, requires_grad=False)
        self.W_K = nn.Parameter(W_K, requires_grad=False)
        self.W_V = nn.Parameter(W_V, requires_grad=False)
        self.W_O = nn.Parameter(W_O, requires_grad=False)
        self.base_qcfg = QuantConfig(bits=cfg.base_bits, group_size=cfg.group_size)

    # ── projections ──────────────────────────────────────────────────
    def _project(self, hidden: Tensor):
        """hidden [B, T, dm] -> q [B, Hq, T, D], k / v [B, Hkv, T, D]."""
        cfg = self.cfg
        B, T, _ = hidden.shape
        Hq, Hkv, D = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        q = (hidden @ self.W_Q.T).reshape(B, T, Hq, D).transpose(1, 2)
        k = (hidden @ self.W_K.T).reshape(B, T, Hkv, D).transpose(1, 2)
        v = (hidden @ self.W_V.T).reshape(B, T, Hkv, D).transpose(1, 2)
        return q, k, v

    def _out(self, O: Tensor) -> Tensor:
        """O [B, Hq, T, D] -> [B, T, dm]."""
        B, Hq, T, D = O.shape
        return O.transpose(1, 2).reshape(B, T, Hq * D) @ self.W_O.T

    # ── prefill ──────────────────────────────────────────────────────
    def prefill(self, cache: CAREKVCache, hidden: Tensor, sink_tokens: int = 4,
                attention_mask: Optional[Tensor] = None,
                position_embeddings: Optional[Tuple[Tensor, Tensor]] = None,
                token_start_abs: int = 0, debug_stats: Optional[Dict[str, Any]] = None, seq: int = 0) -> Tensor:
        """hidden [T, dm] of sequence `seq` -> attention output [T, dm] (layer.py:643-845)."""
        pe = None
        if position_embeddings is not None:
            cos, sin = position_embeddings
            pe = (cos if cos.dim() == 3 else cos.unsqueeze(0), sin if sin.dim() == 3 else sin.unsqueeze(0))
        return self.prefill_batch(cache, hidden.unsqueeze(0), sink_tokens, attention_mask, pe,
                                  token_start_abs, seq_begin=seq)[0]

    def prefill_batch(self, cache: CAREKVCache, hidden: Tensor, sink_tokens: int = 4,
                      attention_mask: Optional[Tensor] = None,
                      position_embeddings: Optional[Tuple[Tensor, Tensor]] = None,
                      token_start_abs: int = 0, seq_begin: int = 0) -> Tensor:
        """hidden [B, T, dm] of sequences seq_begin .. seq_begin+B -> [B, T, dm]."""
        mode = resolve_prefill_mode()
        if mode == "carekv_eval":
            raise NotImplementedError(
                "CAREKV_PREFILL_MODE=carekv_eval: the in-memory residual upper bound (layer.py:363-453) is not "
                "built in this library; use fp, base_quant or carekv_stored")
        if mode not in ("fp", "base_quant", "carekv_stored"):
            raise ValueError(f"Unknown CAREKV_PREFILL_MODE={mode}")
        cfg = self.cfg
        B, T, _ = hidden.shape
        g = cfg.num_heads // cfg.num_kv_heads
        q, k, v = self._project(hidden)
        q_post, k_post = _rope(q, k, position_embeddings)
        eng = engine_for(cache)
        eng.prefill_store(self.layer_id, k_post.contiguous(), v.contiguous(), seq_begin=seq_begin,
                          token_start=token_start_abs, sink_tokens=sink_tokens)
        if mode == "fp":
            K_att, V_att = k_post, v
        else:
            K_att, V_att = self._quantize_dequantize(k_post, "K"), self._quantize_dequantize(v, "V")
        if mode == "carekv_stored" and any_read_budget(cfg):
            O = self._stored_correction(eng, q_post, K_att, V_att, attention_mask, seq_begin)
            return self._out(O)
        if g > 1:
            K_att = K_att.repeat_interleave(g, dim=1)
            V_att = V_att.repeat_interleave(g, dim=1)
        O = causal_attention(q_post, K_att, V_att, attention_mask)
        return self._out(O)

    def _stored_correction(self, eng: DecodeEngine, q: Tensor, K_hat: Tensor, V_hat: Tensor,
                           attention_mask: Optional[Tensor], seq_begin: int, chunk: int = 256) -> Tensor:
        """Base attention over K_hat / V_hat plus the stored-slot correction
        (layer.py:458-637): q [B, Hq, T, D]; K_hat, V_hat [B, Hkv, T, D] in the
        activation dtype.  Returns the corrected attention output [B, Hq, T, D].

        Per sequence and chunk of positions the causal attention runs in
        PyTorch as layer.py:936-972 does (fp32 logits and softmax, weights cast
        to the activation dtype, output in the activation dtype); the weights,
        logits, base output and the fp32 attn @ V_hat feed the route kernel,
        which reads V_hat and its page norms instead of the cache's int8-scale
        dequantisation, as the reference passes V_hat_stack."""
        cfg = self.cfg
        B, Hq, T, D = q.shape
        H, QN, PS = cfg.num_kv_heads, Hq // cfg.num_kv_heads, cfg.page_size
        dt = q.dtype
        out = torch.empty_like(q)
        for b in range(B):
            seq = seq_begin + b
            P = eng._pages(seq, self.layer_id)
            if eng.cache.lengths[seq][self.layer_id] != T:
                raise NotImplementedError("carekv_stored prefill correction: the sequence must hold exactly this "
                                          "prefill (a prompt written in one call)")
            N = P * PS
            Kb, Vb = K_hat[b], V_hat[b]                                   # [H, T, D]
            if QN > 1:
                Kq, Vq = Kb.repeat_interleave(QN, dim=0), Vb.repeat_interleave(QN, dim=0)
            else:
                Kq, Vq = Kb, Vb
            v_rows = torch.zeros(H, N, D, dtype=torch.float32, device=q.device)
            v_rows[:, :T] = Vb.float()
            v_pnorm = v_rows.view(H, P, PS * D).norm(dim=-1).contiguous()
            mask_b = None
            if attention_mask is not None:
                am = attention_mask
                if am.dim() == 4:
                    am = am[b if am.shape[0] > 1 else 0, 0]
                elif am.dim() == 3:
                    am = am[b if am.shape[0] > 1 else 0]
                mask_b = am
            for t0 in range(0, T, chunk):
                t1 = min(T, t0 + chunk)
                tc = t1 - t0
                scores = torch.einsum("hid,hjd->hij", q[b, :, t0:t1].float(), Kq.float()) / math.sqrt(D)
                if mask_b is not None:
                    scores = scores + mask_b[t0:t1, :T].to(device=scores.device, dtype=scores.dtype).unsqueeze(0)
                else:
                    rows = torch.arange(t0, t1, device=q.device).unsqueeze(1)
                    cols = torch.arange(T, device=q.device).unsqueeze(0)
                    scores = scores.masked_fill(cols > rows, torch.finfo(torch.float32).min)
                attn_w = torch.softmax(scores, dim=-1, dtype=torch.float32).to(dt)
                o_base = torch.einsum("hij,hjd->hid", attn_w, Vq)             # [Hq, tc, D], activation dtype
                A = attn_w.float()
                o_exact = torch.einsum("hij,hjd->hid", A, Vq.float())

                def rows_of(x, fill):                                       # [Hq, tc, T] -> [tc, H, QN, N]
                    y = torch.full((Hq, tc, N), fill, dtype=torch.float32, device=q.device)
                    y[..., :T] = x
                    return y.view(H, QN, tc, N).permute(2, 0, 1, 3).contiguous()

                def per_row(x):                                             # [Hq, tc, ...] -> [tc, H, QN, ...]
                    return x.reshape(H, QN, tc, *x.shape[2:]).movedim(2, 0).contiguous()
                res = eng.prefill_correct(
                    self.layer_id, seq, q[b, :, t0:t1].transpose(0, 1).contiguous(), attn=rows_of(A, 0.0),
                    o_base=per_row(o_base.float()), o_exact=per_row(o_exact), attn_sum=per_row(A.sum(-1)),
                    logits=rows_of(scores, torch.finfo(torch.float32).min), row_max=per_row(scores.amax(-1)),
                    v_rows=v_rows, v_pnorm=v_pnorm)
                out[b, :, t0:t1] = res.transpose(0, 1)
        return out

    def _quantize_dequantize(self, x: Tensor, kind: str = "V") -> Tensor:
        """x [..., D] -> per-group quantize then dequantize with scales in x's
        dtype (layer.py:185-195): the K_hat / V_hat the reference's prefill
        attends over (layer.py:298-299), before the cache's int8 scale step.
        KIVI-style base: per-channel K over the sequence axis, per-token V
        (layer.py:706-712, kivi_helpers.py:35-59)."""
        if self.cfg.is_kivi:
            from .quantizer import quant_dequant_kivi_k, quant_dequant_kivi_v
            return quant_dequant_kivi_k(x, self.cfg.base_bits) if kind == "K" else \
                quant_dequant_kivi_v(x, self.cfg.base_bits)
        D = x.shape[-1]
        flat = x.reshape(-1, D).contiguous()
        codes, scale = quantize(flat, self.base_qcfg)
        return dequantize(codes, scale, flat.shape, self.base_qcfg).to(x.dtype).reshape(x.shape)

    # ── decode ───────────────────────────────────────────────────────
    def decode_step(self, cache: CAREKVCache, hidden: Tensor,
                    position_embeddings: Optional[Tuple[Tensor, Tensor]] = None,
                    debug_stats: Optional[Dict[str, Any]] = None, seq: int = 0) -> Tensor:
        """hidden [1, dm] of sequence `seq` -> [1, dm] (layer.py:978-1163)."""
        return self.decode_step_batch(cache, hidden.reshape(1, -1), position_embeddings, seq_begin=seq)

    def decode_step_batch(self, cache: CAREKVCache, hidden: Tensor,
                          position_embeddings: Optional[Tuple[Tensor, Tensor]] = None,
                          seq_begin: int = 0) -> Tensor:
        """hidden [B, dm] (one new token per sequence) -> [B, dm].

        Appends the token's K / V (quantize, pack; the page-full residual store
        when a page completes) and runs decode attention with the residual
        correction over every sequence in one launch per kernel.  The route
        kind, k correction scale and score normalisation come from the
        CAREKV_* environment knobs as in layer.py:1148-1150.
        """
        cfg = self.cfg
        B = hidden.shape[0]
        q, k, v = self._project(hidden.reshape(B, 1, -1))
        pe = None
        if position_embeddings is not None:
            cos, sin = position_embeddings
            cos = cos.reshape(-1, 1, cos.shape[-1])
            sin = sin.reshape(-1, 1, sin.shape[-1])
            if cos.shape[0] == 1 and B > 1:
                cos, sin = cos.expand(B, 1, -1), sin.expand(B, 1, -1)
            pe = (cos, sin)
        q_post, k_post = _rope(q, k, pe)
        eng = engine_for(cache)
        eng.append(self.layer_id, k_post[:, :, 0].contiguous(), v[:, :, 0].contiguous(), seq_begin=seq_begin)
        O = eng.attend(self.layer_id, q_post[:, :, 0].contiguous(), seq_begin=seq_begin)   # [B, Hq, D]
        return O.reshape(B, cfg.num_heads * cfg.head_dim) @ self.W_O.T
