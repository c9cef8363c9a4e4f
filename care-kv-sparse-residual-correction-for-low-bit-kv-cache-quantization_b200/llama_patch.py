"""HuggingFace Llama patch: every attention module runs through CARE-KV.

Mirrors ``patch_llama_model`` / ``CAREKVLlamaAttention`` (llama_patch.py:35-352)
for the installed transformers (5.x attention contract: keyword
``past_key_values`` / ``position_embeddings``, returns ``(attn_output,
attn_weights)``).

* All layers share one CAREKVCache arena sized for the batch of the first
  prefill; a new prefill (T > 1, or the first call) at layer 0 resets it.
* A batch runs as one call per layer (one arena, one kernel launch per
  kernel), not a loop over sequences.
* HF's own cache only has to report the sequence length (generate derives
  positions and masks from it).  The reference updates it with full-size
  fp16 zero tensors (llama_patch.py:270-285), doubling peak memory; here the
  update carries (B, 1, T, 1) zeros, so the HF cache costs B*T elements per
  layer.
* Without ``position_embeddings`` the original HF attention runs, as in the
  reference (llama_patch.py:158-163); ``CAREKV_RETURN=original`` forces it.
"""

from __future__ import annotations

import os
from typing import Dict, Optional

import torch
from torch import nn

from .cache import CAREKVCache
from .config import CacheConfig
from .layer import CAREKVLayer


class _Shared:
    """State shared by the patched layers of one model."""

    def __init__(self, cfg: CacheConfig, device):
        self.cfg = cfg
        self.device = device
        self.cache: Optional[CAREKVCache] = None
        self.epoch = 0      # bumped by every reset; a layer has prefilled when its epoch matches

    def cache_for(self, batch: int, device) -> CAREKVCache:
        if self.cache is None or self.cache.batch != batch:
            self.cache = CAREKVCache(self.cfg, device, batch=batch)
        return self.cache

    def reset(self):
        if self.cache is not None:
            self.cache.reset()
        self.epoch += 1


class CAREKVLlamaAttention(nn.Module):
    """Wraps an HF attention module; forward runs CAREKVLayer prefill / decode."""

    def __init__(self, original_attn: nn.Module, cfg: CacheConfig, layer_id: int, device: torch.device,
                 shared: Optional[_Shared] = None):
        super().__init__()
        self.cfg = cfg
        self.layer_id = layer_id
        self.device = device
        self.original_attn = original_attn
        for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
            if getattr(getattr(original_attn, name), "bias", None) is not None:
                raise NotImplementedError(f"{name} has a bias; CAREKVLayer takes weight matrices only")
        self.care_layer = CAREKVLayer(cfg, layer_id, original_attn.q_proj.weight.data,
                                      original_attn.k_proj.weight.data, original_attn.v_proj.weight.data,
                                      original_attn.o_proj.weight.data, device)
        self.shared = shared if shared is not None else _Shared(cfg, device)
        self._epoch = -1    # shared epoch of this layer's last prefill

    def reset_cache(self):
        self.shared.reset()

    def _original(self, hidden_states, **kwargs):
        return self.original_attn(hidden_states, **kwargs)

    def forward(self, hidden_states, position_embeddings=None, attention_mask=None, past_key_values=None,
                cache_position=None, **kwargs):
        call = dict(position_embeddings=position_embeddings, attention_mask=attention_mask,
                    past_key_values=past_key_values, cache_position=cache_position, **kwargs)
        if os.environ.get("CAREKV_RETURN", "care").lower() in {"original", "passthrough", "hf"}:
            return self._original(hidden_states, **call)
        if position_embeddings is None:
            return self._original(hidden_states, **call)
        B, T, _ = hidden_states.shape
        sh = self.shared
        use_cache = kwargs.get("use_cache", past_key_values is not None)
        hf_len = 0
        if past_key_values is not None:
            try:
                hf_len = past_key_values.get_seq_length(self.layer_id)
            except Exception:
                hf_len = 0
        new_prompt = (T > 1 or self._epoch != sh.epoch
                      or (use_cache and past_key_values is not None and hf_len == 0))
        if new_prompt and self.layer_id == 0:
            sh.reset()
        cache = sh.cache_for(B, hidden_states.device)
        if new_prompt:
            out = self.care_layer.prefill_batch(cache, hidden_states, attention_mask=_square_mask(attention_mask, T),
                                                position_embeddings=position_embeddings, token_start_abs=0)
            self._epoch = sh.epoch
        else:
            out = self.care_layer.decode_step_batch(cache, hidden_states[:, 0], position_embeddings).unsqueeze(1)
        if use_cache and past_key_values is not None and hasattr(past_key_values, "update"):
            z = hidden_states.new_zeros((B, 1, T, 1))
            try:
                past_key_values.update(z, z, self.layer_id)
            except Exception:
                pass
        return out.to(hidden_states.dtype), None


def _square_mask(mask, T):
    """The additive [.., T, T] part of an HF 4D mask, or None (causal)."""
    if mask is None or not torch.is_tensor(mask) or mask.dtype == torch.bool:
        return None
    return mask[..., -T:, -T:]


def patch_llama_model(model: nn.Module, care_cfg: CacheConfig, device: Optional[torch.device] = None) -> nn.Module:
    """Replace every attention module with CAREKVLlamaAttention, in place
    (llama_patch.py:292-352): modules whose class name contains "Attention"
    and that have q_proj; the layer id is the first integer of the module
    path; all layers share one cache arena."""
    if device is None:
        try:
            device = next(model.parameters()).device
        except StopIteration:
            device = torch.device("cpu")
    shared = _Shared(care_cfg, device)
    targets = []
    for name, module in model.named_modules():
        if "Attention" in type(module).__name__ and hasattr(module, "q_proj"):
            targets.append((name, module))
    for name, module in targets:
        parts = name.split(".")
        parent = model
        for part in parts[:-1]:
            parent = getattr(parent, part)
        layer_id = next((int(p) for p in parts if p.isdigit()), 0)
        setattr(parent, parts[-1], CAREKVLlamaAttention(module, care_cfg, layer_id, device, shared))
    model._carekv_shared = shared
    return model


def reset_all_caches(model: nn.Module) -> None:
    """Forget every sequence of a patched model (the next call is a prefill)."""
    sh = getattr(model, "_carekv_shared", None)
    if sh is not None:
        sh.reset()
