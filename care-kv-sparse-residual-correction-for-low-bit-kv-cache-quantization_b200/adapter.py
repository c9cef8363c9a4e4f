"""CAREKVAdapter: the reference's paper-best setup helper (baselines/carekv_adapter.py:15-172).

Same constructor as the reference (fixed RK/RV budgets or adaptive scores,
store budgets SK/SV, base bits, slot geometry) and the same CAREKV_*
environment it writes before patching a model.  Differences, each forced by
what this library builds:

* ``setup_model`` patches a model object (or loads a local checkpoint
  directory); this build has no model hub access.
* The uniform and KIVI-style (``kivi_style`` / ``kvquant_style``) base
  quantizers are built; the rotation and calibrated bases raise
  NotImplementedError.
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from .config import CacheConfig, apply_carekv_env_overrides
from .llama_patch import patch_llama_model


class CAREKVAdapter:
    family = "care_kv"
    uses_residual = True
    uses_query_aware_routing = True

    def __init__(self, mode: str = "fixed", rel_threshold: float = 0.0, sk: int = 2, sv: int = 4, rk: int = 2,
                 rv: int = 2, max_rk: int = 4, max_rv: int = 4, bits: int = 3, base_quantizer: str = "uniform",
                 bits_k: int = -1, bits_v: int = -1, max_pages: int = 0, k_store_mode: str = "post_rope",
                 correction_impl: str = "cached", k_channel_group: int = 32, v_token_block: int = 4,
                 prefill_mode: str = "carekv_stored"):
        if base_quantizer not in ("uniform", "kivi_style", "kvquant_style"):
            raise NotImplementedError(f"base_quantizer={base_quantizer}: the uniform and KIVI-style bases are built")
        if mode not in ("fixed", "adaptive"):
            raise ValueError(f"mode={mode}")
        self.mode = mode
        self.rel_threshold = rel_threshold
        self.sk, self.sv = sk, sv
        self.rk, self.rv = rk, rv
        self.max_rk, self.max_rv = max_rk, max_rv
        self.bits = bits
        self.base_quantizer = base_quantizer
        self.k_store_mode = k_store_mode
        self.correction_impl = correction_impl
        self.k_channel_group = k_channel_group
        self.v_token_block = v_token_block
        self.bits_k = bits_k if bits_k > 0 else bits
        self.bits_v = bits_v if bits_v > 0 else bits
        self.max_pages = max_pages if max_pages > 0 else 512
        self.prefill_mode = prefill_mode
        self.name = (f"CAREKV_adaptive_rel{rel_threshold:.2f}" if mode == "adaptive"
                     else f"CAREKV_fixed_SK{sk}SV{sv}_RK{rk}RV{rv}")
        self.bit_width = f"INT{bits}"
        self.k_quant_scheme = "per-channel-group=32 + selected residual slots"
        self.v_quant_scheme = "per-channel-group=32 + selected residual slots"
        self.model = None

    def env(self) -> dict:
        """The CAREKV_* settings the reference adapter writes (carekv_adapter.py:106-150)."""
        e = dict(CAREKV_PREFILL_MODE=self.prefill_mode, CAREKV_PREFILL_RESIDUAL_KIND="both",
                 CAREKV_ROUTE_POLICY="joint", CAREKV_SCORE_NORMALIZE="1",
                 CAREKV_CORRECTION_IMPL=self.correction_impl, CAREKV_BUDGET_POLICY="uniform",
                 CAREKV_PACKED_BASE="1", CAREKV_SCALE_QUANT="int8", CAREKV_BASE_BITS=str(self.bits),
                 CAREKV_GROUP_SIZE="32", CAREKV_STORE_BUDGET_MODE="absolute",
                 CAREKV_STORE_ABS_K=str(self.sk), CAREKV_STORE_ABS_V=str(self.sv),
                 CAREKV_BASE_QUANTIZER=self.base_quantizer, CAREKV_K_BITS=str(self.bits_k),
                 CAREKV_V_BITS=str(self.bits_v), CAREKV_K_STORE_MODE=self.k_store_mode,
                 CAREKV_K_CHANNEL_GROUP=str(self.k_channel_group), CAREKV_V_TOKEN_BLOCK=str(self.v_token_block))
        if self.mode == "adaptive":
            e.update(CAREKV_READ_BUDGET_MODE="adaptive_score", CAREKV_READ_ABS_K=str(self.max_rk),
                     CAREKV_READ_ABS_V=str(self.max_rv), CAREKV_READ_RELATIVE_THRESHOLD=str(self.rel_threshold),
                     CAREKV_READ_ABSOLUTE_THRESHOLD="0.0", CAREKV_READ_MIN_KEEP="0")
        else:
            e.update(CAREKV_READ_BUDGET_MODE="absolute", CAREKV_READ_ABS_K=str(self.rk),
                     CAREKV_READ_ABS_V=str(self.rv), CAREKV_READ_RELATIVE_THRESHOLD="0.0",
                     CAREKV_READ_ABSOLUTE_THRESHOLD="0.0", CAREKV_READ_MIN_KEEP="0")
        return e

    def cache_config(self, hf_config) -> CacheConfig:
        """CacheConfig for an HF model config, after the adapter's env overrides."""
        H = hf_config.num_attention_heads
        kw = dict(num_layers=hf_config.num_hidden_layers, num_heads=H,
                  num_kv_heads=getattr(hf_config, "num_key_value_heads", H),
                  head_dim=getattr(hf_config, "head_dim", None) or hf_config.hidden_size // H,
                  max_pages=self.max_pages, route_policy="joint")
        return CacheConfig(**apply_carekv_env_overrides(kw))

    def setup_model(self, model_or_path, device: Optional[torch.device] = None):
        """Write the env, build the CacheConfig and patch the model (in place)."""
        for k, v in self.env().items():
            os.environ[k] = v
        model = model_or_path
        if isinstance(model_or_path, str):
            from transformers import LlamaForCausalLM
            model = LlamaForCausalLM.from_pretrained(model_or_path, local_files_only=True)
            if device is not None:
                model = model.to(device)
        self.care_cfg = self.cache_config(model.config)
        self.model = patch_llama_model(model, self.care_cfg, device)
        return self.model
