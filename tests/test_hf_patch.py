"""HF Llama patch (llama_patch.py:35-352 of the reference) on a tiny random Llama.

CPU: module replacement, layer ids, the CAREKV_RETURN=original passthrough and
the prefill-mode switches.  GPU: the patched model's prefill logits equal
the unpatched model's (CAREKV_PREFILL_MODE=fp attends over full-precision
K / V), decode steps through the CARE-KV cache stay close to the unpatched
model, and HF's cache length advances without full-size dummy tensors.
"""

import pytest
import torch

from conftest import load_pkg
from helpers import PAPER_BEST_ENV, env

transformers = pytest.importorskip("transformers")


def tiny_llama(seed=0):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(vocab_size=256, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512,
                      attn_implementation="eager")
    return LlamaForCausalLM(cfg).eval()


def care_cfg(pkg, layers=2, max_pages=16):
    return pkg.CacheConfig(num_layers=layers, num_heads=4, num_kv_heads=2, head_dim=64, page_size=16,
                           max_pages=max_pages, base_bits=3, group_size=32, packed_base=True, scale_quant="int8",
                           store_budget_mode="absolute", store_abs_k=1, store_abs_v=1,
                           read_budget_mode="absolute", read_abs_k=1, read_abs_v=1, route_policy="joint")


def test_patch_replaces_every_attention_module():
    pkg = load_pkg()
    model = tiny_llama()
    pkg.patch_llama_model(model, care_cfg(pkg), device=torch.device("cpu"))
    mods = [m for m in model.modules() if type(m).__name__ == "CAREKVLlamaAttention"]
    assert [m.layer_id for m in mods] == [0, 1]
    assert all(m.shared is mods[0].shared for m in mods)


def test_passthrough_matches_unpatched_on_cpu():
    pkg = load_pkg()
    ids = torch.randint(0, 256, (1, 12), generator=torch.Generator().manual_seed(3))
    ref = tiny_llama()
    with torch.no_grad():
        want = ref(ids).logits
    model = pkg.patch_llama_model(tiny_llama(), care_cfg(pkg), device=torch.device("cpu"))
    with env(CAREKV_RETURN="original"), torch.no_grad():
        got = model(ids).logits
    torch.testing.assert_close(got, want)


def test_prefill_mode_resolution_and_unbuilt_modes():
    pkg = load_pkg()
    from importlib import import_module
    layer_mod = import_module(pkg.__name__ + ".layer")
    for raw, want in (("fp", "fp"), ("quant", "base_quant"), ("int", "base_quant"), ("carekv", "carekv_eval"),
                      ("carekv_stored", "carekv_stored")):
        with env(CAREKV_PREFILL_MODE=raw):
            assert layer_mod.resolve_prefill_mode() == want
    cfg = care_cfg(pkg)
    W = torch.zeros(256, 256)
    layer = pkg.CAREKVLayer(cfg, 0, W, W[:128], W[:128], W)
    # the in-memory residual upper bound (layer.py:363-453) is the one prefill mode not built
    with env(CAREKV_PREFILL_MODE="carekv_eval"):
        with pytest.raises(NotImplementedError):
            layer.prefill(None, torch.zeros(4, 256))


@pytest.mark.gpu
def test_patched_model_prefill_and_decode_on_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from transformers import DynamicCache
    pkg = load_pkg()
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(4)
    prompt = torch.randint(0, 256, (2, 37), generator=g).to(dev)
    steps = torch.randint(0, 256, (2, 12), generator=g).to(dev)
    ref = tiny_llama().to(dev)
    with env(CAREKV_PREFILL_MODE="fp", **PAPER_BEST_ENV), torch.no_grad():
        model = pkg.patch_llama_model(tiny_llama().to(dev), care_cfg(pkg), device=dev)
        rc, pc = DynamicCache(), DynamicCache()
        want = ref(prompt, past_key_values=rc, use_cache=True).logits
        got = model(prompt, past_key_values=pc, use_cache=True).logits
        torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-4)
        for j in range(steps.shape[1]):
            tok = steps[:, j:j + 1]
            w = ref(tok, past_key_values=rc, use_cache=True).logits[:, -1]
            o = model(tok, past_key_values=pc, use_cache=True).logits[:, -1]
            assert torch.isfinite(o).all()
            cos = torch.nn.functional.cosine_similarity(o, w, dim=-1)
            assert (cos > 0.98).all(), (j, cos)
        assert pc.get_seq_length(0) == 37 + steps.shape[1]
        # the HF cache carries (B, 1, T, 1) placeholders, not K / V
        assert pc.layers[0].keys.shape[1] == 1 and pc.layers[0].keys.shape[-1] == 1
        cache = model._carekv_shared.cache
        assert cache.total_valid_tokens(0, 0, seq=1) == 37 + steps.shape[1]
        cache.check_errors()


def test_adapter_env_config_and_patch():
    pkg = load_pkg()
    from importlib import import_module
    ad_mod = import_module(pkg.__name__ + ".adapter")
    ad = ad_mod.CAREKVAdapter(sk=1, sv=1, rk=2, rv=3, max_pages=16)
    e = ad.env()
    assert e["CAREKV_STORE_ABS_K"] == "1" and e["CAREKV_READ_ABS_V"] == "3"
    assert e["CAREKV_READ_BUDGET_MODE"] == "absolute" and e["CAREKV_PREFILL_MODE"] == "carekv_stored"
    # the KIVI-style base is built; rotation / calibrated bases are not
    assert ad_mod.CAREKVAdapter(base_quantizer="kivi_style").base_quantizer == "kivi_style"
    with pytest.raises(NotImplementedError):
        ad_mod.CAREKVAdapter(base_quantizer="rotatekv_style")
    keys = list(e)
    saved = {k: __import__("os").environ.get(k) for k in keys}
    try:
        model = ad.setup_model(tiny_llama(), device=torch.device("cpu"))
        c = ad.care_cfg
        assert (c.num_layers, c.num_heads, c.num_kv_heads, c.head_dim) == (2, 4, 2, 64)
        assert (c.store_abs_k, c.store_abs_v, c.read_abs_k, c.read_abs_v) == (1, 1, 2, 3)
        assert c.base_bits == 3 and c.scale_quant == "int8" and c.packed_base
        assert sum(type(m).__name__ == "CAREKVLlamaAttention" for m in model.modules()) == 2
    finally:
        import os as _os
        for k, v in saved.items():
            if v is None:
                _os.environ.pop(k, None)
            else:
                _os.environ[k] = v
