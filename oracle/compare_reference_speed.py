"""Time the reference's own CPU decode path against the oracle port (host only).

Test and measurement infrastructure, never part of the product: it imports
the reference tree (pure PyTorch) from a checkout given on the command line,
so it runs where that checkout exists, not on a GPU box.

    python oracle/compare_reference_speed.py --reference /path/to/reference [--seconds 20]

One (sequence, layer, kv head) slice of the bench workload (Llama-2-7B MHA
shape: D 128, context 4096, INT3 g32, int8 page scales, 1 K + 1 V slot per
page, read ratio 0.03, joint top-k, paper-best router settings), one query:

  reference: CAREKVCache.read_base_concat -> dequantize -> logits, softmax,
             A @ V -> attention.vectorized_joint_correction
             (the reference decode hot path, attention.py:576-957)
  port:      oracle.decode_attention_kvh on the same seeded inputs

Prints one JSON line with seconds per slice for both and their ratio.
"""

import argparse
import json
import math
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

PAPER_ENV = {"CAREKV_KSCORE_LIVE": "1", "CAREKV_K_CORRECTION_MODE": "exact", "CAREKV_SCORE_NORMALIZE": "1",
             "CAREKV_STORE_POLICY": "residual_kind_aware", "CAREKV_PREFILL_RESIDUAL_KIND": "both"}


def time_loop(fn, seconds):
    fn()
    n, t0 = 0, time.perf_counter()
    while True:
        fn()
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 3:
            return el / n, n


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--seconds", type=float, default=20.0)
    ap.add_argument("--context", type=int, default=4096)
    args = ap.parse_args()
    os.environ.update(PAPER_ENV)
    from make_golden import import_reference, make_layer
    import_reference(args.reference)
    import torch
    import torch.nn.functional as F
    from CARE_KV.care_kv.cache import CacheConfig, CAREKVCache
    from CARE_KV.care_kv.quantizer import QuantConfig, dequantize
    from CARE_KV.care_kv.residual_router import ResidualRouter
    from CARE_KV.care_kv import attention as att
    import oracle
    from oracle import OracleCache, StoreConfig, RouteConfig

    D, N = 128, args.context
    rng = np.random.default_rng(0)
    K = rng.standard_normal((N, D)).astype(np.float32)
    K[:, :4] *= 20
    V = rng.standard_normal((N, D)).astype(np.float32)
    q = rng.standard_normal((1, D)).astype(np.float32)

    # reference
    cfg = CacheConfig(num_layers=1, num_heads=1, num_kv_heads=1, head_dim=D, page_size=16,
                      max_pages=(N + 15) // 16 + 1, base_bits=3, group_size=32, k_channel_group=32,
                      v_token_block=4, sketch_dim=32, packed_base=True, scale_quant="int8",
                      store_budget_mode="absolute", store_abs_k=1, store_abs_v=1, read_budget_mode="ratio",
                      read_budget_ratio=0.03, route_policy="joint")
    layer = make_layer(cfg, 1, 1, D, "fp32", 0)
    cache = CAREKVCache(cfg)
    layer._write_pages_for_kv_head(cache, 0, torch.from_numpy(K), torch.from_numpy(V), token_start_abs=0,
                                   sink_tokens=4)
    router = ResidualRouter(cfg, 0, torch.device("cpu"))
    qc = QuantConfig(bits=3, group_size=32)
    Qq = torch.from_numpy(q)

    def ref_step():
        pids = cache.all_page_ids(0, 0)
        Kc, Ks, Vc, Vs, _ = cache.read_base_concat(0, 0, pids)
        Nv = Kc.shape[0]
        Kb = dequantize(Kc, Ks, (Nv, D), qc).float()
        Vb = dequantize(Vc, Vs, (Nv, D), qc).float()
        S = (Kb @ Qq.T).T * (1.0 / math.sqrt(D))
        A = F.softmax(S, dim=-1)
        O = A @ Vb
        return O + att.vectorized_joint_correction(cache, cfg, router, 0, 0, pids, Q_q=Qq, S=S, A=A, V_base=Vb,
                                                   O_base=O, kind="both", k_corr_scale=0.1, score_normalize=True)

    # port
    sc = StoreConfig(head_dim=D, base_bits=3, group_size=32, store_abs_k=1, store_abs_v=1)
    oc = OracleCache(1, 1, D, (N + 15) // 16 + 8, sc, scale_quant="int8")
    oc.prefill_write(0, 0, K, V, "fp32")
    rc = RouteConfig(head_dim=D, read_budget_mode="ratio", read_budget_ratio=0.03)

    def port_step():
        return oracle.decode_attention_kvh(oc, 0, 0, q, rc)

    t_ref, n_ref = time_loop(ref_step, args.seconds)
    t_port, n_port = time_loop(port_step, args.seconds)
    print(json.dumps(dict(context=N, torch_threads=torch.get_num_threads(), reference_s_per_slice=t_ref,
                          reference_steps=n_ref, port_s_per_slice=t_port, port_steps=n_port,
                          port_over_reference_speed=t_ref / t_port)))


if __name__ == "__main__":
    main()
