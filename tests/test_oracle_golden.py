"""Pin the CPU oracle to the reference through its golden fixtures (CPU only).

The fixtures in tests/golden/ were produced by running the reference
package itself (tests/golden/make_golden.py).  Integer and byte outputs must
match bit for bit; floating outputs match to the stated tolerances.
"""

import json
import os

import numpy as np
import pytest

import oracle
from oracle import StoreConfig, OracleCache, RouteConfig

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    z = np.load(os.path.join(GOLDEN, name), allow_pickle=False)
    return z, json.loads(str(z["meta"]))


def test_quant_golden():
    z, cases = _load("quant.npz")
    assert len(cases) == 27
    for c in cases:
        k, dt, bits, gs = c["key"], c["dt"], c["bits"], c["group_size"]
        x = z[k + "_x"]
        codes, scale = oracle.quantize(x, bits, gs, dt)
        assert np.array_equal(codes, z[k + "_codes"]), (c, "codes")
        assert np.array_equal(scale, z[k + "_scale"]), (c, "scale")
        assert np.array_equal(oracle.pack_codes_2d(codes, bits), z[k + "_packed"]), (c, "packed")
        assert np.array_equal(oracle.unpack_codes_2d(z[k + "_packed"], bits, c["D"]), codes)
        xh = oracle.dequantize(codes, scale, gs, dt)
        assert np.array_equal(xh, z[k + "_xhat"]), (c, "x_hat")
        _, _, res = oracle.quantize_and_residual(x, bits, gs, dt)
        assert np.array_equal(res, z[k + "_resid"]), (c, "residual")
        s8, master = oracle.int8_scale_write(scale, dt)
        assert np.array_equal(s8, z[k + "_s8"]), (c, "int8 scale codes")
        assert np.float32(master) == z[k + "_master"], (c, "master")
        r4, r4s, _ = oracle.pack_4bit(res[:, :32])
        assert np.array_equal(r4, z[k + "_r4"]), (c, "4-bit slot")
        assert np.float32(r4s) == z[k + "_r4s"], (c, "4-bit slot scale")


def _store_cfg(c):
    return StoreConfig(head_dim=c["D"], page_size=16, base_bits=c["bits"], group_size=c["group_size"],
                       k_channel_group=32, v_token_block=4, sketch_dim=32,
                       store_budget_mode=c["store_budget_mode"], store_abs_k=c["store_abs_k"],
                       store_abs_v=c["store_abs_v"], store_budget_ratio=c["store_budget_ratio"],
                       store_policy=c["store_policy"], residual_kind=c["kind"])


def _check_cache(oc, z, key, c):
    assert np.array_equal(oc.k_codes, z[key + "_kcodes"]), "K codes"
    assert np.array_equal(oc.v_codes, z[key + "_vcodes"]), "V codes"
    if c["scale_quant"] == "int8":
        assert np.array_equal(oc.k_scale, z[key + "_kscale"]), "K int8 scales"
        assert np.array_equal(oc.v_scale, z[key + "_vscale"]), "V int8 scales"
        assert np.array_equal(oc.k_master, z[key + "_kmaster"]), "K masters"
        assert np.array_equal(oc.v_master, z[key + "_vmaster"]), "V masters"
    else:
        assert np.array_equal(oc.k_scale, z[key + "_kscale"]), "K scales"
        assert np.array_equal(oc.v_scale, z[key + "_vscale"]), "V scales"
    assert np.array_equal(oc.valid, z[key + "_valid"]), "valid tokens"
    assert np.array_equal(oc.next_page, z[key + "_npages"]), "page counts"
    metas = json.loads(str(z[key + "_meta"]))
    for m in metas:
        om = oc.meta[m["l"]][m["h"]][m["p"]]
        assert om is not None
        assert om["k_slots"] == m["k"], ("K slot ids", m)
        assert om["v_slots"] == m["v"], ("V slot ids", m)
        tag = f"{m['l']}_{m['h']}_{m['p']}"
        # error norms are fp32 reductions stored as fp16: allow one fp16 ulp
        np.testing.assert_allclose(om["k_err"], z[f"{key}_kerr_{tag}"], rtol=1e-3, atol=1e-7)
        np.testing.assert_allclose(om["v_err"], z[f"{key}_verr_{tag}"], rtol=1e-3, atol=1e-7)
        np.testing.assert_allclose(om["k_sketch"], z[f"{key}_ksk_{tag}"], rtol=2e-3, atol=1e-6)
    kb = z[key + "_kbuf"]
    assert oc.next_k_slot == kb.shape[0]
    for sid in range(kb.shape[0]):
        assert np.array_equal(oc.k_slots[sid][0], kb[sid]), ("K slot payload", sid)
        assert np.float32(oc.k_slots[sid][1]) == z[key + "_kbufs"][sid]
    vb = z[key + "_vbuf"]
    assert oc.next_v_slot == vb.shape[0]
    for sid in range(vb.shape[0]):
        assert np.array_equal(oc.v_slots[sid][0], vb[sid]), ("V slot payload", sid)
        assert np.float32(oc.v_slots[sid][1]) == z[key + "_vbufs"][sid]


@pytest.mark.parametrize("ci", range(7))
def test_store_and_decode_golden(ci):
    z, cases = _load("store_decode.npz")
    c = cases[ci]
    key, dt = c["key"], c["dt"]
    oc = OracleCache(1, c["Hkv"], c["D"], c["max_pages"], _store_cfg(c),
                     scale_quant=c["scale_quant"])
    K, V = z[key + "_K"], z[key + "_V"]
    for h in range(c["Hkv"]):
        oc.prefill_write(0, h, K[h], V[h], dt)
    _check_cache(oc, z, key, c)

    rc = RouteConfig(head_dim=c["D"])
    grp = c["Hq"] // c["Hkv"]
    for s in range(c["steps"]):
        pos = int(oc.valid[0, 0, :oc.next_page[0, 0]].sum())
        for h in range(c["Hkv"]):
            oc.append(0, h, z[key + "_dk"][s][h], z[key + "_dv"][s][h], dt, pos_abs=pos)
        O_ref = z[key + "_dO"][s]
        for h in range(c["Hkv"]):
            q = z[key + "_dq"][s][h * grp:(h + 1) * grp]
            O, _ = oracle.decode_attention_kvh(oc, 0, h, q, rc, correction=False)
            O = oracle.round_to(O, dt)
            # the reference returns O rounded to the model dtype: allow one ulp of it
            tol = {"fp32": 1e-5, "fp16": 2e-3, "bf16": 8e-3}[dt]
            np.testing.assert_allclose(O, O_ref[h * grp:(h + 1) * grp], rtol=tol, atol=tol)
    _check_cache(oc, z, key + "d", c)


@pytest.mark.parametrize("ci", range(9))
def test_correction_golden(ci):
    z, cases = _load("correction.npz")
    c = cases[ci]
    key = c["key"]
    D, Hq, Hkv = c["D"], c["Hq"], c["Hkv"]
    scfg = StoreConfig(head_dim=D, base_bits=3, group_size=32, store_budget_mode="absolute",
                       store_abs_k=c["store_abs_k"], store_abs_v=c["store_abs_v"])
    oc = OracleCache(1, Hkv, D, c["max_pages"], scfg, scale_quant="int8")
    K, V, Q = z[key + "_K"], z[key + "_V"], z[key + "_Q"]
    for h in range(Hkv):
        oc.prefill_write(0, h, K[h], V[h], "fp32")
    rc = RouteConfig(head_dim=D, kind=c["kind"], route_policy=c["route_policy"],
                     score_normalize=c["score_normalize"], kscore_live=c["kscore_live"],
                     k_correction_mode=c["k_correction_mode"], k_corr_scale=0.1,
                     read_budget_mode=c["read_budget_mode"], read_abs_k=c["read_abs_k"],
                     read_abs_v=c["read_abs_v"], read_budget_ratio=c["read_budget_ratio"])
    grp = Hq // Hkv
    for h in range(Hkv):
        S, A, O = z[f"{key}_S_{h}"], z[f"{key}_A_{h}"], z[f"{key}_O_{h}"]
        Kh, Vh, _ = oc.read_base_concat(0, h)
        q = Q[h * grp:(h + 1) * grp]
        S2, A2, O2 = oracle.base_attention(Kh, Vh, q, D)
        np.testing.assert_allclose(S2, S, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(A2, A, rtol=1e-4, atol=1e-7)
        np.testing.assert_allclose(O2, O, rtol=1e-4, atol=1e-5)
        delta, info = oracle.vectorized_joint_correction(oc, 0, h, q, S, A, Vh, O, rc)
        for nm, onm in (("score_K", "score_K"), ("score_V", "score_V")):
            gk = f"{key}_{nm}_{h}"
            if gk in z:
                np.testing.assert_allclose(info[onm], z[gk], rtol=2e-5, atol=1e-9)
        for nm in ("sel_k", "sel_v"):
            gk = f"{key}_{nm}_{h}"
            if gk in z:
                assert np.array_equal(info[nm], z[gk]), (c["name"], h, nm)
        reads = z[f"{key}_reads_{h}"]
        assert info["k_reads"] == reads[0] and info["v_reads"] == reads[1], (c["name"], h)
        np.testing.assert_allclose(delta, z[f"{key}_delta_{h}"], rtol=1e-4, atol=2e-6)
        if c["name"] == "read0":
            assert np.all(delta == 0)


# ───────────────────────────── KIVI helpers ─────────────────────────────
KIVI = np.load(os.path.join(GOLDEN, "kivi.npz"))
KIVI_META = json.loads(str(KIVI["meta"]))


@pytest.mark.parametrize("case", KIVI_META, ids=[f"{c['dtype']}_b{c['bits']}_{c['key']}" for c in KIVI_META])
def test_oracle_kivi_matches_reference(case):
    from oracle.quant import kivi_quant_dequant
    x = KIVI[case["key"] + "_x"]
    for axis, name in ((-2, "_k"), (-1, "_v")):
        got = kivi_quant_dequant(x, case["bits"], case["dtype"], axis)
        np.testing.assert_array_equal(got, KIVI[case["key"] + name], err_msg=f"{case['key']}{name}")


def _check_kivi_cache(oc, z, key):
    """fp16 side buffers bit for bit (NaN where the reference has NaN), valid
    counts, slot ids, payloads and error norms."""
    np.testing.assert_array_equal(oc.k_hat16, z[key + "_khat"], err_msg="K_hat side buffer")
    np.testing.assert_array_equal(oc.v_hat16, z[key + "_vhat"], err_msg="V_hat side buffer")
    assert np.array_equal(oc.valid, z[key + "_valid"]), "valid tokens"
    assert np.array_equal(oc.next_page, z[key + "_npages"]), "page counts"
    for m in json.loads(str(z[key + "_meta"])):
        om = oc.meta[m["l"]][m["h"]][m["p"]]
        assert om is not None
        assert om["k_slots"] == m["k"], ("K slot ids", m)
        assert om["v_slots"] == m["v"], ("V slot ids", m)
        tag = f"{m['l']}_{m['h']}_{m['p']}"
        np.testing.assert_allclose(om["k_err"], z[f"{key}_kerr_{tag}"], rtol=1e-3, atol=1e-7)
        np.testing.assert_allclose(om["v_err"], z[f"{key}_verr_{tag}"], rtol=1e-3, atol=1e-7)
    for kind, slots, nxt in (("k", oc.k_slots, oc.next_k_slot), ("v", oc.v_slots, oc.next_v_slot)):
        buf = z[f"{key}_{kind}buf"]
        assert nxt == buf.shape[0]
        for sid in range(buf.shape[0]):
            assert np.array_equal(slots[sid][0], buf[sid]), (kind, "payload", sid)
            assert np.float32(slots[sid][1]) == z[f"{key}_{kind}bufs"][sid]


@pytest.mark.parametrize("ci", range(4))
def test_kivi_store_and_decode_golden(ci):
    """KIVI-style base (base_quantizer='kivi_style'): per-channel K / per-token
    V prefill store, decode appends and base decode attention against the
    reference's own outputs."""
    z, cases = _load("kivi_store.npz")
    c = cases[ci]
    key, dt = c["key"], c["dt"]
    sc = StoreConfig(head_dim=c["D"], base_bits=c["bits"], group_size=32, store_abs_k=c["store_abs_k"],
                     store_abs_v=c["store_abs_v"], store_budget_mode="absolute")
    oc = OracleCache(1, c["Hkv"], c["D"], c["max_pages"], sc, scale_quant="none", base="kivi")
    K, V = z[key + "_K"], z[key + "_V"]
    for h in range(c["Hkv"]):
        oc.prefill_write(0, h, K[h], V[h], dt)
    _check_kivi_cache(oc, z, key)
    rc = RouteConfig(head_dim=c["D"])
    grp = c["Hq"] // c["Hkv"]
    for s in range(c["steps"]):
        pos = int(oc.valid[0, 0, :oc.next_page[0, 0]].sum())
        for h in range(c["Hkv"]):
            oc.append(0, h, z[key + "_dk"][s][h], z[key + "_dv"][s][h], dt, pos_abs=pos)
        O_ref = z[key + "_dO"][s]
        for h in range(c["Hkv"]):
            O, _ = oracle.decode_attention_kvh(oc, 0, h, z[key + "_dq"][s][h * grp:(h + 1) * grp], rc,
                                               correction=False)
            tol = {"fp32": 1e-5, "fp16": 2e-3, "bf16": 8e-3}[dt]
            np.testing.assert_allclose(oracle.round_to(O, dt), O_ref[h * grp:(h + 1) * grp], rtol=tol, atol=tol)
    _check_kivi_cache(oc, z, key + "d")


def _legacy_setup(c, z):
    from oracle.legacy_router import legacy_correction  # noqa: F401
    sc = StoreConfig(head_dim=c["D"], base_bits=3, group_size=32, store_abs_k=c["store_abs_k"],
                     store_abs_v=c["store_abs_v"], store_budget_mode="absolute", sketch_dim=32)
    oc = OracleCache(1, c["Hkv"], c["D"], 24, sc, scale_quant="int8")
    K, V = z[c["key"] + "_K"], z[c["key"] + "_V"]
    for h in range(c["Hkv"]):
        oc.prefill_write(0, h, K[h], V[h], "fp32")
    rc = RouteConfig(head_dim=c["D"], kind=c["kind"], route_policy=c["policy"], score_normalize=c["normalize"],
                     k_correction_mode=c["kmode"], read_budget_mode=c["read_mode"], read_abs_k=c["read_abs_k"],
                     read_abs_v=c["read_abs_v"], read_budget_ratio=c["ratio"])
    return oc, rc


@pytest.mark.parametrize("ci", range(11))
def test_legacy_router_golden(ci):
    """The legacy cached router (ResidualRouter.route + apply_slot_corrections)
    against the reference's per-query-head decode attention."""
    from oracle.legacy_router import legacy_correction
    z, cases = _load("legacy_router.npz")
    c = cases[ci]
    oc, rc = _legacy_setup(c, z)
    sels = json.loads(str(z[c["key"] + "_sel"]))
    Q = z[c["key"] + "_Q"]
    n = 0
    for h in range(c["Hkv"]):
        K_hat, V_hat, _ = oc.read_base_concat(0, h)
        for j in range(Q.shape[1]):
            q = Q[h, j]
            S, A, O = oracle.base_attention(K_hat, V_hat, q[None], c["D"])
            d, info = legacy_correction(oc, 0, h, q, S[0], A[0], O[0], V_hat, rc, oc.sketch_P, kind=c["kind"],
                                        score_normalize=c["normalize"], k_corr_scale=c["k_corr_scale"],
                                        exact=c["kmode"] == "exact", baseline=c["baseline"], rel_thr=c["rel"],
                                        abs_thr=c["abs"], min_keep=c["min_keep"])
            want = sels[n]
            assert sorted(map(list, info["k_sel"])) == sorted(want["k"]), (h, j, info["k_sel"], want["k"])
            assert sorted(map(list, info["v_sel"])) == sorted(want["v"]), (h, j, info["v_sel"], want["v"])
            np.testing.assert_allclose(O[0] + d, z[c["key"] + "_O"][n], rtol=1e-4, atol=1e-5, err_msg=f"{h} {j}")
            n += 1
