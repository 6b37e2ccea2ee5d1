"""oracle/gqa_ref.py against the reference's own GroupQueryAttention oracle
(tests/ops/test_gqa_position_cache.py:88-134, rotary :71-85, attention_bias :119-121), its integer
oracle (tests/ops/test_quantized_kv.py:122-193, sliding caches included) and the sliding-cache
expectation of test_gqa_position_cache.py:427-488, fixtures in tests/golden/gqa_golden.npz."""

import json
import os

import numpy as np
import pytest

from oracle import gqa_ref

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "gqa_golden.npz")
DATA = np.load(GOLDEN)
META = json.loads(bytes(DATA["meta"]).decode())


def feeds_of(name):
    prefix = f"{name}/in/"
    return {k[len(prefix):]: DATA[k] for k in DATA.files if k.startswith(prefix)}


@pytest.mark.parametrize("case", META, ids=[c["name"] for c in META])
def test_oracle_matches_reference_oracle(case):
    f = feeds_of(case["name"])
    mode = case.get("mode", 0)
    res = gqa_ref.group_query_attention(
        f["q"], f["k"] if case["new_seq"] else None, f["v"] if case["new_seq"] else None, f["pk"], f["pv"],
        f["lengths"], f["total"], num_heads=4, kv_num_heads=2, causal=case["causal"], window=case["window"],
        softcap=0.7 if case["composed"] else 0.0, sink=f.get("sink"), cos=f.get("cos"), sin=f.get("sin"),
        position_ids=f.get("pos"), interleaved=case.get("interleaved", False), bias=f.get("bias"), qk_output=mode,
        k_scale=f.get("k_scale"), v_scale=f.get("v_scale"), sliding=case.get("sliding", False))
    out, pk, pv = res[:3]
    tol = 1e-5 if case["dtype"] == "float32" else 2e-3
    if mode:  # qk_output diagnostics
        np.testing.assert_allclose(res[3].astype(np.float32), DATA[f"{case['name']}/out/qk"].astype(np.float32),
                                   rtol=tol, atol=tol)
    want = DATA[f"{case['name']}/out/output"]
    np.testing.assert_allclose(out.astype(np.float32), want.astype(np.float32), rtol=tol, atol=tol)
    # present: the reference keeps the cap-row buffer; this restatement has max(cap, total) rows
    cap = case["cap"]
    np.testing.assert_array_equal(pk[:, :, :cap], DATA[f"{case['name']}/out/present_k"])
    np.testing.assert_array_equal(pv[:, :, :cap], DATA[f"{case['name']}/out/present_v"])


def test_growing_cache_appends_after_capacity():
    rng = np.random.default_rng(1)
    q = rng.normal(size=(1, 1, 4 * 32)).astype(np.float32)
    k = rng.normal(size=(1, 1, 2 * 32)).astype(np.float32)
    v = rng.normal(size=(1, 1, 2 * 32)).astype(np.float32)
    pk = rng.normal(size=(1, 2, 5, 32)).astype(np.float32)
    pv = rng.normal(size=(1, 2, 5, 32)).astype(np.float32)
    out, nk, nv = gqa_ref.group_query_attention(q, k, v, pk, pv, np.array([5]), 6, num_heads=4, kv_num_heads=2)
    assert nk.shape == (1, 2, 6, 32)
    np.testing.assert_array_equal(nk[:, :, :5], pk)
    np.testing.assert_array_equal(nk[0, :, 5], k[0, 0].reshape(2, 32))
    # one query over all 6 keys, by hand
    keys = nk[0].repeat(2, 0)
    vals = nv[0].repeat(2, 0)
    qh = q[0, 0].reshape(4, 32)
    s = np.einsum("hd,hkd->hk", qh, keys) / np.sqrt(32)
    p = np.exp(s - s.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    np.testing.assert_allclose(out[0, 0].reshape(4, 32), np.einsum("hk,hkd->hd", p, vals), rtol=1e-5, atol=1e-6)


def test_oracle_qk_norm_matches_reference_case():
    """q/k RMS norm inputs 14 / 15 (tests/ops/test_gqa11.py:52-130, fp32, eps 1e-5)."""
    f = {k.split("/")[-1]: DATA[k] for k in DATA.files if k.startswith("qknorm/in/")}
    out, pk, pv = gqa_ref.group_query_attention(
        f["q"], f["k"], f["v"], f["pk"], f["pv"], f["lengths"], f["total"], num_heads=4, kv_num_heads=2,
        q_norm=f["qw"], k_norm=f["kw"], norm_eps=float(f["eps"][0]))
    np.testing.assert_allclose(out, DATA["qknorm/out/output"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(pk, DATA["qknorm/out/present_k"], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(pv, DATA["qknorm/out/present_v"])
