"""The CPU oracle against golden vectors produced by the reference's own numpy oracles.

``tests/golden/paged_golden.npz`` holds outputs of the reference's ``_paged_ref``
(tests/ops/test_paged_attention.py:63-158), its quantized ``_paged_ref``
(tests/ops/test_quantized_kv.py:395-450) and its ``_encode``/``_decode``
(tests/ops/test_quantized_kv.py:22-47), computed on the inputs that ``cases.py`` rebuilds.
"""

import numpy as np
import pytest

import cases
from make_golden import digest
from oracle import paged_ref as ref

GOLDEN = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden",
                                            "paged_golden.npz"))


def _float_call(case, feeds):
    kw = dict(case.get("ref_kwargs", {}))
    call = dict(
        slot_mapping=feeds.get("slot_mapping"),
        is_causal=kw.get("is_causal", True),
        local_window_size=kw.get("local_window_size", -1),
        head_sink=feeds.get("head_sink"),
        cos=feeds.get("cos"), sin=feeds.get("sin"),
        interleaved=bool(kw.get("interleaved", 0)),
        q_norm=feeds.get("q_norm"), k_norm=feeds.get("k_norm"),
        norm_eps=kw.get("norm_eps", 1e-6),
    )
    return ref.paged_attention(
        feeds["query"], feeds["key"], feeds["value"], feeds["key_cache"], feeds["value_cache"],
        feeds["cumulative_sequence_length"], feeds["past_seqlens"], feeds["block_table"],
        case["H"], case["KV"], **call)


def _apply_delta(cache, slots, rows):
    flat = cache.reshape(cache.shape[0] * cache.shape[1], -1).copy()
    if len(slots):
        flat[slots] = rows.reshape(len(slots), -1)
    return flat.reshape(cache.shape)


FLOAT_CASES = [c for c in cases.float_cases() if not c["name"].startswith("long_p16383")]


@pytest.mark.parametrize("case", FLOAT_CASES, ids=lambda c: c["name"])
def test_oracle_matches_reference_float(case):
    feeds = cases.float_inputs(case)
    name = case["name"]
    assert digest(cases.input_arrays(feeds)) == str(GOLDEN[f"{name}/digest"]), "input stream changed"
    out, kc, vc = _float_call(case, feeds)
    want = GOLDEN[f"{name}/output"]
    # fp32 restatement vs fp32 reference: only the activation rounding after RoPE / norm differs.
    np.testing.assert_allclose(out, want, rtol=2e-3, atol=2e-3 * max(1.0, float(np.abs(want).max())) * 1e-2 + 1e-4)
    for tag, got, before in (("k", kc, feeds["key_cache"]), ("v", vc, feeds["value_cache"])):
        expect = _apply_delta(before, GOLDEN[f"{name}/{tag}_slots"], GOLDEN[f"{name}/{tag}_rows"])
        np.testing.assert_array_equal(got.view(np.uint16), expect.view(np.uint16))


@pytest.mark.parametrize("case", cases.quant_cases(), ids=lambda c: c["name"])
def test_oracle_matches_reference_quant(case):
    feeds = cases.quant_inputs(case)
    name = case["name"]
    assert digest(cases.input_arrays(feeds)) == str(GOLDEN[f"{name}/digest"])
    kv, head = 2, case["head"]
    kq = ref.QuantSpec(case["bits"], feeds["k_scale"])
    vq = ref.QuantSpec(case["bits"], feeds["v_scale"])
    out, pk, pv = ref.paged_attention(
        feeds["q"], feeds["k"], feeds["v"], feeds["pk"], feeds["pv"], feeds["cum"], feeds["past"],
        feeds["table"], 4, kv, slot_mapping=feeds.get("slots"),
        is_causal=case.get("causal", True), local_window_size=case.get("window", -1),
        softcap=0.7 if case.get("composed") else 0.0, head_sink=feeds.get("sink"),
        cos=feeds.get("cos"), sin=feeds.get("sin"), kquant=kq, vquant=vq, head_size=head)
    np.testing.assert_array_equal(pk, GOLDEN[f"{name}/pk"])
    np.testing.assert_array_equal(pv, GOLDEN[f"{name}/pv"])
    want = GOLDEN[f"{name}/output"]
    # the reference packs the output in the activation dtype (fp16)
    np.testing.assert_allclose(out, want, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("scale", [1.0, 0.0, 0.3])
def test_codec_byte_equations(bits, scale):
    values = GOLDEN["codec/values"]
    s = np.array([scale], np.float32)
    key = f"codec/{bits}/{scale}"
    codes = ref.quant_encode(values, s, bits, paged=True)
    np.testing.assert_array_equal(codes, GOLDEN[f"{key}/codes"])
    np.testing.assert_array_equal(ref.quant_encode(values, s, bits, paged=False),
                                  GOLDEN[f"{key}/codes_gqa"])
    np.testing.assert_array_equal(ref.quant_decode(codes, s, bits, 16), GOLDEN[f"{key}/decoded"])


# The C restatement (oracle/paged_ref.c, through oracle/cpu_oracle.py) is the checker of the
# full-size GPU parity tests and the timed CPU baseline; it covers float caches without RoPE or
# q/k norm, so it is pinned on those golden cases, in both output modes.
C_CASES = [c for c in FLOAT_CASES if not any(k in cases.float_inputs(c) for k in ("cos", "q_norm"))]


@pytest.mark.parametrize("case", C_CASES, ids=lambda c: c["name"])
def test_c_oracle_matches_reference_float(case):
    from oracle import cpu_oracle

    feeds = cases.float_inputs(case)
    name = case["name"]
    kw = dict(case.get("ref_kwargs", {}))
    sink = feeds.get("head_sink")
    call = dict(slot_mapping=feeds.get("slot_mapping"), is_causal=kw.get("is_causal", True),
                local_window_size=kw.get("local_window_size", -1),
                head_sink=None if sink is None else sink.astype(np.float32), threads=2)
    meta = [feeds[n] for n in ("cumulative_sequence_length", "past_seqlens", "block_table")]
    want = GOLDEN[f"{name}/output"]
    kc, vc = feeds["key_cache"].copy(), feeds["value_cache"].copy()
    out32 = cpu_oracle.paged_attention(feeds["query"], feeds["key"], feeds["value"], kc, vc, *meta,
                                       case["H"], case["KV"], fp32_out=True, **call)
    # fp32 against fp32: only the summation order differs (eight-lane partial sums here)
    np.testing.assert_allclose(out32, want, rtol=1e-4, atol=1e-4)
    for tag, got, before in (("k", kc, feeds["key_cache"]), ("v", vc, feeds["value_cache"])):
        expect = _apply_delta(before, GOLDEN[f"{name}/{tag}_slots"], GOLDEN[f"{name}/{tag}_rows"])
        np.testing.assert_array_equal(got.view(np.uint16), expect.view(np.uint16))
    # the rounded mode is the fp32 output rounded once to the activation dtype
    out16 = cpu_oracle.paged_attention(feeds["query"], feeds["key"], feeds["value"], feeds["key_cache"].copy(),
                                       feeds["value_cache"].copy(), *meta, case["H"], case["KV"], **call)
    np.testing.assert_array_equal(out16, out32.astype(out16.dtype))


def latent_oracle(feeds, case=cases.LATENT):
    return ref.paged_attention(
        feeds["query"], feeds["key"], None, feeds["key_cache"], None, feeds["cumulative_sequence_length"],
        feeds["past_seqlens"], feeds["block_table"], case["H"], case["KV"], scale=case["scale"],
        cos=feeds["cos"], sin=feeds["sin"], rotary_offset=case["offset"], latent_v_head=case["vd"])


def test_oracle_matches_reference_latent():
    """LATENT layout (test_paged_attention.py:669-764): values are the first vd channels of the
    rotated keys; the appended key rows are bit-exact, the output within the activation rounding
    of the rotated rows (the reference test keeps them in fp32)."""
    feeds = cases.latent_inputs()
    assert digest(cases.input_arrays(feeds)) == str(GOLDEN["latent/digest"])
    out, kc, vc = latent_oracle(feeds)
    assert vc is None
    np.testing.assert_array_equal(kc.view(np.uint16), GOLDEN["latent/key_cache"].view(np.uint16))
    np.testing.assert_allclose(out, GOLDEN["latent/output"], rtol=2e-3, atol=2e-3)
