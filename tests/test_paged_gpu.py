"""GPU parity of the PagedAttention path against the golden vectors and the CPU oracle.

Golden cases restate the reference's own tests (tests/ops/test_paged_attention.py,
tests/ops/test_quantized_kv.py) with their tolerances; caches are compared bit-exactly
(the reference compares them with assert_array_equal).
"""

import numpy as np
import pytest

import cases
from oracle import paged_ref as ref

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # collected on CPU boxes, skipped there
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_helpers import run_float_case, to_dev, to_np  # noqa: E402

GOLDEN = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden",
                                            "paged_golden.npz"))

# Reference tolerances per test family (test_paged_attention.py :234, :316, :376, :441, :826).
TOL = {"core": (2e-2, 2e-2), "head256": (2e-2, 2e-2), "replay": (2e-2, 2e-2),
       "multiblock": (2e-2, 2e-2), "long": (3e-3, 2e-4), "overlay": (3e-3, 2e-4),
       "prefill": (3e-3, 2e-4), "writeback": (2e-2, 2e-2), "rotary": (2e-2, 2e-2),
       "ort129": (2e-2, 2e-2), "duplicate": (2e-2, 2e-2)}


def _expected_cache(before, slots, rows):
    flat = before.reshape(before.shape[0] * before.shape[1], -1).copy()
    if len(slots):
        flat[slots] = rows.reshape(len(slots), -1)
    return flat.reshape(before.shape)


def _attrs(case):
    kw = dict(case.get("ref_kwargs", {}))
    out = {}
    if "is_causal" in kw:
        out["is_causal"] = int(kw["is_causal"])
    if "local_window_size" in kw:
        out["local_window_size"] = kw["local_window_size"]
    if "interleaved" in kw:
        out["rotary_interleaved"] = kw["interleaved"]
    if "norm_eps" in kw:
        out["qk_norm_epsilon"] = kw["norm_eps"]
    return out


FLOAT_CASES = cases.float_cases()


@pytest.mark.parametrize("path", ["auto", "generic"])
@pytest.mark.parametrize("case", FLOAT_CASES, ids=lambda c: c["name"])
def test_golden_float(case, path):
    feeds = cases.float_inputs(case)
    out, kc, vc = run_float_case(feeds, case["H"], case["KV"], attrs=_attrs(case),
                                 force_generic=(path == "generic"))
    name = case["name"]
    want = GOLDEN[f"{name}/output"]
    family = name.split("_")[0]
    if family == "vector":
        np.testing.assert_allclose(out, want.astype(np.float16).astype(np.float32), rtol=2e-3, atol=0.5)
    else:
        rtol, atol = TOL[family]
        np.testing.assert_allclose(out, want, rtol=rtol, atol=atol)
    for tag, got, before in (("k", kc, feeds["key_cache"]), ("v", vc, feeds["value_cache"])):
        expect = _expected_cache(before, GOLDEN[f"{name}/{tag}_slots"], GOLDEN[f"{name}/{tag}_rows"])
        if "q_norm" in feeds:  # normalised rows: reference compares with rtol=atol=2e-3
            np.testing.assert_allclose(got.astype(np.float32), expect.astype(np.float32), rtol=2e-3, atol=2e-3)
        else:
            np.testing.assert_array_equal(got.view(np.uint16), expect.view(np.uint16))


def test_device_metadata_matches_host_metadata():
    case = next(c for c in FLOAT_CASES if c["name"] == "writeback_g1_r1_s88")
    feeds = cases.float_inputs(case)
    a = run_float_case(feeds, case["H"], case["KV"], metadata="host")
    b = run_float_case(feeds, case["H"], case["KV"], metadata="device")
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


def test_duplicate_slots_last_writer_wins():
    """test_paged_attention.py:605-663: two tokens write slot 0; the later token's row stays
    and the input cache equals the cache output (aliased)."""
    case = next(c for c in FLOAT_CASES if c["name"] == "duplicate_slots")
    feeds = cases.float_inputs(case)
    for metadata in ("host", "device"):
        _, kc, vc = run_float_case(feeds, 1, 1, metadata=metadata)
        assert np.all(kc[0, 0, 0] == 2) and np.all(vc[0, 0, 0] == 4)


@pytest.mark.parametrize("case", cases.quant_cases(), ids=lambda c: c["name"])
def test_golden_quant(case):
    from onnxruntime_ep_b200 import paged_attention
    feeds = cases.quant_inputs(case)
    name = case["name"]
    q, k, v = (to_dev(feeds[n]) for n in ("q", "k", "v"))
    pk, pv = to_dev(feeds["pk"]), to_dev(feeds["pv"])
    kw = {}
    if "cos" in feeds:
        kw.update(cos_cache=to_dev(feeds["cos"]), sin_cache=to_dev(feeds["sin"]), do_rotary=1)
    if "sink" in feeds:
        kw["head_sink"] = to_dev(feeds["sink"])
    modes = case["modes"]
    out, pk2, pv2 = paged_attention(
        q, k, v, pk, pv, torch.from_numpy(feeds["cum"]), torch.from_numpy(feeds["past"]),
        torch.from_numpy(feeds["table"]),
        slot_mapping=None if "slots" not in feeds else torch.from_numpy(feeds["slots"]),
        k_scale=to_dev(feeds["k_scale"].reshape(-1)), v_scale=to_dev(feeds["v_scale"].reshape(-1)),
        num_heads=4, kv_num_heads=2, k_quant_type=modes[0], v_quant_type=modes[1],
        is_causal=int(case.get("causal", True)), local_window_size=case.get("window", -1),
        softcap=0.7 if case.get("composed") else 0.0, check_status=True, **kw)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(pk2.cpu().numpy(), GOLDEN[f"{name}/pk"])
    np.testing.assert_array_equal(pv2.cpu().numpy(), GOLDEN[f"{name}/pv"])
    np.testing.assert_allclose(out.float().cpu().numpy(), GOLDEN[f"{name}/output"], rtol=2e-2, atol=2e-2)


# ------------------------------------------------------------------------------------------
# bf16 decode at the BASELINE geometry (32 q / 8 kv heads, d=128, bs=16), reduced batch.
# ------------------------------------------------------------------------------------------
def decode_feeds(seed, B, H, KV, D, bs, lo, hi, nb, dtype=None, nq=1, scale_kv=None):
    dtype = dtype or ref.BF16
    rng = np.random.default_rng(seed)
    L = rng.integers(lo, hi, size=B, endpoint=True)
    maxb = int(-(-int(L.max()) // bs))
    perm = rng.permutation(nb)
    bt = np.zeros((B, maxb), np.int32)
    off = 0
    for b in range(B):
        n = -(-int(L[b]) // bs)
        bt[b, :n] = perm[off:off + n]
        off += n
    s = scale_kv if scale_kv is not None else 1.0 / np.sqrt(D)
    nt = B * nq
    feeds = {
        "query": (rng.standard_normal((nt, H * D), np.float32) * s).astype(dtype),
        "key": (rng.standard_normal((nt, KV * D), np.float32) * s).astype(dtype),
        "value": (rng.standard_normal((nt, KV * D), np.float32) * s).astype(dtype),
        "key_cache": (rng.standard_normal((nb, bs, KV, D), np.float32) * s).astype(dtype),
        "value_cache": (rng.standard_normal((nb, bs, KV, D), np.float32) * s).astype(dtype),
        "cumulative_sequence_length": (np.arange(B + 1) * nq).astype(np.int32),
        "past_seqlens": (L - nq).astype(np.int32),
        "block_table": bt,
    }
    return feeds


def oracle_float(feeds, H, KV, **kw):
    return ref.paged_attention(
        feeds["query"], feeds["key"], feeds["value"], feeds["key_cache"], feeds["value_cache"],
        feeds["cumulative_sequence_length"], feeds["past_seqlens"], feeds["block_table"], H, KV,
        slot_mapping=feeds.get("slot_mapping"), **kw)


@pytest.mark.parametrize("nq,H,KV", [(1, 32, 8), (2, 32, 8), (1, 64, 8), (8, 8, 8)])
@pytest.mark.parametrize("metadata", ["host", "device"])
def test_bf16_decode_matches_oracle(nq, H, KV, metadata):
    feeds = decode_feeds(7 + nq + H, B=12, H=H, KV=KV, D=128, bs=16, lo=nq, hi=1200, nb=1200, nq=nq)
    out, kc, vc = run_float_case(feeds, H, KV, metadata=metadata)
    want, wkc, wvc = oracle_float(feeds, H, KV)
    # BASELINE tolerance: max-abs 2e-3 against the fp32 recomputation (bf16 output rounding
    # is part of the measured error).
    assert np.abs(out - want).max() <= 2e-3
    np.testing.assert_array_equal(kc.view(np.uint16), wkc.view(np.uint16))
    np.testing.assert_array_equal(vc.view(np.uint16), wvc.view(np.uint16))


@pytest.mark.parametrize("tiles", [1, 3, 8, 64])
def test_split_count_does_not_change_results_beyond_rounding(tiles):
    feeds = decode_feeds(99, B=6, H=32, KV=8, D=128, bs=16, lo=1, hi=3000, nb=1400)
    out, _, _ = run_float_case(feeds, 32, 8, min_tiles_per_warp=tiles)
    want, _, _ = oracle_float(feeds, 32, 8)
    assert np.abs(out - want).max() <= 2e-3


@pytest.mark.parametrize("D", [64, 256])
@pytest.mark.parametrize("window,causal,softcap,sink", [(-1, 1, 0.0, False), (37, 1, 0.0, False),
                                                      (-1, 0, 0.0, True), (-1, 1, 5.0, True)])
def test_decode_head_sizes_and_masks(D, window, causal, softcap, sink):
    H, KV = 16, 4
    feeds = decode_feeds(5 + D, B=5, H=H, KV=KV, D=D, bs=32, lo=1, hi=900, nb=200, dtype=np.float16)
    kw = {}
    if sink:
        feeds["head_sink"] = np.linspace(-1, 1, H).astype(np.float16)
    out, _, _ = run_float_case(feeds, H, KV, attrs=dict(local_window_size=window, is_causal=causal,
                                                       softcap=softcap))
    want, _, _ = oracle_float(feeds, H, KV, local_window_size=window, is_causal=bool(causal),
                              softcap=softcap, head_sink=feeds.get("head_sink"))
    assert np.abs(out - want).max() <= 2e-3


def test_invalid_metadata_host_messages():
    from onnxruntime_ep_b200 import B200Error
    case = next(c for c in FLOAT_CASES if c["name"] == "core_gqa_b3")
    feeds = cases.float_inputs(case)
    bad = dict(feeds, slot_mapping=np.full(feeds["query"].shape[0], -2, np.int32))
    with pytest.raises(B200Error, match="slot_mapping must contain -1 or valid physical cache slots"):
        run_float_case(bad, 4, 2)
    bad = dict(feeds, block_table=np.full_like(feeds["block_table"], 10_000))
    with pytest.raises(B200Error, match="block table contains an invalid physical block"):
        run_float_case(bad, 4, 2)
    cum = feeds["cumulative_sequence_length"].copy()
    cum[1] = cum[2] + 1
    with pytest.raises(B200Error, match="inconsistent cumulative lengths"):
        run_float_case(dict(feeds, cumulative_sequence_length=cum), 4, 2)


def test_invalid_metadata_device_status():
    """Device-resident metadata: kernels never read out of bounds, flag the status word and
    b200_read_status turns it into the reference's message."""
    from onnxruntime_ep_b200 import B200Error
    case = next(c for c in FLOAT_CASES if c["name"] == "core_gqa_b3")
    feeds = cases.float_inputs(case)
    bad = dict(feeds, block_table=np.full_like(feeds["block_table"], 10_000))
    with pytest.raises(B200Error, match="invalid physical block"):
        run_float_case(bad, 4, 2, metadata="device")
    # the status word is cleared by the next good call
    run_float_case(feeds, 4, 2, metadata="device")
