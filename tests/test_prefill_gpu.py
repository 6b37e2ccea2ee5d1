"""GPU parity of the tcgen05 prefill kernel (head size 128, fp16/bf16, block size multiple of 16)
against the CPU oracle and against the generic kernel, on ragged batches that mix prefill
chunks (with and without cached prefix) and decode rows."""

import numpy as np
import pytest

from oracle import paged_ref as ref
from oracle import tolerance

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_helpers import run_float_case  # noqa: E402


def mixed_feeds(seed, H, KV, nqs, pasts, D=128, bs=16, dtype=None, scale=0.5):
    dtype = dtype or ref.BF16
    rng = np.random.default_rng(seed)
    nqs, pasts = np.asarray(nqs), np.asarray(pasts)
    B = len(nqs)
    totals = nqs + pasts
    need = -(-totals // bs)
    maxb = int(need.max())
    nb = int(need.sum()) + 8
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((B, maxb), np.int32)
    off = 0
    for b in range(B):
        bt[b, :need[b]] = perm[off:off + need[b]]
        off += int(need[b])
    nt = int(nqs.sum())
    f = lambda *s: (rng.standard_normal(s, np.float32) * scale).astype(dtype)
    return {
        "query": f(nt, H * D), "key": f(nt, KV * D), "value": f(nt, KV * D),
        "key_cache": f(nb, bs, KV, D), "value_cache": f(nb, bs, KV, D),
        "cumulative_sequence_length": np.concatenate([[0], np.cumsum(nqs)]).astype(np.int32),
        "past_seqlens": pasts.astype(np.int32), "block_table": bt,
    }


def oracle(feeds, H, KV, **kw):
    return ref.paged_attention(
        feeds["query"], feeds["key"], feeds["value"], feeds["key_cache"], feeds["value_cache"],
        feeds["cumulative_sequence_length"], feeds["past_seqlens"], feeds["block_table"], H, KV,
        slot_mapping=feeds.get("slot_mapping"), **kw)


def check(out, want, dtype_is_bf16=True):
    # fp32 recomputation tolerance 2e-3 on the error beyond the 16-bit output's own rounding
    # (half an ulp of the output format)
    rep = tolerance.report(out, want, bits=8 if dtype_is_bf16 else 11)
    assert rep["max_excess"] <= 2e-3, rep


@pytest.mark.parametrize("H,KV", [(32, 4), (64, 8), (16, 16), (32, 2)])
@pytest.mark.parametrize("causal", [1, 0])
def test_prefill_mixed_batch_matches_oracle(H, KV, causal):
    nqs = [300, 200, 1, 129, 16]
    pasts = [0, 150, 500, 0, 37]
    feeds = mixed_feeds(3 + H + KV + causal, H, KV, nqs, pasts)
    out, kc, vc = run_float_case(feeds, H, KV, attrs=dict(is_causal=causal))
    want, wkc, wvc = oracle(feeds, H, KV, is_causal=bool(causal))
    check(out, want)
    np.testing.assert_array_equal(kc.view(np.uint16), wkc.view(np.uint16))
    np.testing.assert_array_equal(vc.view(np.uint16), wvc.view(np.uint16))


@pytest.mark.parametrize("window,softcap,sink", [(64, 0.0, False), (-1, 8.0, True), (200, 0.0, True)])
def test_prefill_window_softcap_sink(window, softcap, sink):
    H, KV = 32, 4
    feeds = mixed_feeds(17, H, KV, [260, 90], [0, 300], dtype=np.float16)
    if sink:
        feeds["head_sink"] = np.linspace(-1, 1, H).astype(np.float16)
    out, _, _ = run_float_case(feeds, H, KV, attrs=dict(local_window_size=window, softcap=softcap))
    want, _, _ = oracle(feeds, H, KV, local_window_size=window, softcap=softcap,
                        head_sink=feeds.get("head_sink"))
    check(out, want, dtype_is_bf16=False)


def test_prefill_fast_and_generic_agree():
    H, KV = 32, 8
    feeds = mixed_feeds(23, H, KV, [512, 77], [0, 1000])
    fast, _, _ = run_float_case(feeds, H, KV)
    slow, _, _ = run_float_case(feeds, H, KV, force_generic=True)
    assert np.abs(fast - slow).max() <= 4e-3


@pytest.mark.parametrize("metadata", ["host", "device"])
def test_prefill_with_remapped_slots_uses_reference_semantics(metadata):
    """slot_mapping that sends new rows elsewhere (or skips them) routes the sequence to the
    generic kernel, which reads the new rows directly as the reference does."""
    H, KV = 32, 4
    feeds = mixed_feeds(31, H, KV, [150, 40], [0, 64])
    nt = 190
    nb = feeds["key_cache"].shape[0]
    rng = np.random.default_rng(5)
    slots = rng.permutation(nb * 16)[:nt].astype(np.int32)
    slots[::7] = -1
    feeds["slot_mapping"] = slots
    out, kc, vc = run_float_case(feeds, H, KV, metadata=metadata)
    want, wkc, wvc = oracle(feeds, H, KV)
    check(out, want)
    np.testing.assert_array_equal(kc.view(np.uint16), wkc.view(np.uint16))
