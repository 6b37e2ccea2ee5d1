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
    want, _, _ = oracle(feeds, H, KV)
    check(fast, want)
    check(slow, want)
    # each within 2e-3 of the oracle beyond rounding: a value near a bf16 boundary may round to
    # neighbouring outputs, one output ulp apart
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(slow), 2.0 ** -126))) - 7)
    assert np.all(np.abs(fast - slow) <= 4e-3 + ulp)


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


def _unused_slots(feeds):
    """(block, slot) of every cache slot past a sequence's last key in its last block."""
    bs = feeds["key_cache"].shape[1]
    totals = np.diff(feeds["cumulative_sequence_length"]) + feeds["past_seqlens"]
    slots = []
    for b, n in enumerate(totals):
        if n % bs:
            blk = feeds["block_table"][b, (n - 1) // bs]
            slots += [(blk, s) for s in range(n % bs, bs)]
    return slots


@pytest.mark.parametrize("dtype,pasts", [(ref.BF16, [0, 150, 37]), (np.float16, [0, 150, 37]), (ref.BF16, [0, 0, 0])])
def test_prefill_ignores_unused_slots(dtype, pasts):
    """NaN in the slots past each sequence's last key (the tail of its last page): the output
    is the oracle's, which reads only the sequence's keys (as the reference's gather does).
    Without cached prefixes (pasts 0) the bf16 prefill reads V from the call's fp16 copy."""
    H, KV = 32, 4
    feeds = mixed_feeds(41, H, KV, [300, 200, 129], pasts, dtype=dtype)
    nan = np.array(np.nan, np.float32).astype(dtype)
    unused = _unused_slots(feeds)
    assert len(unused) > 0
    for blk, s in unused:
        feeds["key_cache"][blk, s] = nan
        feeds["value_cache"][blk, s] = nan
    out, kc, vc = run_float_case(feeds, H, KV)
    want, wkc, wvc = oracle(feeds, H, KV)
    assert np.isfinite(out).all()
    check(out, want, dtype_is_bf16=dtype is ref.BF16)
    np.testing.assert_array_equal(kc.view(np.uint16), wkc.view(np.uint16))
    np.testing.assert_array_equal(vc.view(np.uint16), wvc.view(np.uint16))


@pytest.mark.parametrize("pasts", [[0, 150], [0, 20]])
def test_prefill_bf16_values_beyond_fp16(pasts):
    """bf16 V values beyond the fp16 range (P . V stays in bf16, P as hi + lo halves): finite
    outputs, the oracle's result within the precision of a 16-bit-significand P.  With
    pasts [0, 20] the value in the cache sits in a cached prefix; the new-row value of sequence 0
    alone would send a no-prefix call from its fp16 V copy to the bf16 fallback launch."""
    H, KV, D = 32, 4, 128
    feeds = mixed_feeds(43, H, KV, [300, 200], pasts)
    big = np.array([7.0e4, -2.5e5], np.float32).astype(ref.BF16)
    feeds["value"][5, :D] = big[0]                      # a new row of sequence 0, kv head 0
    blk = feeds["block_table"][1, 20 // 16]              # a cached row of sequence 1, kv head 2
    feeds["value_cache"][blk, 20 % 16, 2] = big[1]
    out, kc, vc = run_float_case(feeds, H, KV)
    want, wkc, wvc = oracle(feeds, H, KV)
    assert np.isfinite(out).all() and np.abs(want).max() > 100.0
    # On a wide tile P carries about 16 significant bits (hi + lo bf16 halves), so an output of
    # magnitude X (here up to ~1e4) may differ from the fp32 oracle by ~2^-16 X besides rounding.
    excess = tolerance.excess(out, want, 8) - 2.0 ** -15 * np.abs(want)
    assert excess.max() <= 2e-3, tolerance.report(out, want)
    np.testing.assert_array_equal(vc.view(np.uint16), wvc.view(np.uint16))


@pytest.mark.parametrize("H,KV", [(32, 4), (64, 8), (16, 16)])
def test_prefill_bf16_without_prefix_reads_fp16_v_copy(H, KV):
    """bf16 prefill sequences without a cached prefix (decode rows may have one): P . V runs on
    an fp16 copy of the call's new V rows with one fp16 P; the output is the oracle's within the
    usual bound, caches bit-exact."""
    nqs, pasts = [300, 200, 1, 129, 16], [0, 0, 500, 0, 0]
    feeds = mixed_feeds(47 + H, H, KV, nqs, pasts)
    out, kc, vc = run_float_case(feeds, H, KV)
    want, wkc, wvc = oracle(feeds, H, KV)
    check(out, want)
    np.testing.assert_array_equal(kc.view(np.uint16), wkc.view(np.uint16))
    np.testing.assert_array_equal(vc.view(np.uint16), wvc.view(np.uint16))


def test_prefill_bf16_fp16_copy_out_of_range_falls_back():
    """A new V value beyond the fp16 range in a no-prefix call: the fp16-copy launch steps aside
    and the bf16 launch computes the call, with the oracle's result."""
    H, KV, D = 32, 4, 128
    feeds = mixed_feeds(53, H, KV, [300, 200], [0, 0])
    feeds["value"][310, D:2 * D] = np.array(9.0e4, np.float32).astype(ref.BF16)  # sequence 1, kv head 1
    out, kc, vc = run_float_case(feeds, H, KV)
    want, wkc, wvc = oracle(feeds, H, KV)
    assert np.isfinite(out).all() and np.abs(want).max() > 100.0
    excess = tolerance.excess(out, want, 8) - 2.0 ** -15 * np.abs(want)
    assert excess.max() <= 2e-3, tolerance.report(out, want)
    np.testing.assert_array_equal(vc.view(np.uint16), wvc.view(np.uint16))


@pytest.mark.parametrize("dtype,pasts", [(ref.BF16, [0, 0, 500, 0]), (ref.BF16, [0, 150, 500, 37]),
                                         (np.float16, [0, 0, 500, 0])])
def test_prefill_packed_qkv(dtype, pasts):
    """Packed QKV (key and value inside the query rows, attention.rs:3877-3890): the prefill,
    the fp16 V copy and decode read K and V at the packed row stride; output and caches are the
    oracle's."""
    from onnxruntime_ep_b200 import paged_attention
    from gpu_helpers import to_dev, to_np

    H, KV = 32, 4
    feeds = mixed_feeds(59, H, KV, [300, 200, 1, 129], pasts, dtype=dtype)
    packed = np.concatenate([feeds["query"], feeds["key"], feeds["value"]], axis=1)
    meta = {n: torch.from_numpy(feeds[n]) for n in ("cumulative_sequence_length", "past_seqlens", "block_table")}
    out, kc, vc = paged_attention(
        to_dev(packed), None, None, to_dev(feeds["key_cache"]), to_dev(feeds["value_cache"]),
        meta["cumulative_sequence_length"], meta["past_seqlens"], meta["block_table"],
        num_heads=H, kv_num_heads=KV, check_status=True)
    torch.cuda.synchronize()
    want, wkc, wvc = ref.paged_attention(
        packed, None, None, feeds["key_cache"], feeds["value_cache"],
        feeds["cumulative_sequence_length"], feeds["past_seqlens"], feeds["block_table"], H, KV)
    check(out.float().cpu().numpy(), want, dtype_is_bf16=dtype is ref.BF16)
    np.testing.assert_array_equal(to_np(kc).view(np.uint16), wkc.view(np.uint16))
    np.testing.assert_array_equal(to_np(vc).view(np.uint16), wvc.view(np.uint16))
