"""GPU parity of fp8 e4m3 KV caches with per-(block, kv head) fp32 scales (an extension the
reference does not have, so parity is against the fp32 dequantised recomputation of
oracle/paged_ref.py, max-abs 5e-3 beyond the bf16 output's own rounding): the decode fast path,
the generic kernel, and the fp8 encoding of the appended rows (bit-exact).  Unused slots hold
NaN codes, which must not reach the output."""

import numpy as np
import pytest

from oracle import paged_ref as ref
from oracle import tolerance

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_helpers import to_dev  # noqa: E402
from onnxruntime_ep_b200 import paged_attention  # noqa: E402

NAN_E4M3 = 0x7F


def fp8_case(seed, H, KV, D, nqs, pasts, act=None, bs=16):
    act = act or ref.BF16
    rng = np.random.default_rng(seed)
    nqs, pasts = np.asarray(nqs), np.asarray(pasts)
    B = len(nqs)
    totals = nqs + pasts
    need = -(-totals // bs)
    nb = int(need.sum()) + 4
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((B, int(need.max())), np.int32)
    off = 0
    for b in range(B):
        bt[b, :need[b]] = perm[off:off + need[b]]
        off += int(need[b])
    ks = rng.uniform(0.01, 0.1, (nb, KV)).astype(np.float32)
    vs = rng.uniform(0.01, 0.1, (nb, KV)).astype(np.float32)
    kc = ref.fp8_encode(rng.standard_normal((nb, bs, KV, D)), ks[:, None, :, None])
    vc = ref.fp8_encode(rng.standard_normal((nb, bs, KV, D)), vs[:, None, :, None])
    # slots past each sequence's end hold NaN codes
    kcb, vcb = kc.view(np.uint8), vc.view(np.uint8)
    for b in range(B):
        for pos in range(int(totals[b]), int(need[b]) * bs):
            blk, o = bt[b, pos // bs], pos % bs
            kcb[blk, o] = NAN_E4M3
            vcb[blk, o] = NAN_E4M3
    nt = int(nqs.sum())
    f = lambda *s: (rng.standard_normal(s, np.float32) * 0.5).astype(act)
    return dict(query=f(nt, H * D), key=f(nt, KV * D), value=f(nt, KV * D), key_cache=kc, value_cache=vc,
                cum=np.concatenate([[0], np.cumsum(nqs)]).astype(np.int32), past=pasts.astype(np.int32), bt=bt,
                ks=ks, vs=vs)


def run(c, H, KV, force_generic=False):
    q, k, v = (to_dev(c[n]) for n in ("query", "key", "value"))
    kc = torch.from_numpy(c["key_cache"].view(np.uint8)).cuda().view(torch.float8_e4m3fn)
    vc = torch.from_numpy(c["value_cache"].view(np.uint8)).cuda().view(torch.float8_e4m3fn)
    out, kc2, vc2 = paged_attention(
        q, k, v, kc, vc, torch.from_numpy(c["cum"]), torch.from_numpy(c["past"]), torch.from_numpy(c["bt"]),
        num_heads=H, kv_num_heads=KV, k_scale=torch.from_numpy(c["ks"]).cuda(),
        v_scale=torch.from_numpy(c["vs"]).cuda(), force_generic=force_generic, check_status=True)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), kc2.view(torch.uint8).cpu().numpy(), vc2.view(torch.uint8).cpu().numpy()


def oracle(c, H, KV):
    return ref.paged_attention(c["query"], c["key"], c["value"], c["key_cache"], c["value_cache"], c["cum"],
                               c["past"], c["bt"], H, KV, fp8_scales=(c["ks"], c["vs"]))


def check(out, want, bf16=True):
    # north-star fp8-KV tolerance 5e-3 on the error beyond the output's own rounding (half an ulp)
    assert np.isfinite(out).all()
    rep = tolerance.report(out, want, bits=8 if bf16 else 11)
    assert rep["max_excess"] <= 5e-3, rep


@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("generic", [False, True])
def test_fp8_decode_and_prefill_match_dequantised_recomputation(D, generic):
    H, KV = 16, 2
    c = fp8_case(7 + D, H, KV, D, nqs=[1, 1, 1, 1, 1, 30], pasts=[100, 1500, 2999, 17, 640, 200])
    out, kc, vc = run(c, H, KV, force_generic=generic)
    want, wkc, wvc = oracle(c, H, KV)
    check(out, want)
    np.testing.assert_array_equal(kc, wkc.view(np.uint8))
    np.testing.assert_array_equal(vc, wvc.view(np.uint8))


def test_fp8_config5_geometry():
    """BASELINE config 5 per GPU: one kv head, 8 q heads, d128, long contexts (shortened)."""
    H, KV = 8, 1
    rng = np.random.default_rng(5)
    pasts = rng.integers(4096, 12000, size=12)
    c = fp8_case(5, H, KV, 128, nqs=[1] * 12, pasts=list(pasts))
    out, kc, vc = run(c, H, KV)
    want, _, _ = oracle(c, H, KV)
    check(out, want)


def test_fp8_fp16_activations():
    H, KV = 8, 2
    c = fp8_case(11, H, KV, 128, nqs=[1, 1, 2], pasts=[333, 64, 900], act=np.float16)
    out, _, _ = run(c, H, KV)
    want, _, _ = oracle(c, H, KV)
    check(out, want, bf16=False)


def test_bf16_cache_nan_in_unused_slots_does_not_reach_output():
    """16-bit caches: slots past a sequence's end hold NaN; decode must stay finite and exact."""
    from gpu_helpers import run_float_case

    H, KV, D, bs = 16, 2, 128, 16
    rng = np.random.default_rng(3)
    nqs, pasts = np.array([1, 1, 1]), np.array([70, 300, 1000])
    totals = nqs + pasts
    need = -(-totals // bs)
    nb = int(need.sum()) + 2
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((3, int(need.max())), np.int32)
    off = 0
    for b in range(3):
        bt[b, :need[b]] = perm[off:off + need[b]]
        off += int(need[b])
    f = lambda *s: (rng.standard_normal(s, np.float32) * 0.5).astype(ref.BF16)
    kc, vc = f(nb, bs, KV, D), f(nb, bs, KV, D)
    for b in range(3):
        for pos in range(int(totals[b]), int(need[b]) * bs):
            kc[bt[b, pos // bs], pos % bs] = np.nan
            vc[bt[b, pos // bs], pos % bs] = np.nan
    nt = int(nqs.sum())
    feeds = dict(query=f(nt, H * D), key=f(nt, KV * D), value=f(nt, KV * D), key_cache=kc, value_cache=vc,
                 cumulative_sequence_length=np.concatenate([[0], np.cumsum(nqs)]).astype(np.int32),
                 past_seqlens=pasts.astype(np.int32), block_table=bt)
    out, _, _ = run_float_case(feeds, H, KV)
    want, _, _ = ref.paged_attention(feeds["query"], feeds["key"], feeds["value"], kc, vc,
                                     feeds["cumulative_sequence_length"], feeds["past_seqlens"], bt, H, KV)
    assert np.isfinite(out).all()
    rep = tolerance.report(out, want, bits=8)
    assert rep["max_excess"] <= 2e-3, rep
