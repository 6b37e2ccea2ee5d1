"""GPU parity of the LATENT cache layout and of head sizes above 256 (generic kernel).

LATENT (attention.rs:3862-3867, :4058-4062, :4210-4212): one kv head, value and value_cache
absent, every value row is the first v_head_size channels of the (rotated) key row, and the
output has v_head_size channels per head.  Checked against the reference test's own case
(golden vectors, test_paged_attention.py:669-764), then at an MLA-like geometry (576-channel
keys, 512-channel values, rotary over the last 64 channels) against the CPU oracle, with the
appended key rows bit-exact.  Head sizes 320 and 512 with the SEPARATE layout run on the same
generic kernel."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import cases  # noqa: E402
from gpu_helpers import to_dev, to_np  # noqa: E402
from onnxruntime_ep_b200 import paged_attention  # noqa: E402
from oracle import paged_ref as ref  # noqa: E402
from oracle import tolerance  # noqa: E402

GOLDEN = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "paged_golden.npz"))


def run_latent(feeds, H, vd, scale, offset=0, rotary=True):
    kc = to_dev(feeds["key_cache"])
    kw = {}
    if rotary:
        kw = dict(cos_cache=to_dev(feeds["cos"]), sin_cache=to_dev(feeds["sin"]), do_rotary=1, rotary_offset=offset)
    out, kc2, _ = paged_attention(
        to_dev(feeds["query"]), to_dev(feeds["key"]), None, kc, None,
        torch.from_numpy(feeds["cumulative_sequence_length"]), torch.from_numpy(feeds["past_seqlens"]),
        torch.from_numpy(feeds["block_table"]), num_heads=H, kv_num_heads=1, scale=scale,
        kv_cache_layout="LATENT", v_head_size=vd, check_status=True, **kw)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), to_np(kc2)


def test_latent_golden_case():
    lat = cases.LATENT
    feeds = cases.latent_inputs()
    out, kc = run_latent(feeds, lat["H"], lat["vd"], lat["scale"], lat["offset"])
    assert out.shape == (lat["nt"], lat["H"] * lat["vd"])
    np.testing.assert_array_equal(kc.view(np.uint16), GOLDEN["latent/key_cache"].view(np.uint16))
    # the reference test's own bound is rtol = atol = 2e-2 on fp16 outputs; the error beyond the
    # fp16 output's rounding is held to 2e-3 here
    assert tolerance.report(out, GOLDEN["latent/output"], bits=11)["max_excess"] <= 2e-3


def mla_case(seed, H=16, d=576, vd=512, rot=64, bs=16, nqs=(1, 1, 20, 1), pasts=(0, 37, 50, 700), dt=ref.BF16):
    rng = np.random.default_rng(seed)
    nqs, pasts = np.asarray(nqs), np.asarray(pasts)
    totals = nqs + pasts
    need = -(-totals // bs)
    nb = int(need.sum()) + 3
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((len(nqs), int(need.max())), np.int32)
    off = 0
    for b in range(len(nqs)):
        bt[b, :need[b]] = perm[off:off + need[b]]
        off += int(need[b])
    nt = int(nqs.sum())
    f = lambda *s: (rng.standard_normal(s, np.float32) * 0.3).astype(dt)
    half = rot // 2
    inv = 1.0 / (10000.0 ** (np.arange(half) / half))
    ang = np.arange(int(totals.max()) + 8)[:, None] * inv[None, :]
    return dict(query=f(nt, H * d), key=f(nt, d), key_cache=f(nb, bs, 1, d),
                cumulative_sequence_length=np.concatenate([[0], np.cumsum(nqs)]).astype(np.int32),
                past_seqlens=pasts.astype(np.int32), block_table=bt,
                cos=np.cos(ang).astype(dt), sin=np.sin(ang).astype(dt))


@pytest.mark.parametrize("rotary", [True, False])
def test_latent_mla_geometry(rotary):
    H, d, vd = 16, 576, 512
    feeds = mla_case(7, H=H, d=d, vd=vd)
    scale = 1.0 / np.sqrt(192.0)
    out, kc = run_latent(feeds, H, vd, scale, offset=vd if rotary else 0, rotary=rotary)
    kw = dict(cos=feeds["cos"], sin=feeds["sin"], rotary_offset=vd) if rotary else {}
    want, wkc, _ = ref.paged_attention(
        feeds["query"], feeds["key"], None, feeds["key_cache"], None, feeds["cumulative_sequence_length"],
        feeds["past_seqlens"], feeds["block_table"], H, 1, scale=scale, latent_v_head=vd, **kw)
    assert out.shape == (feeds["query"].shape[0], H * vd)
    np.testing.assert_array_equal(kc.view(np.uint16), wkc.view(np.uint16))
    rep = tolerance.report(out, want, bits=8)
    assert rep["max_excess"] <= 2e-3, rep


@pytest.mark.parametrize("d", [320, 512])
def test_separate_heads_above_256(d):
    H, KV, bs = 4, 2, 16
    rng = np.random.default_rng(d)
    nqs, pasts = np.array([1, 3, 1]), np.array([100, 20, 333])
    totals = nqs + pasts
    need = -(-totals // bs)
    nb = int(need.sum()) + 2
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((3, int(need.max())), np.int32)
    off = 0
    for b in range(3):
        bt[b, :need[b]] = perm[off:off + need[b]]
        off += int(need[b])
    nt = int(nqs.sum())
    f = lambda *s: (rng.standard_normal(s, np.float32) * 0.3).astype(ref.BF16)
    q, k, v = f(nt, H * d), f(nt, KV * d), f(nt, KV * d)
    kc, vc = f(nb, bs, KV, d), f(nb, bs, KV, d)
    cum = np.concatenate([[0], np.cumsum(nqs)]).astype(np.int32)
    out, kc2, vc2 = paged_attention(to_dev(q), to_dev(k), to_dev(v), to_dev(kc), to_dev(vc), torch.from_numpy(cum),
                                    torch.from_numpy(pasts.astype(np.int32)), torch.from_numpy(bt), num_heads=H,
                                    kv_num_heads=KV, check_status=True)
    torch.cuda.synchronize()
    want, wkc, wvc = ref.paged_attention(q, k, v, kc, vc, cum, pasts.astype(np.int32), bt, H, KV)
    assert tolerance.report(out.float().cpu().numpy(), want, bits=8)["max_excess"] <= 2e-3
    np.testing.assert_array_equal(to_np(kc2).view(np.uint16), wkc.view(np.uint16))
    np.testing.assert_array_equal(to_np(vc2).view(np.uint16), wvc.view(np.uint16))
