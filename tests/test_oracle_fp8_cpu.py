"""The C oracle's fp8 e4m3 cache path against the numpy restatement (CPU only).

fp8 KV caches are an extension the reference does not have, so there are no golden vectors:
the C encoder is pinned against ml_dtypes' float8_e4m3fn conversion (round to nearest even)
on every code boundary, and the C attention against ``oracle/paged_ref.py``'s fp32 dequantised
recomputation on the same inputs.
"""

import numpy as np
import pytest

from oracle import cpu_oracle
from oracle import paged_ref as ref

ml_dtypes = pytest.importorskip("ml_dtypes")


def test_e4m3_encoder_matches_ml_dtypes_on_every_boundary():
    codes = np.arange(256, dtype=np.uint8)
    vals = codes.view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    fin = np.sort(np.unique(np.abs(vals[np.isfinite(vals)])))
    mids = (fin[1:] + fin[:-1]) / 2  # ties: round half to even
    x = np.concatenate([fin, mids, np.nextafter(mids, np.float32(0)), np.nextafter(mids, np.float32(1e3)),
                        [448, 460, 464, 470, 1e6, 1e-12, 0.0]]).astype(np.float32)
    x = np.concatenate([x, -x, np.random.default_rng(0).standard_normal(50000).astype(np.float32) * 100])
    want = np.clip(x, -448, 448).astype(ml_dtypes.float8_e4m3fn).view(np.uint8)
    np.testing.assert_array_equal(cpu_oracle.e4m3_encode(x), want)


@pytest.mark.parametrize("causal,window,softcap,sink", [(1, -1, 0.0, False), (1, 40, 0.0, True),
                                                        (0, -1, 3.0, False)])
def test_c_fp8_attention_matches_numpy_restatement(causal, window, softcap, sink):
    rng = np.random.default_rng(5)
    H, KV, D, bs = 16, 2, 128, 16
    nqs = np.array([1, 1, 7, 1])
    pasts = np.array([300, 37, 120, 0])
    totals = nqs + pasts
    need = -(-totals // bs)
    nb = int(need.sum()) + 3
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((len(nqs), int(need.max())), np.int32)
    off = 0
    for b in range(len(nqs)):
        bt[b, :need[b]] = perm[off:off + need[b]]
        off += int(need[b])
    ks = rng.uniform(0.01, 0.1, (nb, KV)).astype(np.float32)
    vs = rng.uniform(0.01, 0.1, (nb, KV)).astype(np.float32)
    kc = ref.fp8_encode(rng.standard_normal((nb, bs, KV, D)), ks[:, None, :, None])
    vc = ref.fp8_encode(rng.standard_normal((nb, bs, KV, D)), vs[:, None, :, None])
    nt = int(nqs.sum())
    f = lambda *s: rng.standard_normal(s, np.float32).astype(ref.BF16)
    q, k, v = f(nt, H * D), f(nt, KV * D), f(nt, KV * D)
    cum = np.concatenate([[0], np.cumsum(nqs)]).astype(np.int32)
    hs = rng.standard_normal(H).astype(np.float32) if sink else None
    kw = dict(is_causal=bool(causal), local_window_size=window, softcap=softcap, head_sink=hs)
    want, wkc, wvc = ref.paged_attention(q, k, v, kc, vc, cum, pasts.astype(np.int32), bt, H, KV,
                                         fp8_scales=(ks, vs), **kw)
    kc2, vc2 = kc.copy(), vc.copy()
    got = cpu_oracle.paged_attention_fp8(q, k, v, kc2, vc2, ks, vs, cum, pasts.astype(np.int32), bt, H, KV,
                                         threads=2, **kw)
    np.testing.assert_array_equal(kc2.view(np.uint8), wkc.view(np.uint8))
    np.testing.assert_array_equal(vc2.view(np.uint8), wvc.view(np.uint8))
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
