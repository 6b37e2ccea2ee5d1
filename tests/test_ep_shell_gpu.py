"""The ORT plugin-EP glue (csrc/ep_shell.cpp) running Compute on the GPU through the fake ORT host.

Each case builds the node as ORT would see it, claims and compiles it through the glue, binds the
tensors in a kernel context (device memory, or host memory that the glue stages) and checks:
  - PagedAttention: attention against the CPU oracle (error beyond the bf16 output's rounding
    <= 2e-3), the caches updated in place bit-exactly, cache outputs that are not aliased to
    their inputs receiving the updated caches, output shapes as ORT would be asked for them;
  - GroupQueryAttention: output and present caches against the reference-restating oracle at the
    config-1 shapes (fp32, present bit-exact), with lengths read on the host;
  - invalid metadata surfacing as ORT_EP_FAIL with the reference's message;
  - the device allocator and the data transfer.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import ort_host as oh  # noqa: E402
from gpu_helpers import to_dev, to_np  # noqa: E402
from oracle import cpu_oracle, gqa_ref, tolerance  # noqa: E402
from oracle import paged_ref as ref  # noqa: E402

H, KV, D, BS, NB, B, MAXB = 8, 2, 128, 16, 64, 4, 16


@pytest.fixture
def ep():
    h = oh.Host()
    assert h.devices([(oh.GPU, oh.NVIDIA)])[:2] == (0, 1)
    assert h.create_ep() == 0, oh.last_error()
    yield h
    h.close()


def _paged_feeds(seed=0):
    rng = np.random.default_rng(seed)
    lens = np.array([1, 37, 200, 130], np.int32)
    nq = np.array([1, 1, 5, 1], np.int32)
    cum = np.concatenate([[0], np.cumsum(nq)]).astype(np.int32)
    past = (lens - nq).astype(np.int32)
    bt = rng.permutation(NB).astype(np.int32).reshape(B, MAXB)
    nt = int(cum[-1])
    f = lambda *s: (rng.standard_normal(s, np.float32) * 0.3).astype(ref.BF16)
    return dict(query=f(nt, H * D), key=f(nt, KV * D), value=f(nt, KV * D), key_cache=f(NB, BS, KV, D),
                value_cache=f(NB, BS, KV, D), cum=cum, past=past, bt=bt)


def _paged_graph(outputs):
    g = oh.Graph()
    oh.paged_node(g, "pa", H=H, KV=KV, d=D, dt=oh.BF16, nb=NB, bs=BS, B=B, maxb=MAXB, outputs=outputs)
    return g


def _bind(ctx, name, arr, dtype):
    """A numpy array (host memory) or a torch CUDA tensor into the kernel context."""
    if isinstance(arr, torch.Tensor):
        ctx.input(name, dtype, tuple(arr.shape), arr.data_ptr(), arr.numel() * arr.element_size())
    else:
        ctx.input(name, dtype, arr.shape, arr.ctypes.data, arr.nbytes)


def _run_paged(ep, feeds, *, on_device, outputs=1, alias_cache_out=False, reverse=False):
    g = _paged_graph(outputs)
    ctx = oh.KernelContext()
    try:
        rc, claimed, _ = ep.capability(g)
        assert rc == 0 and claimed == [0], ep.report()
        idx = ep.compile(g, 0, reverse=reverse)
        assert idx >= 0, oh.last_error()
        conv = (lambda a: to_dev(a)) if on_device else (lambda a: np.ascontiguousarray(a).copy())
        t = {k: conv(v) for k, v in feeds.items()}
        for name, key, dt in (("query", "query", oh.BF16), ("key", "key", oh.BF16), ("value", "value", oh.BF16),
                              ("key_cache", "key_cache", oh.BF16), ("value_cache", "value_cache", oh.BF16),
                              ("cum", "cum", oh.I32), ("past", "past", oh.I32), ("block_table", "bt", oh.I32)):
            _bind(ctx, f"pa.{name}", t[key], dt)
        nt = feeds["query"].shape[0]
        out = torch.empty((nt, H * D), dtype=torch.bfloat16, device="cuda") if on_device else \
            np.zeros((nt, H * D), ref.BF16)
        ptr = out.data_ptr() if on_device else out.ctypes.data
        ctx.output("pa.out", oh.BF16, (nt, H * D), ptr, nt * H * D * 2)
        cache_outs = []
        for j, name in ((1, "key_cache"), (2, "value_cache")):
            if outputs > j:
                src = t[name]
                if alias_cache_out:
                    dst = src
                else:
                    dst = torch.empty_like(src) if on_device else np.zeros_like(src)
                p = dst.data_ptr() if on_device else dst.ctypes.data
                ctx.output(f"pa.{name}_out", oh.BF16, (NB, BS, KV, D), p, NB * BS * KV * D * 2)
                cache_outs.append(dst)
        rc = ep.compute(idx, ctx)
        assert rc == 0, oh.last_error()
        assert ctx.requested("pa.out") == (nt, H * D)
        host = (lambda a: to_np(a)) if on_device else (lambda a: a)
        return host(out), host(t["key_cache"]), host(t["value_cache"]), [host(c) for c in cache_outs]
    finally:
        ctx.close()
        g.close()


def _expected(feeds):
    kc, vc = feeds["key_cache"].copy(), feeds["value_cache"].copy()
    want = cpu_oracle.paged_attention(feeds["query"], feeds["key"], feeds["value"], kc, vc, feeds["cum"],
                                      feeds["past"], feeds["bt"], H, KV, fp32_out=True)
    return want, kc, vc


def _same_bits(a, b):
    return np.array_equal(np.asarray(a).view(np.uint16), np.asarray(b).view(np.uint16))


@pytest.mark.parametrize("on_device", [True, False], ids=["device_tensors", "host_tensors"])
def test_paged_compute_matches_the_oracle(ep, on_device):
    feeds = _paged_feeds(1)
    want, wkc, wvc = _expected(feeds)
    out, kc, vc, _ = _run_paged(ep, feeds, on_device=on_device)
    rep = tolerance.report(out.astype(np.float32), want, bits=8)
    assert rep["max_excess"] <= 2e-3, rep
    # the caches are updated in place in the input buffers, bit-exactly
    assert _same_bits(kc, wkc) and _same_bits(vc, wvc)


@pytest.mark.parametrize("alias", [False, True], ids=["separate_cache_outputs", "aliased_cache_outputs"])
def test_paged_cache_outputs(ep, alias):
    feeds = _paged_feeds(2)
    want, wkc, wvc = _expected(feeds)
    out, kc, vc, (kco, vco) = _run_paged(ep, feeds, on_device=True, outputs=3, alias_cache_out=alias)
    assert tolerance.report(out.astype(np.float32), want, bits=8)["max_excess"] <= 2e-3
    assert _same_bits(kco, wkc) and _same_bits(vco, wvc)
    assert _same_bits(kc, wkc) and _same_bits(vc, wvc)


def test_fused_input_order_does_not_matter(ep):
    feeds = _paged_feeds(3)
    a = _run_paged(ep, feeds, on_device=True)[0]
    b = _run_paged(ep, feeds, on_device=True, reverse=True)[0]
    assert _same_bits(a, b)


def test_invalid_block_id_is_an_ep_failure(ep):
    feeds = _paged_feeds(4)
    feeds["bt"][2, 3] = NB + 7  # a block of sequence 2's context outside the pool
    with pytest.raises(AssertionError):
        _run_paged(ep, feeds, on_device=True)
    code, msg = oh.last_error()
    assert code == oh.ORT_EP_FAIL and "invalid physical block" in msg


@pytest.mark.parametrize("seqlens_on_device", [True, False])
def test_gqa_compute_config1_shapes(ep, seqlens_on_device):
    Hg, KVg, Dg, cap = 32, 8, 128, 2048
    rng = np.random.default_rng(5)
    qn = rng.standard_normal((1, 1, Hg * Dg), np.float32)
    kn = rng.standard_normal((1, 1, KVg * Dg), np.float32)
    vn = rng.standard_normal((1, 1, KVg * Dg), np.float32)
    pkn = rng.standard_normal((1, KVg, cap, Dg), np.float32)
    pvn = rng.standard_normal((1, KVg, cap, Dg), np.float32)
    lens = np.array([cap - 1], np.int32)  # one new token after cap - 1 cached ones
    total = np.array([cap], np.int32)
    want, wk, wv = gqa_ref.group_query_attention(qn, kn, vn, pkn, pvn, lens, cap, num_heads=Hg, kv_num_heads=KVg)
    g = oh.Graph()
    ctx = oh.KernelContext()
    try:
        oh.gqa_node(g, "gqa", H=Hg, KV=KVg, d=Dg, dt=oh.F32, B=1, S=1, cap=cap)
        rc, claimed, _ = ep.capability(g)
        assert rc == 0 and claimed == [0], ep.report()
        idx = ep.compile(g, 0)
        assert idx >= 0, oh.last_error()
        dev = {k: to_dev(v) for k, v in dict(query=qn, key=kn, value=vn, past_key=pkn, past_value=pvn).items()}
        for k, v in dev.items():
            _bind(ctx, f"gqa.{k}", v, oh.F32)
        meta = dict(seqlens_k=lens.copy(), total=total.copy())
        if seqlens_on_device:
            meta = {k: to_dev(v) for k, v in meta.items()}  # kept alive until Compute has run
        for k, v in meta.items():
            _bind(ctx, f"gqa.{k}", v, oh.I32)
        out = torch.empty((1, 1, Hg * Dg), device="cuda")
        pk = torch.empty((1, KVg, cap, Dg), device="cuda")
        pv = torch.empty_like(pk)
        ctx.output("gqa.out", oh.F32, (1, 1, Hg * Dg), out.data_ptr(), out.numel() * 4)
        ctx.output("gqa.present_key", oh.F32, (1, KVg, cap, Dg), pk.data_ptr(), pk.numel() * 4)
        ctx.output("gqa.present_value", oh.F32, (1, KVg, cap, Dg), pv.data_ptr(), pv.numel() * 4)
        rc = ep.compute(idx, ctx)
        assert rc == 0, oh.last_error()
        assert ctx.requested("gqa.present_key") == (1, KVg, cap, Dg)
        got = out.cpu().numpy()
        assert float(np.abs(got - want).max()) <= 2e-5 + 2e-5 * float(np.abs(want).max())
        assert np.array_equal(pk.cpu().numpy(), wk) and np.array_equal(pv.cpu().numpy(), wv)
    finally:
        ctx.close()
        g.close()


def test_allocator_hands_out_device_memory(ep):
    from onnxruntime_ep_b200._capi import LIB

    assert ep.allocator("B200") == 1
    p = ep.alloc(1 << 20)
    assert p
    flag = ctypes.c_int32()
    assert LIB.b200_ep_is_device_pointer(ctypes.c_void_p(p), ctypes.byref(flag)) == 0 and flag.value == 1
    ep.free(p)


def test_data_transfer_round_trip(ep):
    assert ep.transfer() == 0
    a = np.arange(4096, dtype=np.float32)
    d = torch.empty(4096, device="cuda")
    back = np.zeros_like(a)
    assert ep.copy(oh.F32, (4096,), a.ctypes.data, a.nbytes, (4096,), d.data_ptr(), a.nbytes) == 0
    torch.cuda.synchronize()
    assert np.array_equal(d.cpu().numpy(), a)
    d.mul_(2)
    torch.cuda.synchronize()
    assert ep.copy(oh.F32, (4096,), d.data_ptr(), a.nbytes, (4096,), back.ctypes.data, a.nbytes) == 0
    assert np.array_equal(back, 2 * a)


def test_latent_node_through_the_glue(ep):
    """The reference's LATENT case (test_paged_attention.py:669-764) as ORT would hand it over:
    value / value_cache absent, a key_cache_out output, output [nt, H * v_head_size]."""
    import cases

    golden = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden",
                                                "paged_golden.npz"))
    lat = cases.LATENT
    feeds = cases.latent_inputs()
    H, d, vd, nt = lat["H"], lat["d"], lat["vd"], lat["nt"]
    g = oh.Graph()
    ctx = oh.KernelContext()
    try:
        n = g.node("PagedAttention", "lat")
        n.input("lat.q", oh.F16, (-1, H * d)).input("lat.k", oh.F16, (-1, d)).input(None)
        n.input("lat.kc", oh.F16, feeds["key_cache"].shape).input(None)
        n.input("lat.cum", oh.I32, (2,)).input("lat.past", oh.I32, (1,)).input("lat.bt", oh.I32, (1, 3))
        n.input("lat.cos", oh.F16, feeds["cos"].shape).input("lat.sin", oh.F16, feeds["sin"].shape)
        n.output("lat.out", oh.F16, (-1, H * vd)).output("lat.kc_out", oh.F16, feeds["key_cache"].shape)
        for k, v in dict(num_heads=H, kv_num_heads=1, v_head_size=vd, kv_cache_layout="LATENT", do_rotary=1,
                         rotary_offset=lat["offset"], scale=float(lat["scale"])).items():
            n.attr(k, v)
        rc, claimed, _ = ep.capability(g)
        assert rc == 0 and claimed == [0], ep.report()
        idx = ep.compile(g, 0)
        assert idx >= 0, oh.last_error()
        dev = {k: to_dev(v) for k, v in feeds.items()}
        for name, key, dt in (("q", "query", oh.F16), ("k", "key", oh.F16), ("kc", "key_cache", oh.F16),
                              ("cum", "cumulative_sequence_length", oh.I32), ("past", "past_seqlens", oh.I32),
                              ("bt", "block_table", oh.I32), ("cos", "cos", oh.F16), ("sin", "sin", oh.F16)):
            _bind(ctx, f"lat.{name}", dev[key], dt)
        out = torch.empty((nt, H * vd), dtype=torch.float16, device="cuda")
        kco = torch.empty_like(dev["key_cache"])
        ctx.output("lat.out", oh.F16, (nt, H * vd), out.data_ptr(), out.numel() * 2)
        ctx.output("lat.kc_out", oh.F16, tuple(kco.shape), kco.data_ptr(), kco.numel() * 2)
        rc = ep.compute(idx, ctx)
        assert rc == 0, oh.last_error()
        assert ctx.requested("lat.out") == (nt, H * vd)
        want_cache = golden["latent/key_cache"].view(np.uint16)
        assert np.array_equal(kco.cpu().numpy().view(np.uint16), want_cache)
        assert np.array_equal(dev["key_cache"].cpu().numpy().view(np.uint16), want_cache)
        rep = tolerance.report(out.float().cpu().numpy(), golden["latent/output"], bits=11)
        assert rep["max_excess"] <= 2e-3, rep
    finally:
        ctx.close()
        g.close()


def test_sliding_gqa_node_through_the_glue(ep):
    """A sliding_window_cache GroupQueryAttention node: present is requested at the past's
    capacity and holds the resident rows (attention.rs:1139-1379); lengths past the capacity."""
    Hg, KVg, Dg, cap, window = 8, 2, 64, 64, 32
    rng = np.random.default_rng(17)
    lens = np.array([199, 49], np.int32)
    total = np.array([200], np.int32)
    qn = rng.standard_normal((2, 1, Hg * Dg), np.float32)
    kn = rng.standard_normal((2, 1, KVg * Dg), np.float32)
    vn = rng.standard_normal((2, 1, KVg * Dg), np.float32)
    pkn = rng.standard_normal((2, KVg, cap, Dg), np.float32)
    pvn = rng.standard_normal((2, KVg, cap, Dg), np.float32)
    want, wk, wv = gqa_ref.group_query_attention(qn, kn, vn, pkn, pvn, lens, total, num_heads=Hg, kv_num_heads=KVg,
                                                 window=window, sliding=True)
    g = oh.Graph()
    ctx = oh.KernelContext()
    try:
        oh.gqa_node(g, "sw", H=Hg, KV=KVg, d=Dg, dt=oh.F32, B=2, S=1, cap=cap,
                    attrs=dict(sliding_window_cache=1, local_window_size=window))
        rc, claimed, _ = ep.capability(g)
        assert rc == 0 and claimed == [0], ep.report()
        idx = ep.compile(g, 0)
        assert idx >= 0, oh.last_error()
        dev = {k: to_dev(v) for k, v in dict(query=qn, key=kn, value=vn, past_key=pkn, past_value=pvn).items()}
        for k, v in dev.items():
            _bind(ctx, f"sw.{k}", v, oh.F32)
        meta = dict(seqlens_k=lens.copy(), total=total.copy())  # kept alive until Compute has run
        for k, v in meta.items():
            _bind(ctx, f"sw.{k}", v, oh.I32)
        out = torch.empty((2, 1, Hg * Dg), device="cuda")
        pk = torch.empty((2, KVg, cap, Dg), device="cuda")
        pv = torch.empty_like(pk)
        ctx.output("sw.out", oh.F32, (2, 1, Hg * Dg), out.data_ptr(), out.numel() * 4)
        ctx.output("sw.present_key", oh.F32, (2, KVg, cap, Dg), pk.data_ptr(), pk.numel() * 4)
        ctx.output("sw.present_value", oh.F32, (2, KVg, cap, Dg), pv.data_ptr(), pv.numel() * 4)
        rc = ep.compute(idx, ctx)
        assert rc == 0, oh.last_error()
        assert ctx.requested("sw.present_key") == (2, KVg, cap, Dg)
        got = out.cpu().numpy()
        assert float(np.abs(got - want).max()) <= 2e-5 + 2e-5 * float(np.abs(want).max())
        assert np.array_equal(pk.cpu().numpy(), wk) and np.array_equal(pv.cpu().numpy(), wv)
    finally:
        ctx.close()
        g.close()
