"""GPU parity of b200_group_query_attention against the reference's own oracle (golden cases)
and against oracle/gqa_ref.py (BASELINE config 1 at full size and a sweep of forms)."""

import json
import os

import numpy as np
import pytest

from oracle import gqa_ref, tolerance

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from onnxruntime_ep_b200 import gqa  # noqa: E402

DEV = torch.device("cuda", 0)
GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "gqa_golden.npz"))
META = json.loads(bytes(GOLDEN["meta"]).decode())
TORCH_DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def dev(a, dtype=None):
    if a is None:
        return None
    t = torch.from_numpy(np.ascontiguousarray(a).view(np.uint16) if a.dtype.name == "bfloat16" else np.ascontiguousarray(a))
    if a.dtype.name == "bfloat16":
        t = t.view(torch.bfloat16)
    return t.to(DEV)


def host(t):
    if t.dtype == torch.bfloat16:
        return t.float().cpu().numpy()
    return t.cpu().numpy()


def check(out, want, dtype):
    out = np.asarray(out, np.float32)
    want = np.asarray(want, np.float32)
    if dtype == "float32":
        bound = 2e-5 + 2e-5 * np.abs(want)
    else:  # fp32 recomputation tolerance on the error beyond the output's rounding (half an ulp)
        rep = tolerance.report(out, want, bits=8 if dtype == "bfloat16" else 11)
        assert rep["max_excess"] <= 2e-3, rep
        return
    err = np.abs(out - want)
    assert np.all(err <= bound), f"max err {err.max()} (worst excess {(err - bound).max()})"


@pytest.mark.parametrize("in_place", [False, True])
@pytest.mark.parametrize("case", META, ids=[c["name"] for c in META])
def test_golden_cases(case, in_place):
    name = case["name"]
    f = {k.split("/")[-1]: GOLDEN[k] for k in GOLDEN.files if k.startswith(f"{name}/in/")}
    q, pk, pv = dev(f["q"]), dev(f["pk"]), dev(f["pv"])
    k = dev(f["k"]) if case["new_seq"] else None
    v = dev(f["v"]) if case["new_seq"] else None
    if not case["new_seq"]:
        k = torch.empty((case["batch"], 0, 2 * 32), dtype=q.dtype, device=DEV)
        v = torch.empty_like(k)
    lengths = dev(f["lengths"])
    kw = dict(num_heads=4, kv_num_heads=2, causal=int(case["causal"]), local_window_size=case["window"],
              softcap=0.7 if case["composed"] else 0.0)
    sink = dev(f["sink"]) if "sink" in f else None
    if in_place:
        kw.update(present_key=pk, present_value=pv)
    if "cos" in f:  # rotary: cos / sin caches, optional position ids (host copy for validation)
        kw.update(do_rotary=1, rotary_interleaved=int(case.get("interleaved", False)), cos_cache=dev(f["cos"]),
                  sin_cache=dev(f["sin"]), position_ids=f.get("pos"))
    if "bias" in f:  # attention_bias [1|B, 1|H, S, total]
        kw["attention_bias"] = dev(f["bias"])
    if case.get("bits"):  # integer caches: codes in pk / pv, scales (inputs 12 / 13)
        kw.update(k_scale=dev(f["k_scale"]), v_scale=dev(f["v_scale"]), k_quant_type=case["quant_modes"][0],
                  v_quant_type=case["quant_modes"][1])
    if case.get("sliding"):  # sliding_window_cache=1: present keeps the past's capacity
        kw["sliding_window_cache"] = 1
    mode = case.get("mode", 0)
    res = gqa.group_query_attention(q, k, v, pk, pv, lengths, int(f["total"][0]), sink, check_status=True,
                                    qk_output=mode, **kw)
    out, ok, ov = res[:3]
    torch.cuda.synchronize()
    check(host(out), GOLDEN[f"{name}/out/output"], case["dtype"])
    if mode:  # qk_output diagnostics [B, H, S, total]
        check(host(res[3]), GOLDEN[f"{name}/out/qk"], case["dtype"])
    np.testing.assert_array_equal(host(ok), GOLDEN[f"{name}/out/present_k"])
    np.testing.assert_array_equal(host(ov), GOLDEN[f"{name}/out/present_v"])


def run_case(rng, *, dtype="bfloat16", B=1, S=1, H=32, KV=8, D=128, cap=2048, lengths=None, total=None,
             causal=1, window=-1, softcap=0.0, sink=False, smooth=-1, packed=False, new_rows=True, past=True,
             in_place=False, rotary=None, bias=None, qk_norm=False, sliding=False):
    npdt = np.float32
    lengths = [cap + S] * B if lengths is None else lengths
    B = len(lengths)
    total = max(lengths) if total is None else total
    new_seq = S if new_rows else 0
    q = (rng.standard_normal((B, S, H * D)) * 0.5).astype(npdt)
    k = (rng.standard_normal((B, new_seq, KV * D)) * 0.5).astype(npdt)
    v = (rng.standard_normal((B, new_seq, KV * D)) * 0.5).astype(npdt)
    pkn = (rng.standard_normal((B, KV, cap, D)) * 0.5).astype(npdt) if past else None
    pvn = (rng.standard_normal((B, KV, cap, D)) * 0.5).astype(npdt) if past else None
    sk = np.linspace(-1, 1, H).astype(npdt) if sink else None
    tdt = TORCH_DT[dtype]
    to = lambda a: None if a is None else torch.from_numpy(a).to(DEV).to(tdt)
    # round the inputs to the activation type first so the oracle sees the same values
    qt, kt, vt, pkt, pvt, skt = map(to, (q, k, v, pkn, pvn, sk))
    back = lambda t: None if t is None else t.float().cpu().numpy()
    qn, kn, vn, pkr, pvr, skr = map(back, (qt, kt, vt, pkt, pvt, skt))
    rot = {}
    kw_rot = {}
    if rotary is not None:  # (half, interleaved, position ids or None), cos / sin in the activation type
        half, inter, ids = rotary
        rows = max(lengths) + 8
        cos = rng.uniform(0.5, 1.5, (rows, half)).astype(npdt)
        sin = rng.uniform(-0.5, 0.5, (rows, half)).astype(npdt)
        ct, st = to(cos), to(sin)
        rot = dict(cos=back(ct), sin=back(st), position_ids=ids, interleaved=inter)
        kw_rot = dict(do_rotary=1, rotary_interleaved=int(inter), cos_cache=ct, sin_cache=st, position_ids=ids)
        if dtype != "float32":
            # the oracle sees the activation type, so its rotated rows are rounded like the kernel's
            import ml_dtypes
            ndt = np.float16 if dtype == "float16" else ml_dtypes.bfloat16
            cast = lambda a: None if a is None else a.astype(ndt)
            qn, kn, vn, pkr, pvr, skr = map(cast, (qn, kn, vn, pkr, pvr, skr))
            rot.update(cos=cast(rot["cos"]), sin=cast(rot["sin"]))
    bias_t = bias_n = None
    if bias is not None:  # (batch dim, head dim) of an attention_bias [1|B, 1|H, S, total]
        bias_t = to(rng.uniform(-2, 2, (bias[0], bias[1], S, total)).astype(npdt))
        bias_n = back(bias_t)
        if dtype != "float32":
            import ml_dtypes
            bias_n = bias_n.astype(np.float16 if dtype == "float16" else ml_dtypes.bfloat16)
    norm_t, norm_n = {}, {}
    if qk_norm:  # q / k RMS norm weights [D] in the activation type, epsilon 1e-5
        qw_t, kw_t = to(rng.uniform(0.5, 1.5, D).astype(npdt)), to(rng.uniform(0.5, 1.5, D).astype(npdt))
        qw_n, kw_n = back(qw_t), back(kw_t)
        if dtype != "float32":
            import ml_dtypes
            ndt = np.float16 if dtype == "float16" else ml_dtypes.bfloat16
            qn, kn, vn, pkr, pvr, skr = (None if a is None else a.astype(ndt) for a in (qn, kn, vn, pkr, pvr, skr))
            qw_n, kw_n = qw_n.astype(ndt), kw_n.astype(ndt)
        norm_t = dict(q_norm_weight=qw_t, k_norm_weight=kw_t, qk_norm_epsilon=1e-5)
        norm_n = dict(q_norm=qw_n, k_norm=kw_n, norm_eps=1e-5)
    want, wk, wv = gqa_ref.group_query_attention(
        qn, kn if new_rows else None, vn if new_rows else None, pkr, pvr, np.asarray(lengths) - 1, total,
        num_heads=H, kv_num_heads=KV, causal=bool(causal), window=window, softcap=softcap, sink=skr,
        smooth_softmax=smooth, out_dtype=np.float32, bias=bias_n, sliding=sliding, **rot, **norm_n)
    want, wk, wv = (np.asarray(x, np.float32) for x in (want, wk, wv))
    lens = torch.tensor(np.asarray(lengths) - 1, dtype=torch.int32, device=DEV)
    kw = dict(num_heads=H, kv_num_heads=KV, causal=causal, local_window_size=window, softcap=softcap,
              smooth_softmax=smooth, attention_bias=bias_t, sliding_window_cache=int(sliding), **kw_rot, **norm_t)
    if in_place:
        kw.update(present_key=pkt, present_value=pvt)
    if packed:
        qkv = torch.cat([qt, kt, vt], dim=2).contiguous()
        out, ok, ov = gqa.group_query_attention(qkv, None, None, pkt, pvt, lens, total, skt, check_status=True, **kw)
    else:
        out, ok, ov = gqa.group_query_attention(qt, kt, vt, pkt, pvt, lens, total, skt, check_status=True, **kw)
    torch.cuda.synchronize()
    check(back(out), want, dtype)
    if ok is not None:
        n = min(ok.shape[2], wk.shape[2])
        if qk_norm:  # normalised key rows: the row sum's order may move the rounding by one ulp
            ulp = {"float32": 2.0 ** -23, "float16": 2.0 ** -10, "bfloat16": 2.0 ** -7}[dtype]
            np.testing.assert_allclose(back(ok)[:, :, :n], wk[:, :, :n], rtol=ulp, atol=1e-6)
        else:
            np.testing.assert_array_equal(back(ok)[:, :, :n], wk[:, :, :n])
        np.testing.assert_array_equal(back(ov)[:, :, :n], wv[:, :, :n])


def test_config1_fp32_growing_cache():
    """B=1, 32q/8kv, d128, fp32, past [1,8,2048,128], one new token, total 2049."""
    run_case(np.random.default_rng(1), dtype="float32", cap=2048, lengths=[2049])


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_decode_dtypes_and_head_sizes(dtype, D):
    run_case(np.random.default_rng(D), dtype=dtype, D=D, H=16, KV=4, cap=700, lengths=[701, 650, 10])


@pytest.mark.parametrize("H,KV", [(8, 8), (32, 4), (64, 8), (24, 2)])
def test_grouping(H, KV):
    run_case(np.random.default_rng(H + KV), H=H, KV=KV, cap=300, lengths=[301, 120])


def test_long_context_split_merge():
    run_case(np.random.default_rng(5), cap=9000, lengths=[9001])


@pytest.mark.parametrize("S", [7, 40, 300])
def test_prefill_rows(S):
    run_case(np.random.default_rng(S), S=S, cap=64, lengths=[64 + S, S + 5], H=8, KV=2)


def test_prefill_without_past():
    run_case(np.random.default_rng(9), S=33, past=False, cap=0, lengths=[33, 20], H=8, KV=2)


@pytest.mark.parametrize("window,softcap,sink,smooth", [(16, 0.0, False, -1), (-1, 5.0, True, -1),
                                                        (40, 3.0, False, 1), (-1, 0.0, False, 1)])
def test_window_softcap_sink(window, softcap, sink, smooth):
    run_case(np.random.default_rng(11), dtype="float16", S=5, cap=128, lengths=[133, 90], H=8, KV=2,
             window=window, softcap=softcap, sink=sink, smooth=smooth)


def test_bidirectional():
    run_case(np.random.default_rng(12), S=9, cap=50, lengths=[59, 30], H=8, KV=4, causal=0)


def test_packed_qkv():
    run_case(np.random.default_rng(13), S=3, cap=40, lengths=[43], packed=True)


def test_past_only_decode():
    run_case(np.random.default_rng(14), S=1, cap=500, lengths=[500, 321], new_rows=False)


def test_in_place_shared_buffer():
    run_case(np.random.default_rng(15), S=2, cap=1024, lengths=[600, 1000], in_place=True)


# ---- rotary embedding inside the node (do_rotary=1) ------------------------------------------
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_config1_with_rotary(dtype):
    """Config-1 shapes with RoPE on the new rows at position query_past (no position_ids)."""
    run_case(np.random.default_rng(21), dtype=dtype, cap=2048, lengths=[2049], rotary=(64, False, None))


@pytest.mark.parametrize("half,inter", [(64, False), (64, True), (32, False), (16, True)])
def test_rotary_forms_with_position_ids(half, inter):
    ids = np.array([[40], [77]], np.int64)  # later call: the first batch * seq flattened ids
    run_case(np.random.default_rng(22 + half), dtype="float16", H=16, KV=4, cap=300, lengths=[301, 120],
             rotary=(half, inter, ids))


def test_rotary_first_prompt_offset_and_packed():
    # total == seq: only the first id is used, as an offset for every batch row
    ids = np.array([[3, 99, 99, 99, 99, 99, 99, 99]], np.int64)
    run_case(np.random.default_rng(23), S=8, cap=0, past=False, lengths=[8], total=8, H=8, KV=2, packed=True,
             rotary=(64, False, ids))


def test_rotary_prefill_rows_and_past_only():
    run_case(np.random.default_rng(24), S=40, cap=64, lengths=[104, 45], H=8, KV=2, rotary=(32, True, None))
    run_case(np.random.default_rng(25), S=1, cap=500, lengths=[500, 321], new_rows=False,
             rotary=(64, False, np.array([[499], [320]], np.int64)))


# ---- attention_bias (input 10) ------------------------------------------------------------
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_config1_with_bias(dtype):
    """Config-1 shapes (the one-wave cluster kernel) with a per-head bias over the 2049 keys."""
    run_case(np.random.default_rng(31), dtype=dtype, cap=2048, lengths=[2049], bias=(1, 32))


@pytest.mark.parametrize("shape", [(2, 8), (1, 1), (2, 1)])
def test_bias_prefill_rows_and_broadcast(shape):
    """Prefill rows (the split-K attention kernel) with batch / head broadcast and a window."""
    run_case(np.random.default_rng(32), dtype="float16", S=24, cap=64, lengths=[88, 50], H=8, KV=2, window=16,
             bias=shape)


def test_bias_with_softcap_sink_and_rotary():
    run_case(np.random.default_rng(33), dtype="bfloat16", S=3, cap=128, lengths=[131, 90], H=16, KV=4,
             softcap=30.0, sink=True, rotary=(64, False, None), bias=(2, 16))


# ---- q / k RMS norm (inputs 14 / 15) --------------------------------------------------------
def test_qk_norm_reference_case():
    """tests/ops/test_gqa11.py:52-130: fp32, 4q/2kv, head 8, past 2, three new rows, eps 1e-5."""
    f = {k.split("/")[-1]: GOLDEN[k] for k in GOLDEN.files if k.startswith("qknorm/in/")}
    out, ok, ov = gqa.group_query_attention(
        dev(f["q"]), dev(f["k"]), dev(f["v"]), dev(f["pk"]), dev(f["pv"]), dev(f["lengths"]), int(f["total"][0]),
        num_heads=4, kv_num_heads=2, q_norm_weight=dev(f["qw"]), k_norm_weight=dev(f["kw"]),
        qk_norm_epsilon=float(f["eps"][0]), check_status=True)
    torch.cuda.synchronize()
    np.testing.assert_allclose(host(out), GOLDEN["qknorm/out/output"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(host(ok), GOLDEN["qknorm/out/present_k"], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(host(ov), GOLDEN["qknorm/out/present_v"])


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_config1_with_qk_norm_and_rotary(dtype):
    run_case(np.random.default_rng(41), dtype=dtype, cap=2048, lengths=[2049], qk_norm=True,
             rotary=(64, False, None))


def test_qk_norm_prefill_rows():
    run_case(np.random.default_rng(42), dtype="float16", S=17, cap=64, lengths=[81, 30], H=8, KV=2, qk_norm=True)


# ---- integer caches (kv_cache_bit_width 8 / 4, inputs 12 / 13) ---------------------------------
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("dtype,S,lengths,cap", [("float32", 1, [2049], 2048), ("bfloat16", 5, [300, 77], 320)])
def test_integer_caches(bits, dtype, S, lengths, cap):
    """Config-1 geometry (and a ragged prefill batch) with int8 / int4 caches: present codes
    bit-exact, attention within the fp32 tolerance of the decoded-cache oracle."""
    run_int(bits, dtype, S, lengths, cap)


def run_int(bits, dtype, S, lengths, cap, window=-1, sliding=False, in_place=False):
    rng = np.random.default_rng(50 + bits + S)
    H, KV, D = 32, 8, 128
    B = len(lengths)
    total = max(lengths)
    tdt = TORCH_DT[dtype]
    to = lambda a: torch.from_numpy(a).to(DEV).to(tdt)
    q, k, v = (to((rng.standard_normal((B, S, n * D)) * 0.5).astype(np.float32)) for n in (H, KV, KV))
    back = lambda t: t.float().cpu().numpy()
    ks = rng.uniform(0.01, 0.05, (KV, D)).astype(np.float32)   # PER_CHANNEL keys
    vs = np.array([0.03], np.float32)                          # PER_TENSOR values
    pkf = (rng.standard_normal((B, KV, cap, D)) * 0.5).astype(np.float32)
    pvf = (rng.standard_normal((B, KV, cap, D)) * 0.5).astype(np.float32)
    pk = gqa_ref.int_encode(pkf, ks.reshape(KV, 1, D), bits)
    pv = gqa_ref.int_encode(pvf, vs, bits)
    qn, kn, vn = back(q), back(k), back(v)
    if dtype != "float32":
        import ml_dtypes
        qn, kn, vn = (a.astype(ml_dtypes.bfloat16) for a in (qn, kn, vn))
    lens = np.asarray(lengths) - 1
    want, wk, wv = gqa_ref.group_query_attention(qn, kn, vn, pk, pv, lens, total, num_heads=H, kv_num_heads=KV,
                                                 out_dtype=np.float32, k_scale=ks, v_scale=vs, window=window,
                                                 sliding=sliding)
    pkt, pvt = torch.from_numpy(pk).to(DEV), torch.from_numpy(pv).to(DEV)
    extra = dict(present_key=pkt, present_value=pvt) if in_place else {}
    out, ok, ov = gqa.group_query_attention(
        q, k, v, pkt, pvt, torch.tensor(lens, dtype=torch.int32, device=DEV), total, num_heads=H, kv_num_heads=KV,
        k_scale=torch.from_numpy(ks).to(DEV), v_scale=torch.from_numpy(vs).to(DEV), k_quant_type="PER_CHANNEL",
        v_quant_type="PER_TENSOR", local_window_size=window, sliding_window_cache=int(sliding), check_status=True,
        **extra)
    torch.cuda.synchronize()
    check(back(out), want, dtype)
    np.testing.assert_array_equal(ok.cpu().numpy(), wk)
    np.testing.assert_array_equal(ov.cpu().numpy(), wv)


# ---- sliding_window_cache=1 (attention.rs:1139-1379) -------------------------------------------
# The cache keeps resident(n) rows of a length-n sequence (whole gaps of cap - window + 1 rows
# reclaimed from the front past the capacity); present (the past's capacity, or the past buffer
# itself) holds the last resident(length) rows, then zeros.  Output within the fp32 tolerance of
# the oracle, present bit-exact over all capacity rows.
@pytest.mark.parametrize("in_place", [False, True])
@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_sliding_decode(dtype, in_place):
    """32q/8kv, d128, a 256-row cache with a 128-token window: two lengths past the capacity
    (rows reclaimed and moved down), one below it."""
    run_case(np.random.default_rng(60), dtype=dtype, cap=256, window=128, lengths=[1000, 300, 200],
             sliding=True, in_place=in_place)


@pytest.mark.parametrize("S,lengths", [(8, [700, 410]), (100, [700, 100]), (300, [700, 300])])
def test_sliding_chunks(S, lengths):
    """Chunks of 8 rows, longer than the window, and longer than the capacity (the rows a chunk
    drops are still read by its first queries)."""
    run_case(np.random.default_rng(61 + S), dtype="bfloat16", S=S, H=8, KV=2, cap=128, window=64, lengths=lengths,
             sliding=True, in_place=True)


def test_sliding_window_equals_capacity():
    """gap 1: every row past the capacity reclaims one."""
    run_case(np.random.default_rng(62), dtype="float16", S=2, H=8, KV=2, cap=64, window=64, lengths=[200, 65, 64],
             sliding=True)


def test_sliding_rotary_bias_composed():
    """Rotary at absolute positions, absolute bias columns, softcap and sink together."""
    run_case(np.random.default_rng(63), dtype="float16", S=3, H=16, KV=4, cap=96, window=40, lengths=[500, 97, 60],
             sliding=True, rotary=(64, False, None), bias=(3, 16), softcap=30.0, sink=True, in_place=True)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("in_place", [False, True])
def test_sliding_integer_caches(bits, in_place):
    """int8 / int4 sliding caches: resident codes moved, new rows encoded, zero codes after."""
    run_int(bits, "bfloat16", 4, [700, 300, 130], 256, window=100, sliding=True, in_place=in_place)
