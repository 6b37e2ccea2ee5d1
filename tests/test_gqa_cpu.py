"""GroupQueryAttention on CPU: the claim predicate (b200_group_query_attention_claim, restating
group_query_attention_claim, rust/src/ops/attention.rs:2407-2754) and the host-side length
validation of b200_group_query_attention (reference messages, attention.rs:989-1030,
:613-630, :663-673).  Validation runs before any device work, so no GPU is needed."""

import ctypes

import numpy as np
import pytest

from onnxruntime_ep_b200 import _capi

F16, BF16, F32, I32, I8 = (_capi.DTYPE_FLOAT16, _capi.DTYPE_BFLOAT16, _capi.DTYPE_FLOAT, _capi.DTYPE_INT32,
                           _capi.DTYPE_INT8)


def tensor(info, dtype, shape):
    info.present = 1
    info.dtype = dtype
    info.rank = len(shape)
    for i, d in enumerate(shape):
        info.shape[i] = d


def gnode(H=32, KV=8, D=128, dt=F32, B=1, S=1, cap=2048, n_inputs=7, n_outputs=3, past=True):
    """BASELINE config 1 node: q [1,1,4096], k/v [1,1,1024], past [1,8,2048,128], fp32."""
    n = _capi.GqaNodeInfo()
    n.num_inputs, n.num_outputs = n_inputs, n_outputs
    n.num_heads, n.kv_num_heads = H, KV
    tensor(n.inputs[0], dt, [B, S, H * D])
    tensor(n.inputs[1], dt, [B, S, KV * D])
    tensor(n.inputs[2], dt, [B, S, KV * D])
    if past:
        tensor(n.inputs[3], dt, [B, KV, cap, D])
        tensor(n.inputs[4], dt, [B, KV, cap, D])
    tensor(n.inputs[5], I32, [B])
    tensor(n.inputs[6], I32, [1])
    tensor(n.outputs[0], dt, [B, S, H * D])
    if n_outputs >= 3:
        tensor(n.outputs[1], dt, [B, KV, -1, D])
        tensor(n.outputs[2], dt, [B, KV, -1, D])
    return n


def claim(n):
    buf = ctypes.create_string_buffer(512)
    ok = _capi.LIB.b200_group_query_attention_claim(ctypes.byref(n), buf, 512)
    return ok, buf.value.decode()


def test_layouts_match_library():
    assert _capi.LIB.b200_gqa_params_size() == ctypes.sizeof(_capi.GqaParams)
    assert _capi.LIB.b200_gqa_node_info_size() == ctypes.sizeof(_capi.GqaNodeInfo)


@pytest.mark.parametrize("dt", [F32, F16, BF16])
def test_claims_config1_node(dt):
    assert claim(gnode(dt=dt)) == (1, "")


def test_claims_packed_qkv_and_no_past():
    n = gnode(past=False)
    n.inputs[1].present = n.inputs[2].present = 0
    tensor(n.inputs[0], F32, [1, 1, (32 + 16) * 128])
    assert claim(n) == (1, "")


def _set(attr, value):
    def f(n):
        setattr(n, attr, value)
        if attr == "causal":
            n.has_causal = 1
        if attr == "local_window_size":
            n.has_local_window_size = 1
        if attr == "smooth_softmax":
            n.has_smooth_softmax = 1
    return f


@pytest.mark.parametrize("mutate,reason", [
    (_set("causal", 2), "causal must be 0 or 1"),
    (_set("local_window_size", 0), "local_window_size must be -1 or positive"),
    (lambda n: (_set("causal", 0)(n), _set("local_window_size", 4)(n)),
     "bidirectional GroupQueryAttention requires local_window_size=-1"),
    (lambda n: setattr(n.inputs[4], "present", 0), "past_key and past_value must be provided together"),
    (lambda n: tensor(n.outputs[0], I32, [1, 1, 4096]), "output must have an MLX float dtype, got int32"),
    (lambda n: setattr(n, "do_rotary", 1), "7-input GroupQueryAttention requires do_rotary=0"),
    (lambda n: tensor(n.inputs[1], F16, [1, 1, 1024]), "input 1 must have output dtype float32, got float16"),
    (lambda n: tensor(n.inputs[5], F32, [1]), "input 5 must have int32 dtype, got float32"),
    (lambda n: setattr(n, "kv_num_heads", 5), "num_heads (32) must be a positive multiple of kv_num_heads (5)"),
    (lambda n: tensor(n.inputs[1], F32, [1, 1, 512]), "key/value must match query batch"),
    (lambda n: tensor(n.inputs[3], F32, [1, 4, 2048, 128]), "past cache must be [batch,kv_num_heads"),
    (lambda n: tensor(n.inputs[6], I32, [2]), "total_sequence_length must be scalar or [1]"),
    (_set("smooth_softmax", 3), "smooth_softmax must be -1"),
    (lambda n: setattr(n, "qk_output", 1), "qk_output must be 0, 1 or 2 and enabled exactly when output_qk is present"),
    (lambda n: setattr(n, "softcap", float("inf")), "softcap must be finite and non-negative"),
])
def test_reference_declines(mutate, reason):
    n = gnode()
    mutate(n)
    ok, why = claim(n)
    assert ok == 0 and why.startswith(reason), why


def rotary(n, half=64, rows=4096, dt=F32, pos=None):
    n.num_inputs = 10 if pos is not None else 9
    n.do_rotary = 1
    tensor(n.inputs[7], dt, [rows, half])
    tensor(n.inputs[8], dt, [rows, half])
    if pos is not None:
        tensor(n.inputs[9], pos[0], pos[1])
    return n


@pytest.mark.parametrize("kw", [dict(), dict(half=32), dict(pos=(_capi.DTYPE_INT64, [1, 1])),
                                dict(pos=(_capi.DTYPE_INT64, [1, 5]))])
def test_rotary_nodes_are_claimed(kw):
    assert claim(rotary(gnode(), **kw)) == (1, "")


@pytest.mark.parametrize("mutate,reason", [
    (lambda n: rotary(n, half=65), "rotary caches must have matching [positions,rotary_dim/2] shapes within the head"),
    (lambda n: (rotary(n), tensor(n.inputs[8], F32, [2048, 64])),
     "rotary caches must have matching [positions,rotary_dim/2] shapes"),
    (lambda n: rotary(n, pos=(I32, [1, 1])), "position_ids must be int64 [batch,>=sequence_length]"),
    (lambda n: rotary(n, pos=(_capi.DTYPE_INT64, [2, 1])), "position_ids must be int64 [batch,>=sequence_length]"),
    (lambda n: rotary(n, dt=F16), "input 7 must have output dtype float32, got float16"),
])
def test_reference_rotary_declines(mutate, reason):
    n = gnode()
    mutate(n)
    ok, why = claim(n)
    assert ok == 0 and why.startswith(reason), why


def int_gnode(bits=8, modes=(b"PER_CHANNEL", b"PER_TENSOR")):
    """Config-1 geometry with integer caches (kv_cache_bit_width, scales on inputs 12 / 13)."""
    n = gnode(n_inputs=14)
    dt = I8 if bits == 8 else _capi.DTYPE_UINT8
    w = 128 if bits == 8 else 64
    for i in (3, 4):
        tensor(n.inputs[i], dt, [1, 8, 2048, w])
    for i in (1, 2):
        tensor(n.outputs[i], dt, [1, 8, -1, w])
    n.kv_cache_bit_width = bits
    n.k_quant_type, n.v_quant_type = modes
    for i, m in ((12, modes[0]), (13, modes[1])):
        tensor(n.inputs[i], F32, [8, 1, 128] if m == b"PER_CHANNEL" else [1])
    return n


@pytest.mark.parametrize("bits", [8, 4])
def test_integer_caches_are_claimed(bits):
    assert claim(int_gnode(bits)) == (1, "")


@pytest.mark.parametrize("mutate,reason", [
    (lambda n: setattr(n, "kv_cache_bit_width", 4), "kv_cache_bit_width must agree with cache storage"),
    (lambda n: setattr(n, "k_quant_type", b"NONE"), "integer k cache requires PER_TENSOR or PER_CHANNEL"),
    (lambda n: tensor(n.inputs[12], F32, [4]), "k_scale must contain 1024 elements"),
    (lambda n: setattr(n.inputs[13], "present", 0), "quantized v cache requires a scale tensor"),
    (lambda n: tensor(n.outputs[1], F32, [1, 8, -1, 128]), "output 1 must retain its cache dtype"),
])
def test_integer_cache_rules(mutate, reason):
    n = int_gnode()
    mutate(n)
    ok, why = claim(n)
    assert ok == 0 and reason in why, why


def test_attention_bias_is_claimed():
    n = gnode()
    n.num_inputs = 11
    tensor(n.inputs[10], F32, [1, 1, 1, 2049])
    assert claim(n) == (1, "")
    tensor(n.inputs[10], F32, [1, 2049])
    ok, why = claim(n)
    assert ok == 0 and "attention_bias (input 10) must have rank 4" in why
    tensor(n.inputs[10], F16, [1, 1, 1, 2049])
    ok, why = claim(n)
    assert ok == 0 and "input 10 must have output dtype" in why


def _sliding(window=64):
    def f(n):
        n.sliding_window_cache = 1
        if window is not None:
            _set("local_window_size", window)(n)
    return f


@pytest.mark.parametrize("bits", [0, 8, 4])
def test_sliding_window_cache_is_claimed(bits):
    n = int_gnode(bits) if bits else gnode()
    _sliding()(n)
    assert claim(n) == (1, "")


# attention.rs:2455-2475, :2588-2591, :2735-2738
@pytest.mark.parametrize("mutate,reason", [
    (_sliding(None), "sliding_window_cache=1 requires local_window_size > 0"),
    (lambda n: (_sliding()(n), setattr(n, "num_outputs", 1)), "sliding_window_cache requires present key/value outputs"),
    (_sliding(4096), "sliding-window key cache capacity must be at least local_window_size"),
    (lambda n: (_sliding()(n), tensor(n.inputs[4], F32, [1, 8, 32, 128])),
     "sliding-window value cache capacity must be at least local_window_size"),
    (lambda n: (_sliding()(n), setattr(n, "qk_output", 1), setattr(n, "num_outputs", 4),
                tensor(n.outputs[3], F32, [1, 32, 1, -1])),
     "sliding_window_cache with QK diagnostics is unsupported"),
])
def test_sliding_window_cache_rules(mutate, reason):
    n = gnode()
    mutate(n)
    ok, why = claim(n)
    assert ok == 0 and reason in why, why


def test_sliding_integer_rows_alignment():
    n = gnode(D=40, n_inputs=14)  # int8 rows of 40 channels: not a multiple of 16
    for i in (3, 4):
        tensor(n.inputs[i], I8, [1, 8, 2048, 40])
    for i in (1, 2):
        tensor(n.outputs[i], I8, [1, 8, -1, 40])
    n.kv_cache_bit_width = 8
    n.k_quant_type = n.v_quant_type = b"PER_TENSOR"
    for i in (12, 13):
        tensor(n.inputs[i], F32, [1])
    assert claim(n) == (1, "")
    _sliding()(n)
    ok, why = claim(n)
    assert ok == 0 and "sliding integer cache rows must satisfy pinned 16-byte alignment" in why, why


def params(lengths, total, S=1, new_seq=1, cap=2048, B=None, causal=1, window=-1, present_cap=None):
    B = len(lengths) if B is None else B
    p = _capi.GqaParams()
    p.num_heads, p.kv_num_heads, p.head_size = 32, 8, 128
    p.is_causal, p.local_window_size, p.smooth_softmax = causal, window, -1
    p.dtype = F32
    p.batch, p.seq, p.new_seq, p.cap = B, S, new_seq, cap
    p.total_sequence_length = total
    p.present_cap = max(cap, total) if present_cap is None else present_cap
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: validation fails first
    for f in ("query", "key", "value", "past_key", "past_value", "seqlens_k", "output", "workspace"):
        setattr(p, f, fake)
    p.present_key, p.present_value = ctypes.c_void_p(0x2000), ctypes.c_void_p(0x3000)
    host = np.asarray(lengths, np.int32)
    p.host_seqlens_k = host.ctypes.data_as(ctypes.c_void_p)
    p.workspace_bytes = 1 << 30
    return p, host


@pytest.mark.parametrize("lengths,total,S,new_seq,cap,message", [
    ([2047], 2049, 1, 1, 2048, "GroupQueryAttention: inconsistent sequence lengths or cache capacity"),
    ([2048], 2050, 1, 1, 2048, "GroupQueryAttention: inconsistent sequence lengths or cache capacity"),
    ([3, 9], 9, 1, 1, 16, "GroupQueryAttention: invalid per-batch or maximum sequence lengths"),
    ([3, 7], 9, 1, 1, 16, "GroupQueryAttention: invalid per-batch or maximum sequence lengths"),
    ([0, 8], 9, 4, 4, 16, "GroupQueryAttention: invalid per-batch or maximum sequence lengths"),
    ([20, 8], 21, 1, 0, 16, "GroupQueryAttention: sequence length exceeds available past cache"),
    ([2048], -1, 1, 1, 2048, "GroupQueryAttention: total_sequence_length is outside int32 range"),
])
def test_length_validation_messages(lengths, total, S, new_seq, cap, message):
    p, keep = params(lengths, total, S=S, new_seq=new_seq, cap=cap)
    rc = _capi.LIB.b200_group_query_attention(ctypes.byref(p), None)
    assert rc == _capi.B200_ERR_FAIL
    assert _capi.LIB.b200_last_error().decode() == message


def sliding_params(lengths, total, S=1, cap=16, window=4, present_cap=None):
    p, keep = params(lengths, total, S=S, new_seq=S, cap=cap, window=window,
                     present_cap=cap if present_cap is None else present_cap)
    p.sliding_window_cache = 1
    return p, keep


# attention.rs:1140-1171 (lengths, bias columns, window / capacity), in that order
@pytest.mark.parametrize("lengths,total,S,cap,window,message", [
    ([3, 9], 9, 1, 16, 4, "GroupQueryAttention: invalid sliding sequence lengths"),
    ([3, 7], 9, 1, 16, 4, "GroupQueryAttention: invalid sliding sequence lengths"),
    ([1, 8], 9, 3, 16, 4, "GroupQueryAttention: invalid sliding sequence lengths"),
    ([40], 41, 1, 16, 17, "GroupQueryAttention: sliding cache requires 0 < local_window_size <= capacity"),
])
def test_sliding_validation_messages(lengths, total, S, cap, window, message):
    p, keep = sliding_params(lengths, total, S=S, cap=cap, window=window)
    assert _capi.LIB.b200_group_query_attention(ctypes.byref(p), None) == _capi.B200_ERR_FAIL
    assert _capi.LIB.b200_last_error().decode() == message


def test_sliding_bias_needs_absolute_columns():
    p, keep = sliding_params([40], 41)
    p.attention_bias = ctypes.c_void_p(0x4000)
    p.bias_batch, p.bias_heads, p.bias_seq, p.bias_total = 1, 1, 1, 16  # the cache's columns
    assert _capi.LIB.b200_group_query_attention(ctypes.byref(p), None) == _capi.B200_ERR_FAIL
    assert _capi.LIB.b200_last_error().decode() == (
        "GroupQueryAttention: sliding attention_bias requires absolute total_sequence_length columns")


def test_sliding_contract_errors():
    p, keep = sliding_params([40], 41, present_cap=41)
    assert _capi.LIB.b200_group_query_attention(ctypes.byref(p), None) == _capi.B200_ERR_INVALID_ARGUMENT
    assert "a sliding present must have the past's capacity" in _capi.LIB.b200_last_error().decode()
    p, keep = sliding_params([40], 41)
    p.new_seq = 0
    assert _capi.LIB.b200_group_query_attention(ctypes.byref(p), None) == _capi.B200_ERR_FAIL
    assert _capi.LIB.b200_last_error().decode() == (
        "GroupQueryAttention: K/V must match Q sequence or be empty with paired non-sliding past")
    p, keep = sliding_params([40], 41)
    p.qk_output, p.output_qk = 1, ctypes.c_void_p(0x5000)
    assert _capi.LIB.b200_group_query_attention(ctypes.byref(p), None) == _capi.B200_ERR_UNSUPPORTED
    assert _capi.LIB.b200_last_error().decode() == "sliding_window_cache with QK diagnostics is unsupported"
    p, keep = sliding_params([40], 41)
    p.present_key = p.present_value = None
    assert _capi.LIB.b200_group_query_attention(ctypes.byref(p), None) == _capi.B200_ERR_INVALID_ARGUMENT
    assert _capi.LIB.b200_last_error().decode() == "sliding_window_cache requires present key/value outputs"


def test_sliding_workspace_holds_staged_present():
    p, keep = sliding_params([40], 41, cap=16)
    n0, n1 = ctypes.c_size_t(0), ctypes.c_size_t(0)
    assert _capi.LIB.b200_group_query_attention_workspace_size(ctypes.byref(p), ctypes.byref(n1)) == 0
    p.sliding_window_cache = 0
    p.present_cap = 41
    assert _capi.LIB.b200_group_query_attention_workspace_size(ctypes.byref(p), ctypes.byref(n0)) == 0
    assert n1.value - n0.value >= 2 * 1 * 8 * 16 * 128 * 4  # K and V rows of the capacity, fp32


def test_new_rows_must_match_query_sequence():
    p, keep = params([2048], 2049, S=2, new_seq=1)
    assert _capi.LIB.b200_group_query_attention(ctypes.byref(p), None) == _capi.B200_ERR_FAIL
    assert _capi.LIB.b200_last_error().decode() == (
        "GroupQueryAttention: K/V must match Q sequence or be empty with paired non-sliding past")


def test_workspace_size_is_shape_only():
    p, keep = params([2048], 2049)
    n = ctypes.c_size_t(0)
    assert _capi.LIB.b200_group_query_attention_workspace_size(ctypes.byref(p), ctypes.byref(n)) == 0
    assert n.value >= 256


# ---- rotary positions, checked on the host before any launch (attention.rs:525-585) ----------
def rotary_params(lengths, total, S, rows=64, ids=None, width=None):
    """`lengths` are seqlens_k values (length - 1), as in ``params``."""
    p, host = params(lengths, total, S=S, new_seq=S, cap=64)
    keep = [host]
    cos = ctypes.c_void_p(0x3000)
    p.do_rotary, p.rotary_dim, p.rotary_positions = 1, 64, rows
    p.cos_cache = p.sin_cache = cos
    if ids is not None:
        ids = np.ascontiguousarray(ids, np.int64)
        keep.append(ids)
        p.position_ids = ctypes.c_void_p(0x4000)
        p.host_position_ids = ids.ctypes.data
        p.position_ids_width = ids.shape[1] if width is None else width
    return p, keep


def gqa_call(p):
    return _capi.LIB.b200_group_query_attention(ctypes.byref(p), None)


def test_rotary_positions_past_the_cache_without_ids():
    p, keep = rotary_params([63], 64, S=1, rows=63)  # length 64: query_past 63 needs 64 rows
    assert gqa_call(p) == _capi.B200_ERR_FAIL
    assert "RotaryEmbedding: requested positions exceed the supplied cache" in _capi.LIB.b200_last_error().decode()


@pytest.mark.parametrize("bad", [-1, 64, 2**32, 2**63 - 1])
def test_rotary_position_ids_out_of_range(bad):
    # later call: the first batch * seq flattened ids must all be inside the cache
    p, keep = rotary_params([4, 5], 6, S=2, ids=[[1, bad], [2, 3]])
    assert gqa_call(p) == _capi.B200_ERR_FAIL
    assert "position_ids exceed the supplied cache" in _capi.LIB.b200_last_error().decode()


def test_rotary_first_prompt_offset_span():
    # total == seq: only the first id counts, and offset + seq must stay inside the cache
    p, keep = rotary_params([2], 3, S=3, ids=[[62, 0, 0]])
    assert gqa_call(p) == _capi.B200_ERR_FAIL
    assert "position_ids exceed the supplied cache" in _capi.LIB.b200_last_error().decode()


def test_rotary_position_ids_too_narrow():
    p, keep = rotary_params([4, 5], 6, S=2, ids=[[1], [2]])
    assert gqa_call(p) == _capi.B200_ERR_FAIL
    assert "position_ids must be int64 [batch,>=sequence]" in _capi.LIB.b200_last_error().decode()
