"""Claim predicate (b200_paged_attention_claim) on CPU: accepts what the reference's
paged_attention_claim accepts (rust/src/ops/attention.rs:4384-4645, kv_cache.rs:16-108) and
declines with the reference's reasons otherwise."""

import ctypes

import pytest

from onnxruntime_ep_b200 import _capi

F16, BF16, F32, I32, I8, U8 = (_capi.DTYPE_FLOAT16, _capi.DTYPE_BFLOAT16, _capi.DTYPE_FLOAT,
                               _capi.DTYPE_INT32, _capi.DTYPE_INT8, _capi.DTYPE_UINT8)
F8 = _capi.DTYPE_FLOAT8E4M3FN


def tensor(info, dtype, shape):
    info.present = 1
    info.dtype = dtype
    info.rank = len(shape)
    for i, d in enumerate(shape):
        info.shape[i] = d


def node(H=4, KV=2, d=16, dt=F16, nb=8, bs=4, B=2, maxb=4, cache_dt=None, n_inputs=8, n_outputs=1):
    n = _capi.NodeInfo()
    n.num_inputs, n.num_outputs = n_inputs, n_outputs
    n.num_heads, n.kv_num_heads, n.is_causal, n.local_window_size = H, KV, 1, -1
    cache_dt = cache_dt or dt
    cw = d if cache_dt != U8 else (d + 1) // 2
    tensor(n.inputs[0], dt, [-1, H * d])
    tensor(n.inputs[1], dt, [-1, KV * d])
    tensor(n.inputs[2], dt, [-1, KV * d])
    tensor(n.inputs[3], cache_dt, [nb, bs, KV, cw])
    tensor(n.inputs[4], cache_dt, [nb, bs, KV, cw])
    tensor(n.inputs[5], I32, [B + 1])
    tensor(n.inputs[6], I32, [B])
    tensor(n.inputs[7], I32, [B, maxb])
    tensor(n.outputs[0], dt, [-1, H * d])
    return n


def claim(n):
    buf = ctypes.create_string_buffer(512)
    ok = _capi.LIB.b200_paged_attention_claim(ctypes.byref(n), buf, 512)
    return ok, buf.value.decode()


def test_claims_plain_fp16_and_bf16():
    for dt in (F16, BF16):
        ok, why = claim(node(dt=dt))
        assert ok == 1 and why == ""


def test_packed_qkv_is_claimed():
    n = node()
    n.inputs[1].present = n.inputs[2].present = 0
    tensor(n.inputs[0], F16, [-1, (4 + 2 * 2) * 16])
    assert claim(n)[0] == 1


@pytest.mark.parametrize("mutate,reason", [
    (lambda n: setattr(n, "is_causal", 2), "is_causal must be 0 or 1"),
    (lambda n: tensor(n.outputs[0], F32, [-1, 64]), "only supported for fp16/bf16"),
    (lambda n: setattr(n, "kv_num_heads", 3), "must be a positive multiple of kv_num_heads"),
    (lambda n: tensor(n.inputs[5], F32, [3]), "input 5 must be int32"),
    (lambda n: setattr(n, "local_window_size", 0), "local_window_size must be -1 or positive"),
    (lambda n: setattr(n, "softcap", -1.0), "softcap must be finite and non-negative"),
    (lambda n: setattr(n, "do_rotary", 1), "do_rotary=1 requires cos_cache and sin_cache"),
    (lambda n: tensor(n.inputs[3], F16, [8, 4, 3, 16]), "key_cache must be [num_blocks,block_size,kv_num_heads,head_size]"),
    (lambda n: (setattr(n, "num_inputs", 11), tensor(n.inputs[10], F32, [-1])), "slot_mapping must be int32"),
    (lambda n: (setattr(n, "num_inputs", 12), tensor(n.inputs[11], F16, [3])), "head_sink must be [num_heads]"),
    (lambda n: (setattr(n, "num_inputs", 13), tensor(n.inputs[12], F16, [16])), "must be provided together"),
    (lambda n: setattr(n, "num_outputs", 4), "requires 1 to 3 outputs"),
])
def test_declines_with_reference_reason(mutate, reason):
    n = node()
    mutate(n)
    ok, why = claim(n)
    assert ok == 0 and reason in why, why


def test_rotary_offset_rules():
    n = node(n_inputs=10)
    n.do_rotary = 1
    tensor(n.inputs[8], F16, [64, 4])
    tensor(n.inputs[9], F16, [64, 4])
    assert claim(n)[0] == 1
    n.rotary_offset = 4
    ok, why = claim(n)
    assert ok == 0 and "multiple of 8" in why
    n.rotary_offset = 16
    ok, why = claim(n)
    assert ok == 0 and "must not exceed head_size" in why


def test_integer_cache_claim():
    n = node(cache_dt=I8, n_inputs=16)
    ok, why = claim(n)
    assert ok == 0 and "requires PER_TENSOR or PER_CHANNEL" in why
    n.k_quant_type = n.v_quant_type = b"PER_TENSOR"
    ok, why = claim(n)
    assert ok == 0 and "requires a scale tensor" in why
    tensor(n.inputs[14], F32, [1])
    tensor(n.inputs[15], F32, [1])
    assert claim(n)[0] == 1
    # int4 storage must be named explicitly (kv_cache.rs:90-100)
    m = node(cache_dt=U8, n_inputs=16)
    m.k_quant_type = m.v_quant_type = b"PER_CHANNEL"
    tensor(m.inputs[14], F32, [2, 1, 16])
    tensor(m.inputs[15], F32, [2, 1, 16])
    ok, why = claim(m)
    assert ok == 0 and "uint8 requires explicit int4" in why
    m.k_cache_dtype = m.v_cache_dtype = b"int4"
    assert claim(m)[0] == 1


def test_forms_not_implemented_are_declined_with_reason():
    n = node(d=1024)
    ok, why = claim(n)
    assert ok == 0 and "head_size above 640" in why
    # the append prologue stages 4 bytes x head x (heads + 2 kv heads) per token for RoPE
    n = node(H=128, KV=1, d=512)
    n.do_rotary = 1
    tensor(n.inputs[8], F16, [4096, 32])
    tensor(n.inputs[9], F16, [4096, 32])
    n.num_inputs = 10
    ok, why = claim(n)
    assert ok == 0 and "prologue's shared memory" in why
    assert claim(latent_node(cache_dt=F8))[0] == 0  # encoded LATENT caches stay with ORT


def latent_node(H=2, d=16, vd=8, cache_dt=None, nb=3, bs=4, maxb=3):
    """The reference's LATENT case (test_paged_attention.py:669-764): one kv head, value and
    value_cache absent, v_head_size < head_size with an explicit scale."""
    n = node(H=H, KV=1, d=d, nb=nb, bs=bs, B=1, maxb=maxb, cache_dt=cache_dt)
    n.kv_cache_layout = b"LATENT"
    n.inputs[2].present = n.inputs[4].present = 0
    n.v_head_size = vd
    n.has_scale, n.scale = 1, 0.2
    tensor(n.outputs[0], F16, [-1, H * vd])
    if cache_dt == F8:
        n.k_cache_dtype = b"float8e4m3"
        tensor(n.inputs[14], F32, [nb, 1])
        n.num_inputs = 16
    return n


def test_latent_layout_is_claimed():
    assert claim(latent_node()) == (1, "")
    n = latent_node()
    n.do_rotary, n.rotary_offset = 1, 8
    tensor(n.inputs[8], F16, [12, 4])
    tensor(n.inputs[9], F16, [12, 4])
    n.num_inputs = 10
    assert claim(n) == (1, "")
    # MLA-like geometry: 576-channel keys, 512-channel values, 16 heads
    assert claim(latent_node(H=16, d=576, vd=512))[0] == 1


@pytest.mark.parametrize("mutate,reason", [
    (lambda n: setattr(n, "kv_num_heads", 2), "LATENT layout requires kv_num_heads=1"),
    (lambda n: setattr(n, "has_scale", 0), "asymmetric value heads requires an explicit scale"),
    (lambda n: setattr(n, "v_head_size", 32), "LATENT v_head_size must not exceed head_size"),
])
def test_latent_layout_rules(mutate, reason):
    n = latent_node()
    mutate(n)
    ok, why = claim(n)
    assert ok == 0 and reason in why, why
