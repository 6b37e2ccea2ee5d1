"""Python mirror of the com.microsoft PagedAttention node on the B200 kernels.

``paged_attention`` takes the node's inputs in the node's order, its attributes as keyword
arguments, and returns the node's outputs ``(output, key_cache, value_cache)``; the caches are
updated in place and returned aliased, which is the reference's in-place cache contract
(rust/src/engine.rs:1212-1364, outputs compared by pointer at :3174-3178).  Errors raise
``B200Error`` with the reference's messages (rust/src/ops/attention.rs:3934-3990).

Torch is only the plumbing here: it owns device memory and the current stream.  All work runs
in ``libb200_paged.so`` through its C ABI.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _capi
from ._capi import LIB, PagedAttentionParams, check

_DTYPES = {
    torch.float16: _capi.DTYPE_FLOAT16,
    torch.bfloat16: _capi.DTYPE_BFLOAT16,
    torch.int8: _capi.DTYPE_INT8,
    torch.uint8: _capi.DTYPE_UINT8,
    torch.float8_e4m3fn: _capi.DTYPE_FLOAT8E4M3FN,
}

_workspaces: dict[int, torch.Tensor] = {}


def _shared_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device scratch buffer, grown on demand (never shrunk)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _workspaces.get(idx)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[idx] = buf
    return buf


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _i32(t, device):
    """(device tensor, host tensor or None) for an int32 metadata input."""
    if t is None:
        return None, None
    t = torch.as_tensor(t)
    if t.dtype != torch.int32:
        raise _capi.B200Error(_capi.B200_ERR_INVALID_ARGUMENT, "PagedAttention: metadata inputs must be int32")
    if t.device.type == "cpu":
        host = t.contiguous()
        return host.to(device, non_blocking=True), host
    return t.contiguous(), None


def build_params(query, key, value, key_cache, value_cache, cum, past, block_table, *, num_heads,
                 kv_num_heads, cos_cache=None, sin_cache=None, slot_mapping=None, head_sink=None,
                 q_norm_weight=None, k_norm_weight=None, k_scale=None, v_scale=None, scale=0.0,
                 is_causal=1, local_window_size=-1, softcap=0.0, do_rotary=0, rotary_interleaved=0,
                 rotary_offset=0, qk_norm_epsilon=1e-6, k_quant_type="NONE", v_quant_type="NONE",
                 output=None, host_metadata=None, min_tiles_per_warp=0, force_generic=False,
                 kv_only=False, kv_cache_layout="SEPARATE", v_head_size=0, workspace=None):
    """Fill a ``B200PagedAttentionParams``.  Returns ``(params, keepalive, output)``.

    The scratch is this device's shared buffer unless ``workspace`` (a uint8 CUDA tensor of at
    least ``b200_paged_attention_workspace_size`` bytes) is given.  Params built on the shared
    buffer must be used in one stream order: calls that may overlap on the GPU need private
    workspaces.  The keepalive holds the buffer, so a later, larger build does not free it.

    ``kv_cache_layout="LATENT"``: one kv head, ``value`` and ``value_cache`` are ``None``, and the
    values are the first ``v_head_size`` channels of the key rows (output ``[nt, H*v_head_size]``)."""
    device = key_cache.device
    H, KV = int(num_heads), int(kv_num_heads)
    keep = []
    latent = kv_cache_layout == "LATENT"
    packed = key is None and value is None and not latent
    if query is None:
        raise _capi.B200Error(_capi.B200_ERR_INVALID_ARGUMENT, "PagedAttention: query is required")
    nt = query.shape[0]
    hidden = query.shape[1]
    d = hidden // (H + 2 * KV) if packed else hidden // H
    act = _DTYPES.get(query.dtype)
    if act not in (_capi.DTYPE_FLOAT16, _capi.DTYPE_BFLOAT16):
        raise _capi.B200Error(_capi.B200_ERR_INVALID_ARGUMENT, "PagedAttention is only supported for fp16/bf16 (T)")
    p = PagedAttentionParams()
    p.num_heads, p.kv_num_heads, p.head_size = H, KV, d
    p.scale = float(scale or 0.0)
    p.is_causal = int(is_causal)
    p.local_window_size = int(local_window_size)
    p.softcap = float(softcap)
    p.act_dtype = act
    p.cache_dtype = _DTYPES[key_cache.dtype]
    p.k_quant_per_channel = int(k_quant_type == "PER_CHANNEL")
    p.v_quant_per_channel = int(v_quant_type == "PER_CHANNEL")
    p.num_tokens = nt
    p.num_blocks, p.block_size = key_cache.shape[0], key_cache.shape[1]
    if query.stride(1) != 1:
        raise _capi.B200Error(_capi.B200_ERR_INVALID_ARGUMENT, "PagedAttention: query rows must be contiguous")
    p.query_row_stride = query.stride(0)
    p.query = _ptr(query)
    if packed:
        esz = query.element_size()
        p.key = ctypes.c_void_p(query.data_ptr() + H * d * esz)
        p.value = ctypes.c_void_p(query.data_ptr() + (H + KV) * d * esz)
        p.key_row_stride = p.value_row_stride = query.stride(0)
    else:
        p.key, p.value = _ptr(key), _ptr(value)
        p.key_row_stride = key.stride(0)
        p.value_row_stride = value.stride(0) if value is not None else 0
    p.key_cache, p.value_cache = _ptr(key_cache), _ptr(value_cache)
    dv = d
    if latent:
        p.kv_cache_latent = 1
        p.v_head_size = int(v_head_size)
        dv = int(v_head_size) or d

    cum_d, cum_h = _i32(cum, device)
    past_d, past_h = _i32(past, device)
    bt_d, bt_h = _i32(block_table, device)
    sm_d, sm_h = _i32(slot_mapping, device)
    keep += [cum_d, past_d, bt_d, sm_d]
    if host_metadata is not None:  # caller-provided host copies of device metadata
        cum_h = torch.as_tensor(host_metadata["cumulative_sequence_length"], dtype=torch.int32)
        past_h = torch.as_tensor(host_metadata["past_seqlens"], dtype=torch.int32)
        bt_h = torch.as_tensor(host_metadata["block_table"], dtype=torch.int32)
        if sm_d is not None and host_metadata.get("slot_mapping") is not None:
            sm_h = torch.as_tensor(host_metadata["slot_mapping"], dtype=torch.int32)
    if bt_d.dim() != 2:
        raise _capi.B200Error(_capi.B200_ERR_FAIL,
                              "PagedAttention: inconsistent cumulative lengths, past lengths or block table")
    p.batch = cum_d.shape[0] - 1
    p.max_blocks_per_seq = bt_d.shape[1]
    if bt_d.shape[0] != p.batch or past_d.shape[0] != p.batch:
        raise _capi.B200Error(_capi.B200_ERR_FAIL,
                              "PagedAttention: inconsistent cumulative lengths, past lengths or block table")
    if sm_d is not None and sm_d.shape[0] != nt:
        raise _capi.B200Error(_capi.B200_ERR_FAIL,
                              "PagedAttention: slot_mapping must contain -1 or valid physical cache slots")
    p.cumulative_sequence_length, p.past_seqlens = _ptr(cum_d), _ptr(past_d)
    p.block_table, p.slot_mapping = _ptr(bt_d), _ptr(sm_d)
    if cum_h is not None and past_h is not None and bt_h is not None:
        cum_h, past_h, bt_h = cum_h.contiguous(), past_h.contiguous(), bt_h.contiguous()
        keep += [cum_h, past_h, bt_h]
        p.host_cumulative_sequence_length = _ptr(cum_h)
        p.host_past_seqlens = _ptr(past_h)
        p.host_block_table = _ptr(bt_h)
        if sm_h is not None:
            sm_h = sm_h.contiguous()
            keep.append(sm_h)
            p.host_slot_mapping = _ptr(sm_h)

    if do_rotary:
        p.do_rotary = 1
        p.rotary_interleaved = int(rotary_interleaved)
        p.rotary_offset = int(rotary_offset)
        p.rotary_dim = cos_cache.shape[1] * 2
        p.rotary_positions = cos_cache.shape[0]
        p.cos_cache, p.sin_cache = _ptr(cos_cache), _ptr(sin_cache)
    p.head_sink = _ptr(head_sink)
    if q_norm_weight is not None:
        p.q_norm_weight, p.k_norm_weight = _ptr(q_norm_weight), _ptr(k_norm_weight)
        p.qk_norm_epsilon = float(qk_norm_epsilon)
    if k_scale is not None:
        p.k_scale, p.v_scale = _ptr(k_scale), _ptr(v_scale)
    if not kv_only:
        if output is None:
            output = torch.empty((nt, H * dv), dtype=query.dtype, device=device)
        p.output = _ptr(output)
    p.decode_min_tiles_per_warp = int(min_tiles_per_warp)
    p.force_generic = int(bool(force_generic))
    nbytes = ctypes.c_size_t(0)
    check(LIB.b200_paged_attention_workspace_size(ctypes.byref(p), ctypes.byref(nbytes)))
    if workspace is None:
        ws = _shared_workspace(device, nbytes.value)
    else:
        ws = workspace
        if ws.dtype != torch.uint8 or ws.device != device or not ws.is_contiguous() or ws.numel() < nbytes.value:
            raise _capi.B200Error(_capi.B200_ERR_WORKSPACE,
                                  "PagedAttention: workspace must be a contiguous uint8 tensor on the caches' "
                                  f"device of at least {nbytes.value} bytes")
    keep.append(ws)
    p.workspace = _ptr(ws)
    p.workspace_bytes = ws.numel()
    return p, keep, output


def paged_attention(query, key, value, key_cache, value_cache, cumulative_sequence_length,
                    past_seqlens, block_table, cos_cache=None, sin_cache=None, slot_mapping=None,
                    head_sink=None, q_norm_weight=None, k_norm_weight=None, k_scale=None,
                    v_scale=None, *, num_heads, kv_num_heads, check_status=False, stream=None,
                    **attrs):
    """Run one PagedAttention node on the current CUDA stream.

    Inputs follow the node's input order (0-15).  ``key``/``value`` ``None`` means packed QKV.
    Returns ``(output, key_cache, value_cache)``.  ``check_status=True`` synchronises and
    raises on device-side metadata errors (the reference reports those eagerly).
    """
    p, keep, out = build_params(
        query, key, value, key_cache, value_cache, cumulative_sequence_length, past_seqlens,
        block_table, num_heads=num_heads, kv_num_heads=kv_num_heads, cos_cache=cos_cache,
        sin_cache=sin_cache, slot_mapping=slot_mapping, head_sink=head_sink,
        q_norm_weight=q_norm_weight, k_norm_weight=k_norm_weight, k_scale=k_scale, v_scale=v_scale,
        **attrs)
    s = stream if stream is not None else torch.cuda.current_stream(key_cache.device)
    check(LIB.b200_paged_attention(ctypes.byref(p), ctypes.c_void_p(s.cuda_stream)))
    if check_status:
        check(LIB.b200_read_status(ctypes.byref(p), ctypes.c_void_p(s.cuda_stream)))
    del keep
    return out, key_cache, value_cache


def kv_append(key, value, key_cache, value_cache, cumulative_sequence_length, past_seqlens,
              block_table, slot_mapping=None, *, kv_num_heads, k_scale=None, v_scale=None,
              check_status=False, stream=None, **attrs):
    """Reshape-and-cache alone: scatter new K/V rows into the paged caches (in place)."""
    KV = int(kv_num_heads)
    d = key.shape[1] // KV
    # The query is not read on this path; the key tensor stands in for its geometry.
    fake_q = key
    p, keep, _ = build_params(
        fake_q, key, value, key_cache, value_cache, cumulative_sequence_length, past_seqlens,
        block_table, num_heads=KV, kv_num_heads=KV, slot_mapping=slot_mapping, k_scale=k_scale,
        v_scale=v_scale, kv_only=True, **attrs)
    p.head_size = d
    s = stream if stream is not None else torch.cuda.current_stream(key_cache.device)
    check(LIB.b200_kv_append(ctypes.byref(p), ctypes.c_void_p(s.cuda_stream)))
    if check_status:
        check(LIB.b200_read_status(ctypes.byref(p), ctypes.c_void_p(s.cuda_stream)))
    del keep
    return key_cache, value_cache


def default_scale(head_size: int) -> float:
    return 1.0 / math.sqrt(head_size)
