"""com.microsoft.GroupQueryAttention on B200 over a contiguous BNSH cache.

Mirror of the node's inputs, attributes and outputs (reference op
rust/src/ops/attention.rs:932-1454, per-batch form :586-848, claim :2407-2754):

    output, present_key, present_value = group_query_attention(
        query, key, value, past_key, past_value, seqlens_k, total_sequence_length,
        head_sink=None, num_heads=..., kv_num_heads=..., ...)

``present`` follows the reference's contracts: by default a new ``[B, KV, max(cap, total), D]``
buffer (growing: past rows, then the new rows); passing ``present_key=past_key,
present_value=past_value`` writes the new rows in place (shared buffer).
``sliding_window_cache=1`` keeps the past's capacity and moves resident rows down as the
window slides (attention.rs:1139-1379).  Errors raise
``B200Error`` with the reference's messages.  There is no CPU fallback.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _capi
from ._capi import (DTYPE_BFLOAT16, DTYPE_FLOAT, DTYPE_FLOAT16, LIB, GqaParams, check)

_DTYPES = {torch.float32: DTYPE_FLOAT, torch.float16: DTYPE_FLOAT16, torch.bfloat16: DTYPE_BFLOAT16}
_workspaces: dict = {}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _workspace(device, nbytes):
    buf = _workspaces.get(device)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[device] = buf
    return buf


def build_params(query, key, value, past_key, past_value, seqlens_k, total_sequence_length,
                 head_sink=None, *, num_heads, kv_num_heads, scale=0.0, causal=1,
                 local_window_size=-1, softcap=0.0, smooth_softmax=-1, present_key=None,
                 present_value=None, with_present=True, host_seqlens_k=None, output=None,
                 do_rotary=0, rotary_interleaved=0, cos_cache=None, sin_cache=None, position_ids=None,
                 attention_bias=None, q_norm_weight=None, k_norm_weight=None, qk_norm_epsilon=1e-6,
                 qk_output=0, output_qk=None, k_scale=None, v_scale=None, k_quant_type="NONE",
                 v_quant_type="NONE", sliding_window_cache=0):
    """Fill a ``B200GqaParams``.  Returns ``(params, keepalive, output, present_key, present_value)``.

    ``do_rotary=1`` takes ``cos_cache``/``sin_cache`` ``[positions, rotary_dim/2]`` (inputs 7 and
    8) and optionally ``position_ids`` int64 ``[batch, >=seq]`` (input 9; a host copy is made for
    the reference's bounds checks).  ``attention_bias`` ``[1|batch, 1|heads, seq, total]`` (input
    10, the activation dtype) is added to the scores of the visible keys.  ``q_norm_weight`` /
    ``k_norm_weight`` ``[head_size]`` (inputs 14 / 15) RMS-normalise every query head and new key
    head before the rotary embedding.  ``qk_output`` 1 / 2 fills ``output_qk`` ``[batch, heads,
    seq, total]`` (allocated when not given) with the visible logits / the probabilities.  int8 /
    uint8 (int4) ``past_key``/``past_value`` select the integer caches, with ``k_scale`` /
    ``v_scale`` fp32 (inputs 12 / 13) and ``k_quant_type`` / ``v_quant_type`` PER_TENSOR or
    PER_CHANNEL; present is allocated in the same storage.  ``sliding_window_cache=1`` keeps a
    sliding-window cache of the past's capacity (present has ``cap`` rows: the last
    ``resident(length)`` rows of each sequence, then zeros; it may be the past buffer)."""
    H, KV = int(num_heads), int(kv_num_heads)
    packed = key is None and value is None  # packed QKV in query (inputs 1 and 2 absent)
    B, S = int(query.shape[0]), int(query.shape[1])
    if packed:
        D = query.shape[2] // (H + 2 * KV)
        new_seq = S
    else:
        D = query.shape[2] // H
        new_seq = int(key.shape[1]) if key is not None else 0
    if isinstance(total_sequence_length, torch.Tensor):
        total = int(total_sequence_length.reshape(-1)[0].item())
    else:
        total = int(np.asarray(total_sequence_length).reshape(-1)[0])
    cap = int(past_key.shape[2]) if past_key is not None else 0
    if host_seqlens_k is None:
        host_seqlens_k = seqlens_k.detach().to("cpu", torch.int32).numpy()
    host_seqlens_k = np.ascontiguousarray(np.asarray(host_seqlens_k, dtype=np.int32))
    dev = query.device
    pcap = cap if sliding_window_cache else max(cap, total)
    int_cache = past_key is not None and past_key.dtype in (torch.int8, torch.uint8)
    if with_present and present_key is None:
        if int_cache:
            width = D if past_key.dtype == torch.int8 else (D + 1) // 2
            present_key = torch.empty((B, KV, pcap, width), dtype=past_key.dtype, device=dev)
        else:
            present_key = torch.empty((B, KV, pcap, D), dtype=query.dtype, device=dev)
        present_value = torch.empty_like(present_key)
    if present_key is not None:
        pcap = int(present_key.shape[2])
    if output is None:
        output = torch.empty((B, S, H * D), dtype=query.dtype, device=dev)
    p = GqaParams()
    p.num_heads, p.kv_num_heads, p.head_size = H, KV, D
    p.scale = float(scale)
    p.is_causal = int(causal)
    p.local_window_size = int(local_window_size)
    p.softcap = float(softcap)
    p.smooth_softmax = int(smooth_softmax)
    p.dtype = _DTYPES[query.dtype]
    p.batch, p.seq, p.new_seq, p.cap = B, S, new_seq, cap
    p.present_cap = pcap if present_key is not None else 0
    p.total_sequence_length = total
    p.sliding_window_cache = int(bool(sliding_window_cache))
    p.query = _ptr(query)
    if packed:
        row = (H + 2 * KV) * D
        p.query_row_stride = p.key_row_stride = p.value_row_stride = row
        esz = query.element_size()
        p.key = ctypes.c_void_p(query.data_ptr() + H * D * esz)
        p.value = ctypes.c_void_p(query.data_ptr() + (H + KV) * D * esz)
    else:
        p.key, p.value = _ptr(key), _ptr(value)
    p.past_key, p.past_value = _ptr(past_key), _ptr(past_value)
    p.present_key, p.present_value = _ptr(present_key), _ptr(present_value)
    p.seqlens_k = _ptr(seqlens_k)
    p.host_seqlens_k = host_seqlens_k.ctypes.data_as(ctypes.c_void_p)
    p.head_sink = _ptr(head_sink)
    p.output = _ptr(output)
    host_ids = None
    if do_rotary:
        p.do_rotary = 1
        p.rotary_interleaved = int(rotary_interleaved)
        p.rotary_dim = int(cos_cache.shape[1]) * 2
        p.rotary_positions = int(cos_cache.shape[0])
        p.cos_cache, p.sin_cache = _ptr(cos_cache), _ptr(sin_cache)
        if position_ids is not None:
            ids = torch.as_tensor(position_ids)
            host_ids = np.ascontiguousarray(ids.detach().to("cpu", torch.int64).numpy())
            if ids.device.type != "cuda":
                ids = ids.to(dev)
            position_ids = ids.contiguous()
            p.position_ids = _ptr(position_ids)
            p.host_position_ids = host_ids.ctypes.data_as(ctypes.c_void_p)
            p.position_ids_width = int(host_ids.shape[1]) if host_ids.ndim == 2 else int(host_ids.size)
    if attention_bias is not None:
        if attention_bias.device.type != "cuda":
            attention_bias = attention_bias.to(dev)
        attention_bias = attention_bias.contiguous()
        if attention_bias.dim() != 4:
            raise _capi.B200Error(_capi.B200_ERR_FAIL,
                                  "GroupQueryAttention: attention_bias must broadcast to [batch,heads,sequence,total]")
        p.attention_bias = _ptr(attention_bias)
        p.bias_batch, p.bias_heads, p.bias_seq, p.bias_total = (int(x) for x in attention_bias.shape)
    if q_norm_weight is not None:
        p.q_norm_weight, p.k_norm_weight = _ptr(q_norm_weight), _ptr(k_norm_weight)
        p.qk_norm_epsilon = float(qk_norm_epsilon)
    if int_cache:
        p.cache_dtype = _capi.DTYPE_INT8 if past_key.dtype == torch.int8 else _capi.DTYPE_UINT8
        k_scale = torch.as_tensor(k_scale, dtype=torch.float32).to(dev).contiguous()
        v_scale = torch.as_tensor(v_scale, dtype=torch.float32).to(dev).contiguous()
        p.k_scale, p.v_scale = _ptr(k_scale), _ptr(v_scale)
        p.k_quant_per_channel = int(k_quant_type == "PER_CHANNEL")
        p.v_quant_per_channel = int(v_quant_type == "PER_CHANNEL")
    if qk_output:
        if output_qk is None:
            output_qk = torch.empty((B, H, S, total), dtype=query.dtype, device=dev)
        p.qk_output, p.output_qk = int(qk_output), _ptr(output_qk)
    nbytes = ctypes.c_size_t(0)
    check(LIB.b200_group_query_attention_workspace_size(ctypes.byref(p), ctypes.byref(nbytes)))
    ws = _workspace(dev, nbytes.value)
    p.workspace = _ptr(ws)
    p.workspace_bytes = ws.numel()
    keep = (query, key, value, past_key, past_value, seqlens_k, head_sink, host_seqlens_k, ws, cos_cache, sin_cache,
            position_ids, host_ids, attention_bias, q_norm_weight, k_norm_weight, k_scale, v_scale, output_qk)
    return p, keep, output, present_key, present_value


def group_query_attention(query, key, value, past_key, past_value, seqlens_k, total_sequence_length,
                          head_sink=None, *, stream=None, check_status=False, **kwargs):
    """One GroupQueryAttention node.  Returns ``(output, present_key, present_value)``, plus
    ``output_qk`` when ``qk_output`` is 1 or 2.

    ``check_status=True`` synchronises and raises ``B200Error`` when a bounded device wait of
    the call ran out."""
    p, keep, out, pk, pv = build_params(query, key, value, past_key, past_value, seqlens_k,
                                        total_sequence_length, head_sink, **kwargs)
    qk = keep[-1]
    s = stream if stream is not None else torch.cuda.current_stream(query.device)
    check(LIB.b200_group_query_attention(ctypes.byref(p), ctypes.c_void_p(s.cuda_stream)))
    if check_status:
        check(LIB.b200_group_query_attention_read_status(ctypes.byref(p), ctypes.c_void_p(s.cuda_stream)))
    del keep
    return (out, pk, pv) if qk is None else (out, pk, pv, qk)
