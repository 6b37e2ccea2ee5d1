"""CPU restatement of the reference GroupQueryAttention op over a contiguous BNSH cache (numpy).

TEST INFRASTRUCTURE ONLY.  Imported by ``tests/`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py``; the product path (``onnxruntime_ep_b200``) never imports it.

Semantics:
* per batch row (rust/src/ops/attention.rs:662-667): ``length = seqlens_k[b] + 1``,
  ``query_past = max(length - S, 0)``, ``past = length if new_seq == 0 else query_past``,
  ``new_rows = length - past`` (0 when new_seq == 0);
* the cache the queries read is past rows ``[0, past)`` then the first ``new_rows`` new rows
  (attention.rs:688-711); ``present`` has ``max(cap, total)`` rows: those ``length`` rows, then
  the old buffer's rows ``[length, cap)``, then zeros (attention.rs:782-809);
* masks, softcap and sink exactly as the reference's own NumPy oracle
  ``_reference`` (tests/ops/test_gqa_position_cache.py:88-134): query row i sees keys
  ``[start, end)`` with ``end = min(past + i + 1, length)`` (causal) or ``length``, and
  ``start = max(0, end - window)`` for ``window > 0``; scores in fp32; softcap
  ``cap * tanh(s / cap)``; a sink joins only the softmax denominator;
* ``smooth_softmax == 1`` is a zero sink in every head (attention.rs:1311-1312);
* rotary embedding of the new query / key rows before K joins present, positions as
  gqa_rotary_rows (attention.rs:538-585) and the oracle's ``_rotate`` (:71-85);
* ``sliding_window_cache=1`` (attention.rs:1139-1379; the reference's integer oracle
  ``_gqa_ref(sliding=True)``, tests/ops/test_quantized_kv.py:122-193, and the inline expectation
  of test_gqa_position_cache.py:427-488): a length-``n`` sequence keeps ``resident(n)`` cache
  rows, ``n`` up to the capacity and otherwise ``n - gap * ceil((n - cap) / gap)`` with
  ``gap = cap - window + 1``; the queries read the ``resident(past)`` cache rows (absolute
  positions from ``past - resident(past)``) and the new rows, windowed on absolute positions,
  bias columns absolute; present (capacity ``cap``) holds the last ``resident(length)`` rows of
  the sequence, then zeros.

Parity pinning: ``tests/golden/make_gqa_golden.py`` runs the reference's ``_reference`` on
seeded inputs and commits its outputs (``gqa_golden.npz``); ``tests/test_gqa_oracle.py``
checks this module against them.
"""

from __future__ import annotations

import numpy as np


def rotate(x, cos, sin, positions, interleaved):
    """Rotary embedding of ``x [heads, seq, D]`` at ``positions [seq]`` over the first
    ``2 * cos.shape[1]`` channels, in fp32, rounded back to ``x.dtype``
    (tests/ops/test_gqa_position_cache.py:71-85)."""
    half = cos.shape[1]
    part = x[..., :2 * half].astype(np.float32)
    c, s = cos[positions].astype(np.float32), sin[positions].astype(np.float32)
    if interleaved:
        partner = np.empty_like(part)
        partner[..., 0::2], partner[..., 1::2] = -part[..., 1::2], part[..., 0::2]
        c, s = np.repeat(c, 2, -1), np.repeat(s, 2, -1)
    else:
        partner = np.concatenate([-part[..., half:], part[..., :half]], -1)
        c, s = np.tile(c, (1, 2)), np.tile(s, (1, 2))
    out = x.copy()
    out[..., :2 * half] = (part * c[None] + partner * s[None]).astype(x.dtype)
    return out


def rms_norm(x, weight, eps):
    """Per-head RMS norm of ``x [heads, seq, D]`` over D in fp32, ``x / sqrt(mean(x^2) + eps) * w``,
    rounded back to ``x.dtype`` (attention.rs:1070-1078; tests/ops/test_gqa11.py:52-130)."""
    xf = x.astype(np.float32)
    denom = np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + np.float32(eps))
    return (xf / denom * np.asarray(weight, np.float32)).astype(x.dtype)


def int_encode(x, scale, bits):
    """Integer cache codes of ``x [..., D]`` (test_quantized_kv.py:22-38 with paged = False):
    rint(x * (1 / scale)) clipped to the code range (scale 0 -> 1); int4 codes +8-biased, two
    per byte, the even channel in the low nibble."""
    x, scale = np.asarray(x, np.float32), np.asarray(scale, np.float32)
    inverse = np.divide(np.float32(1), scale, out=np.ones_like(scale), where=scale != 0)
    limit = 2 ** (bits - 1)
    codes = np.clip(np.rint(x * inverse), -limit, limit - 1).astype(np.int8)
    if bits == 8:
        return codes
    biased = (codes.astype(np.int16) + 8).astype(np.uint8)
    if x.shape[-1] % 2:
        biased = np.concatenate([biased, np.full((*biased.shape[:-1], 1), 8, np.uint8)], -1)
    return biased[..., ::2] | (biased[..., 1::2] << 4)


def int_decode(codes, scale, bits, head):
    """Cached values ``code * scale`` (test_quantized_kv.py:40-46)."""
    if bits == 4:
        values = np.stack([codes & 15, codes >> 4], -1).reshape(*codes.shape[:-1], codes.shape[-1] * 2)[..., :head]
        values = values.astype(np.float32) - 8
    else:
        values = codes.astype(np.float32)
    return values * np.asarray(scale, np.float32)


def rotary_positions(b, seq, query_past, total, position_ids):
    """Positions of batch row ``b``'s query rows (attention.rs:538-585): ``query_past + s``
    without ids; with ids, the first id as an offset on a first prompt (``total == seq``),
    else the flattened ids ``b * seq .. b * seq + seq``."""
    if position_ids is None:
        return query_past + np.arange(seq)
    ids = np.asarray(position_ids).reshape(-1)
    if total == seq:
        return int(ids[0]) + np.arange(seq)
    return ids[b * seq:(b + 1) * seq]


def sliding_resident(length, cap, window):
    """Cache rows a sliding-window cache of capacity ``cap`` keeps of a length-``length``
    sequence (attention.rs:1173-1181): all of them up to the capacity; beyond it whole gaps of
    ``cap - window + 1`` rows are reclaimed from the front."""
    if length <= cap:
        return length
    gap = cap - window + 1
    return length - gap * ((length - cap + gap - 1) // gap)


def group_query_attention(q, k, v, past_k, past_v, seqlens_k, total, *, num_heads, kv_num_heads,
                          scale=None, causal=True, window=-1, softcap=0.0, sink=None,
                          smooth_softmax=-1, cos=None, sin=None, position_ids=None, interleaved=False,
                          out_dtype=None, bias=None, q_norm=None, k_norm=None, norm_eps=1e-6, qk_output=0,
                          k_scale=None, v_scale=None, sliding=False):
    """Returns ``(output [B,S,H*D], present_k, present_v [B,KV,max(cap,total),D])``.

    ``q`` [B,S,H*D]; ``k``/``v`` [B,new_seq,KV*D] (new_seq may be 0); ``past_k``/``past_v``
    [B,KV,cap,D] or None; ``cos``/``sin`` [positions, rotary_dim/2] turn on the rotary
    embedding of the new query and key rows (``position_ids`` [B, >=S] optional).  ``bias``
    [1|B, 1|H, S, total] is added to the (soft-capped) scores of the visible keys
    (test_gqa_position_cache.py:119-121, attention.rs:746-755).  ``q_norm`` / ``k_norm``
    ``[D]`` RMS-normalise the query heads and new key heads before the rotary embedding.
    ``qk_output`` 1 / 2 also returns the diagnostics ``[B, H, S, total]``: the visible logits
    (0 elsewhere) / the probabilities, zero from each row's length on (test_gqa_position_cache.py:
    130-131, attention.rs:771-787).  int8 / uint8 (int4) ``past_k``/``past_v`` hold integer codes
    with ``k_scale`` / ``v_scale`` ``[1]`` or ``[KV, D]``: present is in the same storage, new rows
    are encoded, and the attention reads every row decoded (test_quantized_kv.py:122-193).
    ``sliding`` is sliding_window_cache=1 (``window`` > 0, new rows present, present of the
    past's capacity; ``qk_output`` 0), as ``sliding_resident`` describes.  Arrays keep
    their dtype; math is fp32, the output is rounded to the activation dtype (or kept in
    ``out_dtype``, e.g. fp32 for tolerance checks)."""
    B, S, hidden = q.shape
    H, KV = int(num_heads), int(kv_num_heads)
    D = hidden // H
    g = H // KV
    new_seq = 0 if k is None else k.shape[1]
    total = int(np.asarray(total).reshape(-1)[0])
    cap = 0 if past_k is None else past_k.shape[2]
    pcap = cap if sliding else max(cap, total)
    if sliding:
        assert window > 0 and new_seq == S and past_k is not None and window <= cap and not qk_output
    dt = q.dtype
    scale = 1.0 / np.sqrt(D) if not scale else float(scale)
    bits = 0
    if past_k is not None and past_k.dtype in (np.int8, np.uint8):
        bits = 8 if past_k.dtype == np.int8 else 4
        ksc, vsc = (np.asarray(x, np.float32) for x in (k_scale, v_scale))
        ksc, vsc = (x.reshape(KV, 1, D) if x.size > 1 else x.reshape(1) for x in (ksc, vsc))
        zero = 0 if bits == 8 else 0x88
        pk = np.full((B, KV, pcap, past_k.shape[3]), zero, past_k.dtype)
        pv = np.full((B, KV, pcap, past_k.shape[3]), zero, past_k.dtype)
    else:
        pk = np.zeros((B, KV, pcap, D), dt)
        pv = np.zeros((B, KV, pcap, D), dt)
    out = np.empty((B, S, H * D), out_dtype or dt)
    diag = np.zeros((B, H, S, total), out_dtype or dt)
    if sink is None and smooth_softmax == 1:
        sink = np.zeros(H, np.float32)
    for b in range(B):
        length = int(seqlens_k[b]) + 1
        query_past = max(length - S, 0)
        past = length if new_seq == 0 else query_past
        rows = 0 if new_seq == 0 else length - past
        if past_k is not None and not sliding:
            pk[b, :, :past] = past_k[b, :, :past]
            pv[b, :, :past] = past_v[b, :, :past]
            if length < cap:
                pk[b, :, length:cap] = past_k[b, :, length:cap]
                pv[b, :, length:cap] = past_v[b, :, length:cap]
        kb = None if not new_seq else k[b].reshape(new_seq, KV, D).transpose(1, 0, 2)  # [KV, new_seq, D]
        qb = q[b].reshape(S, H, D).transpose(1, 0, 2)                                      # [H, S, D]
        if q_norm is not None:
            qb = rms_norm(qb, q_norm, norm_eps)
            if new_seq:
                kb = rms_norm(kb, k_norm, norm_eps)
        if cos is not None:
            ids = rotary_positions(b, S, query_past, total, position_ids)
            qb = rotate(qb, cos, sin, ids, interleaved)
            if new_seq:
                kb = rotate(kb, cos, sin, ids, interleaved)
        newk = newv = None
        if rows:  # new rows in the cache's storage form
            vrows = v[b, :rows].reshape(rows, KV, D).transpose(1, 0, 2)
            newk = int_encode(kb[:, :rows], ksc, bits) if bits else kb[:, :rows]
            newv = int_encode(vrows, vsc, bits) if bits else vrows
        if sliding:  # resident past rows ++ new rows; present keeps the last resident(length)
            before, after = sliding_resident(past, cap, window), sliding_resident(length, cap, window)
            origin = past - before
            stored_k = np.concatenate([past_k[b, :, :before], newk.astype(past_k.dtype)], 1)
            stored_v = np.concatenate([past_v[b, :, :before], newv.astype(past_v.dtype)], 1)
            pk[b, :, :after] = stored_k[:, before + rows - after:]
            pv[b, :, :after] = stored_v[:, before + rows - after:]
        else:
            origin = 0
            if rows:
                pk[b, :, past:length] = newk
                pv[b, :, past:length] = newv
            stored_k, stored_v = pk[b, :, :length], pv[b, :, :length]
        n = stored_k.shape[1]  # keys at absolute positions origin .. origin + n - 1 (= length - 1)
        if bits:
            keys = np.repeat(int_decode(stored_k, ksc, bits, D), g, 0)
            vals = np.repeat(int_decode(stored_v, vsc, bits, D), g, 0)
        else:
            keys = np.repeat(stored_k.astype(np.float32), g, 0)   # [H, n, D]
            vals = np.repeat(stored_v.astype(np.float32), g, 0)
        qh = qb.astype(np.float32)  # [H, S, D]
        scores = qh @ keys.transpose(0, 2, 1) * np.float32(scale)
        if softcap > 0:
            scores = softcap * np.tanh(scores / softcap)
        if bias is not None:
            scores = scores + np.asarray(bias)[0 if bias.shape[0] == 1 else b, :, :, origin:length].astype(np.float32)
        end = np.minimum(query_past + np.arange(S) + 1, length) if causal else np.full(S, length)
        start = np.maximum(0, end - window) if window > 0 else np.zeros(S, int)
        cols = origin + np.arange(n)[None]
        visible = (cols >= start[:, None]) & (cols < end[:, None])
        logits = np.where(visible[None], scores, -np.inf)
        if sink is not None:
            s = np.asarray(sink, np.float32).reshape(H, 1, 1)
            logits = np.concatenate([logits, np.broadcast_to(s, (H, S, 1))], -1)
        e = np.exp(logits - logits.max(-1, keepdims=True))
        probs = (e / e.sum(-1, keepdims=True))[..., :n]
        if qk_output:
            diag[b, :, :, :length] = np.where(visible[None], scores, 0) if qk_output == 1 else probs
        out[b] = (probs @ vals).transpose(1, 0, 2).reshape(S, H * D).astype(out.dtype)
    return (out, pk, pv, diag) if qk_output else (out, pk, pv)
