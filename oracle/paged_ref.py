"""CPU restatement of the reference PagedAttention path (numpy).

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path is compared
against; it is imported by ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline``
leg of ``bench.py`` and by nothing else.  The product path (``onnxruntime_ep_b200``) never
imports it and has no CPU fallback.

Semantics follow the reference operator ``paged_attention_op``
(rust/src/ops/attention.rs:3857-4382) and the reference's own numpy oracles:

* tests/ops/test_paged_attention.py:27-58   rotate-half / interleaved RoPE, rotary offset
* tests/ops/test_paged_attention.py:63-158  ``_paged_ref`` (slot write, block-table gather,
  GQA head repeat, fp32 scores, softcap, causal/window masks, sink denominator)
* tests/ops/test_quantized_kv.py:22-47      int8 / int4 cache byte equations
* tests/ops/test_quantized_kv.py:395-450    quantized paged reference

One ordering rule comes from the operator, not from ``_paged_ref``: every KV write of the
whole batch is applied (in token order) before any sequence reads the cache
(attention.rs:4021-4122 builds all scatters, then :4124-4320 reads).  Positions ``>= past``
of a sequence read the sequence's own new rows (attention.rs:4253 ``concat2(gk, kh_new)``),
positions ``< past`` read the updated cache.  Integer caches read every position, the new
ones included, from the decoded cache (attention.rs:4190-4192).  ``_paged_ref`` applies the
writes sequence by sequence; the two agree whenever sequences do not share cache slots,
which holds for every golden case.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference's own ``_paged_ref``,
``_encode``/``_decode`` and quantized ``_paged_ref`` (loaded from the reference test files)
on seeded inputs and commits their outputs; ``tests/test_oracle_golden.py`` checks this
module against them.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

try:  # bf16 / fp8 host types
    import ml_dtypes

    BF16 = np.dtype(ml_dtypes.bfloat16)
    FP8E4M3 = np.dtype(ml_dtypes.float8_e4m3fn)
except Exception:  # pragma: no cover - ml_dtypes ships with the image
    ml_dtypes = None
    BF16 = None
    FP8E4M3 = None


# ----------------------------------------------------------------------------------------
# RoPE and RMS norm (test_paged_attention.py:27-58, attention.rs:3812-3855, :4045-4057)
# ----------------------------------------------------------------------------------------
def rotate_half(x: np.ndarray, interleaved: bool) -> np.ndarray:
    """Rotate-half (NeoX) or interleaved (GPT-J) partner, test_paged_attention.py:27-34."""
    if not interleaved:
        half = x.shape[-1] // 2
        return np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    out = np.empty_like(x)
    out[..., 0::2] = -x[..., 1::2]
    out[..., 1::2] = x[..., 0::2]
    return out


def apply_rope(x, cos, sin, pos, interleaved: bool, offset: int = 0):
    """RoPE of ``x [seq, heads, d]`` at absolute positions ``pos`` over dims
    ``[offset, offset + 2*cos.shape[1])`` (test_paged_attention.py:37-58)."""
    width = cos.shape[-1] * 2
    c, s = cos[pos], sin[pos]
    if not interleaved:
        c = np.concatenate([c, c], axis=-1)
        s = np.concatenate([s, s], axis=-1)
    else:
        c = np.repeat(c, 2, axis=-1)
        s = np.repeat(s, 2, axis=-1)
    out = x.copy()
    part = x[..., offset:offset + width]
    out[..., offset:offset + width] = part * c[:, None, :] + rotate_half(part, interleaved) * s[:, None, :]
    return out


def rms_norm(x, weight, eps):
    """Per-head RMS norm (test_paged_attention.py:101-103, attention.rs:4045-4049)."""
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * weight


# ----------------------------------------------------------------------------------------
# Integer KV codec (kv_cache.rs:170-256, test_quantized_kv.py:22-47)
# ----------------------------------------------------------------------------------------
def quant_encode(x, scale, bits: int, paged: bool = True) -> np.ndarray:
    """Encode fp32 rows ``x [..., d]`` to int8 (``bits=8``) or +8-biased nibbles (``bits=4``,
    even channel in the low nibble, pad nibble 8).  Paged divides and maps a zero scale to a
    zero code (kv_cache.rs:180-188); GQA multiplies by the reciprocal, zero -> 1."""
    x = np.asarray(x, np.float32)
    scale = np.asarray(scale, np.float32)
    shape = np.broadcast_shapes(x.shape, scale.shape)
    if paged:
        scaled = np.divide(x, scale, out=np.zeros(shape, np.float32), where=scale != 0)
    else:
        inverse = np.divide(np.float32(1), scale, out=np.ones_like(scale), where=scale != 0)
        scaled = x * inverse
    limit = 2 ** (bits - 1)
    codes = np.clip(np.rint(scaled), -limit, limit - 1).astype(np.int8)
    if bits == 8:
        return codes
    biased = (codes.astype(np.int16) + 8).astype(np.uint8)
    if biased.shape[-1] % 2:
        biased = np.concatenate([biased, np.full((*biased.shape[:-1], 1), 8, np.uint8)], -1)
    return (biased[..., 0::2] | (biased[..., 1::2] << 4)).astype(np.uint8)


def quant_decode(codes, scale, bits: int, head: int) -> np.ndarray:
    """Inverse of :func:`quant_encode` (kv_cache.rs:222-256)."""
    if bits == 4:
        lo = codes & 15
        hi = codes >> 4
        values = np.stack([lo, hi], -1).reshape(*codes.shape[:-1], codes.shape[-1] * 2)[..., :head]
        values = values.astype(np.float32) - 8
    else:
        values = codes.astype(np.float32)
    return values * np.asarray(scale, np.float32)


def fp8_encode(x, scale):
    """fp8 e4m3 (fn) encode of ``x / scale`` (round to nearest even, saturating to +-448).
    Extension outside the reference contract: per-block-per-head fp32 scale."""
    y = np.asarray(x, np.float32) / np.asarray(scale, np.float32)
    y = np.clip(y, -448.0, 448.0)
    return y.astype(FP8E4M3)


def fp8_decode(codes, scale):
    return codes.astype(np.float32) * np.asarray(scale, np.float32)


# ----------------------------------------------------------------------------------------
# Storage helpers
# ----------------------------------------------------------------------------------------
def to_f32(a) -> np.ndarray:
    return np.asarray(a).astype(np.float32)


def round_to(a: np.ndarray, dtype) -> np.ndarray:
    """Round fp32 to the cache storage dtype (round to nearest even)."""
    return np.asarray(a, np.float32).astype(dtype)


@dataclass
class QuantSpec:
    """Integer cache description: ``bits`` 8 or 4, ``scale`` fp32 ``[1]`` (PER_TENSOR) or
    ``[kv*head]`` (PER_CHANNEL), kv_cache.rs:119-168."""

    bits: int
    scale: np.ndarray

    def scale_view(self, kv: int, head: int):
        s = np.asarray(self.scale, np.float32)
        return s.reshape(kv, head) if s.size > 1 else s.reshape(())


# ----------------------------------------------------------------------------------------
# Slot computation and KV append (attention.rs:4064-4120)
# ----------------------------------------------------------------------------------------
def write_slots(cum, past, block_table, slot_mapping, block_size):
    """List of ``(token, slot)`` pairs in token order; ``slot < 0`` rows are skipped
    (attention.rs:4064-4079)."""
    out = []
    batch = len(cum) - 1
    for b in range(batch):
        s0, s1 = int(cum[b]), int(cum[b + 1])
        for j in range(s1 - s0):
            token = s0 + j
            if slot_mapping is not None:
                slot = int(slot_mapping[token])
            else:
                logical = int(past[b]) + j
                slot = int(block_table[b, logical // block_size]) * block_size + logical % block_size
            if slot >= 0:
                out.append((token, slot))
    return out


def kv_append(key_cache, value_cache, k_rows, v_rows, pairs, kquant=None, vquant=None):
    """Scatter ``k_rows[token]`` / ``v_rows[token]`` (fp32 ``[nt, kv, d]``) into the caches
    ``[NB, bs, kv, d']`` at each ``slot``; later tokens overwrite earlier ones (token order,
    as the reference's per-sequence scatter sequence applies them).  In place."""
    bs = key_cache.shape[1]
    kv = key_cache.shape[2]
    for token, slot in pairs:
        blk, off = divmod(slot, bs)
        for cache, rows, quant in ((key_cache, k_rows, kquant), (value_cache, v_rows, vquant)):
            if cache is None:
                continue
            row = rows[token]
            if quant is not None:
                cache[blk, off] = quant_encode(row, quant.scale_view(kv, row.shape[-1]), quant.bits, paged=True)
            else:
                cache[blk, off] = round_to(row, cache.dtype)


# ----------------------------------------------------------------------------------------
# Attention core (test_paged_attention.py:119-157)
# ----------------------------------------------------------------------------------------
def attend(qh, keys, vals, past, *, scale, is_causal=True, local_window_size=-1,
           softcap=0.0, head_sink=None):
    """``qh [nq, H, d]``, ``keys/vals [total, KV, d]`` (fp32) -> ``[nq, H, dv]`` fp32."""
    nq, H, _ = qh.shape
    total, KV, _ = keys.shape
    g = H // KV
    kh = np.repeat(keys, g, 1).transpose(1, 0, 2)
    vh = np.repeat(vals, g, 1).transpose(1, 0, 2)
    scores = np.einsum("hqd,hkd->hqk", qh.transpose(1, 0, 2), kh) * np.float32(scale)
    if softcap > 0:
        scores = softcap * np.tanh(scores / softcap)
    col = np.arange(total)[None, :]
    row = (past + np.arange(nq))[:, None]
    if is_causal:
        scores = np.where((col > row)[None], -np.inf, scores)
    if local_window_size > 0:
        scores = np.where((col < row - local_window_size + 1)[None], -np.inf, scores)
    if head_sink is None:
        mx = scores.max(-1, keepdims=True)
        e = np.exp(scores - mx)
        attn = e / e.sum(-1, keepdims=True)
    else:
        sink = np.asarray(head_sink, np.float32)[:, None, None]
        mx = np.maximum(scores.max(-1, keepdims=True), sink)
        e = np.exp(scores - mx)
        attn = e / (e.sum(-1, keepdims=True) + np.exp(sink - mx))
    return np.einsum("hqk,hkd->hqd", attn, vh).transpose(1, 0, 2)


# ----------------------------------------------------------------------------------------
# Whole node (attention.rs:3857-4382)
# ----------------------------------------------------------------------------------------
def paged_attention(q, k, v, key_cache, value_cache, cum, past, block_table,
                    num_heads, kv_num_heads, *, slot_mapping=None, scale=None,
                    is_causal=True, local_window_size=-1, softcap=0.0, head_sink=None,
                    cos=None, sin=None, interleaved=False, rotary_offset=0,
                    q_norm=None, k_norm=None, norm_eps=1e-6,
                    kquant: QuantSpec | None = None, vquant: QuantSpec | None = None,
                    fp8_scales=None, head_size=None, round_activations=True, latent_v_head=None):
    """Reference PagedAttention forward.

    Returns ``(output fp32 [nt, H*d], key_cache', value_cache')``; the caches are copies
    updated exactly as the reference updates its input buffers (bit-exact contract).
    ``k``/``v`` ``None`` means packed QKV in ``q`` (attention.rs:3877-3890).
    ``fp8_scales`` (fp32 ``[NB, KV]``, or a ``(k_scales, v_scales)`` pair) selects the
    fp8-e4m3 per-block-per-head extension.
    ``round_activations`` rounds the normalised / rotated Q and K rows back to the activation
    dtype after each step, as the reference's MLX ops do (their outputs carry dtype T); the
    reference test oracle keeps them in fp32, which differs only within tolerance.
    ``latent_v_head`` selects the LATENT layout (attention.rs:4058-4062, :4210-4212,
    test_paged_attention.py:669-764): one kv head, ``v``/``value_cache`` ``None``, and every
    value row is the first ``latent_v_head`` channels of the (rotated / normalised) key row.
    """
    H, KV = int(num_heads), int(kv_num_heads)
    q = np.asarray(q)
    if k is None and v is None:
        d = q.shape[1] // (H + 2 * KV)
        q, k, v = q[:, :H * d], q[:, H * d:(H + KV) * d], q[:, (H + KV) * d:]
    d = head_size or q.shape[1] // H
    nt = q.shape[0]
    batch = len(cum) - 1
    bs = key_cache.shape[1]
    sc = np.float32(scale) if scale not in (None, 0, 0.0) else np.float32(1.0 / math.sqrt(d))
    kc = key_cache.copy()
    vc = value_cache.copy() if value_cache is not None else None

    act = np.asarray(q).dtype
    rnd = (lambda a: a.astype(act).astype(np.float32)) if (round_activations and act != np.float32) else (lambda a: a)
    qf = to_f32(q).reshape(nt, H, d)
    kf = to_f32(k).reshape(nt, KV, d)
    vf = to_f32(v).reshape(nt, KV, -1) if latent_v_head is None else None
    if q_norm is not None:
        qf = rnd(rms_norm(qf, to_f32(q_norm), np.float32(norm_eps)).astype(np.float32))
        kf = rnd(rms_norm(kf, to_f32(k_norm), np.float32(norm_eps)).astype(np.float32))
    if cos is not None:
        cosf, sinf = to_f32(cos), to_f32(sin)
        for b in range(batch):
            s0, s1 = int(cum[b]), int(cum[b + 1])
            if s1 == s0:
                continue
            pos = np.arange(int(past[b]), int(past[b]) + s1 - s0)
            qf[s0:s1] = rnd(apply_rope(qf[s0:s1], cosf, sinf, pos, interleaved, rotary_offset))
            kf[s0:s1] = rnd(apply_rope(kf[s0:s1], cosf, sinf, pos, interleaved, rotary_offset))
    if latent_v_head is not None:
        vf = kf[:, :, :int(latent_v_head)]

    pairs = write_slots(cum, past, block_table, slot_mapping, bs)
    if fp8_scales is not None:
        k8, v8 = fp8_scales if isinstance(fp8_scales, tuple) else (fp8_scales, fp8_scales)
        k8, v8 = np.asarray(k8, np.float32), np.asarray(v8, np.float32)
        for token, slot in pairs:
            blk, off = divmod(slot, bs)
            kc[blk, off] = fp8_encode(kf[token], k8[blk][:, None])
            vc[blk, off] = fp8_encode(vf[token], v8[blk][:, None])
    else:
        kv_append(kc, vc, kf, vf, pairs, kquant, vquant)

    out = np.zeros((nt, H * vf.shape[-1]), np.float32)
    quantized = kquant is not None or fp8_scales is not None
    for b in range(batch):
        s0, s1 = int(cum[b]), int(cum[b + 1])
        nq = s1 - s0
        if nq == 0:
            continue
        pb = int(past[b])
        total = pb + nq
        read_len = total if quantized else pb
        pos = np.arange(read_len)
        blocks = block_table[b, pos // bs].astype(np.int64)
        offs = pos % bs
        if kquant is not None:
            keys = quant_decode(kc[blocks, offs], kquant.scale_view(KV, d), kquant.bits, d)
            vals = quant_decode(vc[blocks, offs], vquant.scale_view(KV, vf.shape[-1]), vquant.bits, vf.shape[-1])
        elif fp8_scales is not None:
            keys = fp8_decode(kc[blocks, offs], k8[blocks][:, :, None])
            vals = fp8_decode(vc[blocks, offs], v8[blocks][:, :, None])
        else:
            keys = to_f32(kc[blocks, offs])
            vals = to_f32(vc[blocks, offs]) if vc is not None else keys[:, :, :vf.shape[-1]]
        if not quantized:
            keys = np.concatenate([keys, kf[s0:s1]], 0)
            vals = np.concatenate([vals, vf[s0:s1]], 0)
        ob = attend(qf[s0:s1], keys, vals, pb, scale=sc, is_causal=is_causal,
                    local_window_size=local_window_size, softcap=softcap,
                    head_sink=None if head_sink is None else to_f32(head_sink))
        out[s0:s1] = ob.reshape(nq, -1)
    return out, kc, vc
