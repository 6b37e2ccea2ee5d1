"""ctypes wrapper of the C oracle (``oracle/paged_ref.c``) — TEST INFRASTRUCTURE ONLY.

Used by tests (large parity cases) and by bench.py's ``cpu_baseline`` / ``--impl reference``
legs.  Arrays are numpy (fp16 or ml_dtypes.bfloat16 activations, int32 metadata).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpaged_oracle.so")


def build() -> str:
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "paged_ref.c")):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(LIB_PATH)
        vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        _lib.oracle_paged_attention_fp8.restype = ctypes.c_int
        _lib.oracle_paged_attention_fp8.argtypes = ([i32] * 9 + [vp] * 11 +
                                                    [f32, i32, i32, f32, vp, vp, i32, i32, i32, i32, vp])
        _lib.oracle_e4m3_encode.restype = None
        _lib.oracle_e4m3_encode.argtypes = [vp, vp, ctypes.c_int64]
        _lib.oracle_paged_attention.restype = ctypes.c_int
        _lib.oracle_paged_attention.argtypes = [i32] * 9 + [vp] * 9 + [f32, i32, i32, f32, vp, vp, i32, i32, i32, i32,
                                                                        vp]
    return _lib


def _p(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def paged_attention(q, k, v, key_cache, value_cache, cum, past, block_table, H, KV, *,
                    slot_mapping=None, scale=0.0, is_causal=True, local_window_size=-1, softcap=0.0,
                    head_sink=None, threads=None, append=True, seq_range=None, out=None, fp32_out=False):
    """Run the C oracle in place on ``key_cache``/``value_cache`` (when ``append``) and return
    the output ``[nt, H*d]`` in the activation dtype, or in fp32 before that rounding when
    ``fp32_out`` (rows of sequences outside ``seq_range`` stay zero)."""
    dt = 16 if q.dtype.name == "bfloat16" else 10
    nt = q.shape[0]
    d = q.shape[1] // H
    B = len(cum) - 1
    NB, bs = key_cache.shape[0], key_cache.shape[1]
    maxb = block_table.shape[1]
    arrs = [np.ascontiguousarray(x) for x in (q, k, v)]
    assert key_cache.flags.c_contiguous and value_cache.flags.c_contiguous
    cum = np.ascontiguousarray(cum, np.int32)
    past = np.ascontiguousarray(past, np.int32)
    bt = np.ascontiguousarray(block_table, np.int32)
    slots = None if slot_mapping is None else np.ascontiguousarray(slot_mapping, np.int32)
    sink = None if head_sink is None else np.ascontiguousarray(np.asarray(head_sink, np.float32))
    out32 = None
    if fp32_out:
        out32 = np.zeros((nt, H * d), np.float32)
        out = np.zeros((1, 1), q.dtype)  # unused
    elif out is None:
        out = np.zeros((nt, H * d), q.dtype)
    threads = threads or os.cpu_count() or 1
    s0, s1 = seq_range if seq_range else (0, B)
    rc = lib().oracle_paged_attention(
        dt, H, KV, d, nt, B, NB, bs, maxb, _p(arrs[0]), _p(arrs[1]), _p(arrs[2]), _p(key_cache),
        _p(value_cache), _p(cum), _p(past), _p(bt), _p(slots), float(scale), int(bool(is_causal)),
        int(local_window_size), float(softcap), _p(sink), _p(out), int(threads), int(bool(append)),
        int(s0), int(s1), _p(out32))
    if rc != 0:
        raise RuntimeError(f"oracle_paged_attention failed ({rc})")
    return out32 if fp32_out else out


def paged_attention_fp8(q, k, v, key_cache, value_cache, k_scale, v_scale, cum, past, block_table, H, KV, *,
                        slot_mapping=None, scale=0.0, is_causal=True, local_window_size=-1, softcap=0.0,
                        head_sink=None, threads=None, append=True, seq_range=None):
    """fp8 e4m3 caches (``uint8`` or ``ml_dtypes.float8_e4m3fn`` arrays ``[NB, bs, KV, d]``) with
    per-(block, kv head) fp32 scales ``[NB, KV]``.  Appends the new rows (encoded) in place when
    ``append`` and returns the fp32 output ``[nt, H*d]``."""
    dt = 16 if q.dtype.name == "bfloat16" else 10
    nt = q.shape[0]
    d = q.shape[1] // H
    B = len(cum) - 1
    NB, bs = key_cache.shape[0], key_cache.shape[1]
    maxb = block_table.shape[1]
    arrs = [np.ascontiguousarray(x) for x in (q, k, v)]
    assert key_cache.flags.c_contiguous and value_cache.flags.c_contiguous
    ks = np.ascontiguousarray(k_scale, np.float32)
    vs = np.ascontiguousarray(v_scale, np.float32)
    cum = np.ascontiguousarray(cum, np.int32)
    past = np.ascontiguousarray(past, np.int32)
    bt = np.ascontiguousarray(block_table, np.int32)
    slots = None if slot_mapping is None else np.ascontiguousarray(slot_mapping, np.int32)
    sink = None if head_sink is None else np.ascontiguousarray(np.asarray(head_sink, np.float32))
    out32 = np.zeros((nt, H * d), np.float32)
    threads = threads or os.cpu_count() or 1
    s0, s1 = seq_range if seq_range else (0, B)
    rc = lib().oracle_paged_attention_fp8(
        dt, H, KV, d, nt, B, NB, bs, maxb, _p(arrs[0]), _p(arrs[1]), _p(arrs[2]), _p(key_cache),
        _p(value_cache), _p(cum), _p(past), _p(bt), _p(slots), _p(ks), _p(vs), float(scale),
        int(bool(is_causal)), int(local_window_size), float(softcap), _p(sink), None, int(threads),
        int(bool(append)), int(s0), int(s1), _p(out32))
    if rc != 0:
        raise RuntimeError(f"oracle_paged_attention_fp8 failed ({rc})")
    return out32


def e4m3_encode(x):
    """The C oracle's fp32 -> e4m3fn encoder (round to nearest even, saturating at 448)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(x.shape, np.uint8)
    lib().oracle_e4m3_encode(_p(x), _p(out), x.size)
    return out
