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
        _lib.oracle_paged_attention.restype = ctypes.c_int
        _lib.oracle_paged_attention.argtypes = [i32] * 9 + [vp] * 9 + [f32, i32, i32, f32, vp, vp, i32, i32, i32, i32]
    return _lib


def _p(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def paged_attention(q, k, v, key_cache, value_cache, cum, past, block_table, H, KV, *,
                    slot_mapping=None, scale=0.0, is_causal=True, local_window_size=-1, softcap=0.0,
                    head_sink=None, threads=None, append=True, seq_range=None, out=None):
    """Run the C oracle in place on ``key_cache``/``value_cache`` (when ``append``) and return
    the output ``[nt, H*d]`` in the activation dtype."""
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
    if out is None:
        out = np.zeros((nt, H * d), q.dtype)
    threads = threads or os.cpu_count() or 1
    s0, s1 = seq_range if seq_range else (0, B)
    rc = lib().oracle_paged_attention(
        dt, H, KV, d, nt, B, NB, bs, maxb, _p(arrs[0]), _p(arrs[1]), _p(arrs[2]), _p(key_cache),
        _p(value_cache), _p(cum), _p(past), _p(bt), _p(slots), float(scale), int(bool(is_causal)),
        int(local_window_size), float(softcap), _p(sink), _p(out), int(threads), int(bool(append)),
        int(s0), int(s1))
    if rc != 0:
        raise RuntimeError(f"oracle_paged_attention failed ({rc})")
    return out
