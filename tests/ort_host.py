"""ctypes driver of the fake ONNX Runtime host (tests/ort_stub/fake_ort.cpp), which loads the EP
glue (onnxruntime-ep-mlx_b200/csrc/ep_shell.cpp, built against tests/ort_stub's stand-in
header) and calls it the way ORT's plugin-EP host does."""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
STUB = os.path.join(HERE, "ort_stub")
SHELL = os.path.join(STUB, "_build", "libonnxruntime_ep_b200.so")
FAKE = os.path.join(STUB, "_build", "libfake_ort.so")

F32, U8, I8, I32, I64, F16, BF16, F8 = 1, 2, 3, 6, 7, 10, 16, 17
CPU, GPU, NPU = 0, 1, 2
NVIDIA = 0x10DE
ORT_OK, ORT_FAIL, ORT_INVALID_ARGUMENT, ORT_NOT_IMPLEMENTED, ORT_EP_FAIL = 0, 1, 2, 9, 11

_vp, _i64p = ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64)


def build() -> None:
    """Build the stub-header glue and the fake host (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", STUB], check=True)


def _load():
    build()
    lib = ctypes.CDLL(FAKE)
    sig = {
        "fake_last_code": (ctypes.c_int, []),
        "fake_last_error": (ctypes.c_char_p, []),
        "fake_live_counts": (None, [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
        "fake_graph_new": (_vp, []),
        "fake_graph_free": (None, [_vp]),
        "fake_node_new": (_vp, [_vp, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p]),
        "fake_node_input": (None, [_vp, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _i64p]),
        "fake_node_input_untyped": (None, [_vp, ctypes.c_char_p]),
        "fake_node_output": (None, [_vp, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _i64p]),
        "fake_node_attr_int": (None, [_vp, ctypes.c_char_p, ctypes.c_int64]),
        "fake_node_attr_float": (None, [_vp, ctypes.c_char_p, ctypes.c_float]),
        "fake_node_attr_string": (None, [_vp, ctypes.c_char_p, ctypes.c_char_p]),
        "fake_kctx_new": (_vp, []),
        "fake_kctx_free": (None, [_vp]),
        "fake_kctx_input": (None, [_vp, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _i64p, _vp, ctypes.c_size_t]),
        "fake_kctx_output": (None, [_vp, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _i64p, _vp, ctypes.c_size_t]),
        "fake_kctx_requested": (ctypes.c_int, [_vp, ctypes.c_char_p, _i64p, ctypes.c_int]),
        "fake_host_open": (_vp, [ctypes.c_char_p, ctypes.c_uint32, ctypes.c_char_p]),
        "fake_create_factories_raw": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t]),
        "fake_host_string": (ctypes.c_char_p, [_vp, ctypes.c_int]),
        "fake_host_vendor_id": (ctypes.c_uint32, [_vp]),
        "fake_host_stream_aware": (ctypes.c_int, [_vp]),
        "fake_host_devices": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_uint32),
                                             ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t),
                                             ctypes.POINTER(ctypes.c_int)]),
        "fake_host_device_memory": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int),
                                                   ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_int)]),
        "fake_host_create_ep": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_char_p),
                                               ctypes.c_size_t, ctypes.c_size_t]),
        "fake_host_ep_name": (ctypes.c_char_p, [_vp]),
        "fake_host_default_memory": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_uint32),
                                                    ctypes.POINTER(ctypes.c_int)]),
        "fake_host_capability": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(ctypes.c_int), ctypes.c_size_t,
                                                ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_int)]),
        "fake_host_report": (ctypes.c_char_p, [_vp]),
        "fake_host_compile": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int]),
        "fake_host_compute": (ctypes.c_int, [_vp, ctypes.c_int, _vp]),
        "fake_host_allocator": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_int]),
        "fake_host_alloc": (_vp, [_vp, ctypes.c_size_t]),
        "fake_host_free": (None, [_vp, _vp]),
        "fake_host_allocator_name": (ctypes.c_char_p, [_vp]),
        "fake_host_transfer": (ctypes.c_int, [_vp]),
        "fake_host_can_copy": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
        "fake_host_copy": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _i64p, _vp, ctypes.c_size_t, ctypes.c_int,
                                          _i64p, _vp, ctypes.c_size_t]),
        "fake_host_close": (None, [_vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    return lib


LIB = _load()


def _shape(shape):
    arr = (ctypes.c_int64 * max(len(shape), 1))(*[int(s) for s in shape])
    return len(shape), arr


def last_error() -> tuple[int, str]:
    return LIB.fake_last_code(), LIB.fake_last_error().decode()


def live_counts() -> tuple[int, int]:
    """(memory infos, statuses) the fake host created and nobody released yet."""
    a, b = ctypes.c_int(), ctypes.c_int()
    LIB.fake_live_counts(ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


class Node:
    def __init__(self, graph, op, domain, name):
        self.handle = LIB.fake_node_new(graph.handle, op.encode(), domain.encode(), name.encode())
        self.name = name

    def input(self, name, dtype=0, shape=()):
        rank, arr = _shape(shape)
        LIB.fake_node_input(self.handle, (name or "").encode(), dtype, rank, arr)
        return self

    def input_untyped(self, name):
        LIB.fake_node_input_untyped(self.handle, name.encode())
        return self

    def output(self, name, dtype=0, shape=()):
        rank, arr = _shape(shape)
        LIB.fake_node_output(self.handle, (name or "").encode(), dtype, rank, arr)
        return self

    def attr(self, key, value):
        if isinstance(value, str):
            LIB.fake_node_attr_string(self.handle, key.encode(), value.encode())
        elif isinstance(value, float):
            LIB.fake_node_attr_float(self.handle, key.encode(), value)
        else:
            LIB.fake_node_attr_int(self.handle, key.encode(), int(value))
        return self


class Graph:
    def __init__(self):
        self.handle = LIB.fake_graph_new()
        self.nodes = []

    def node(self, op, name, domain="com.microsoft") -> Node:
        n = Node(self, op, domain, name)
        self.nodes.append(n)
        return n

    def close(self):
        if self.handle:
            LIB.fake_graph_free(self.handle)
            self.handle = None


class KernelContext:
    """Tensors of one Compute by value name: (dtype, shape, data pointer, bytes)."""

    def __init__(self):
        self.handle = LIB.fake_kctx_new()

    def input(self, name, dtype, shape, ptr, nbytes):
        rank, arr = _shape(shape)
        LIB.fake_kctx_input(self.handle, name.encode(), dtype, rank, arr, ptr, nbytes)

    def output(self, name, dtype, shape, ptr, nbytes):
        rank, arr = _shape(shape)
        LIB.fake_kctx_output(self.handle, name.encode(), dtype, rank, arr, ptr, nbytes)

    def requested(self, name):
        arr = (ctypes.c_int64 * 8)()
        rank = LIB.fake_kctx_requested(self.handle, name.encode(), arr, 8)
        return None if rank < 0 else tuple(arr[:rank])

    def close(self):
        if self.handle:
            LIB.fake_kctx_free(self.handle)
            self.handle = None


class Host:
    """One loaded glue library with its factory (and, after create_ep, its EP)."""

    def __init__(self, max_api_version=31, registration_name=None):
        h = LIB.fake_host_open(SHELL.encode(), max_api_version,
                               registration_name.encode() if registration_name else None)
        if not h:
            code, msg = last_error()
            raise RuntimeError(f"fake host: {code}: {msg}")
        self.handle = h

    def string(self, which):
        return LIB.fake_host_string(self.handle, {"name": 0, "vendor": 1, "version": 2}[which]).decode()

    def vendor_id(self):
        return LIB.fake_host_vendor_id(self.handle)

    def stream_aware(self):
        return bool(LIB.fake_host_stream_aware(self.handle))

    def devices(self, hw):
        """GetSupportedDevices over [(type, vendor)]: (status, ep devices, allocator infos)."""
        n = len(hw)
        types = (ctypes.c_int * max(n, 1))(*[t for t, _ in hw])
        vendors = (ctypes.c_uint32 * max(n, 1))(*[v for _, v in hw])
        num, infos = ctypes.c_size_t(), ctypes.c_int()
        rc = LIB.fake_host_devices(self.handle, types, vendors, n, ctypes.byref(num), ctypes.byref(infos))
        return rc, num.value, infos.value

    def device_memory(self):
        name = ctypes.create_string_buffer(64)
        t, v, i = ctypes.c_int(), ctypes.c_uint32(), ctypes.c_int()
        if LIB.fake_host_device_memory(self.handle, name, 64, ctypes.byref(t), ctypes.byref(v), ctypes.byref(i)):
            return None
        return name.value.decode(), t.value, v.value, i.value

    def create_ep(self, options=None, num_devices=1):
        options = options or {}
        n = len(options)
        keys = (ctypes.c_char_p * max(n, 1))(*[k.encode() for k in options])
        vals = (ctypes.c_char_p * max(n, 1))(*[str(v).encode() for v in options.values()])
        return LIB.fake_host_create_ep(self.handle, keys, vals, n, num_devices)

    def ep_name(self):
        return LIB.fake_host_ep_name(self.handle).decode()

    def default_memory(self):
        t, v, i = ctypes.c_int(), ctypes.c_uint32(), ctypes.c_int()
        rc = LIB.fake_host_default_memory(self.handle, ctypes.byref(t), ctypes.byref(v), ctypes.byref(i))
        return None if rc else (t.value, v.value, i.value)

    def capability(self, graph):
        """GetCapability: (status, claimed node indices, drop_constant_initializers of the fusions)."""
        out = (ctypes.c_int * 64)()
        n, drop = ctypes.c_size_t(), ctypes.c_int()
        rc = LIB.fake_host_capability(self.handle, graph.handle, out, 64, ctypes.byref(n), ctypes.byref(drop))
        return rc, list(out[:n.value]), drop.value

    def report(self):
        return LIB.fake_host_report(self.handle).decode()

    def compile(self, graph, index, reverse=False):
        return LIB.fake_host_compile(self.handle, graph.handle, index, 1 if reverse else 0)

    def compute(self, compiled, ctx):
        return LIB.fake_host_compute(self.handle, compiled, ctx.handle)

    def allocator(self, name="B200", device=0):
        return LIB.fake_host_allocator(self.handle, name.encode(), device)

    def alloc(self, nbytes):
        return LIB.fake_host_alloc(self.handle, nbytes)

    def free(self, ptr):
        LIB.fake_host_free(self.handle, ptr)

    def allocator_name(self):
        return LIB.fake_host_allocator_name(self.handle).decode()

    def transfer(self):
        return LIB.fake_host_transfer(self.handle)

    def can_copy(self, src, dst, device=0):
        kinds = {"cpu": 0, "b200": 1, "other": 2}
        return bool(LIB.fake_host_can_copy(self.handle, kinds[src], kinds[dst], device))

    def copy(self, dtype, shape, src, src_bytes, dst_shape, dst, dst_bytes):
        rank, arr = _shape(shape)
        drank, darr = _shape(dst_shape)
        return LIB.fake_host_copy(self.handle, dtype, rank, arr, src, src_bytes, drank, darr, dst, dst_bytes)

    def close(self):
        if self.handle:
            LIB.fake_host_close(self.handle)
            self.handle = None


def create_factories_raw(max_factories: int) -> int:
    return LIB.fake_create_factories_raw(SHELL.encode(), max_factories)


def paged_node(graph, name="pa", *, H=4, KV=2, d=16, dt=F16, nb=8, bs=4, B=2, maxb=4, cache_dt=None, packed=False,
               outputs=1, attrs=None, extra_inputs=None):
    """A PagedAttention node with the 8 required inputs (dynamic token count) named after `name`."""
    n = graph.node("PagedAttention", name)
    cache_dt = cache_dt or dt
    cw = d if cache_dt != U8 else (d + 1) // 2
    n.input(f"{name}.query", dt, (-1, (H + 2 * KV) * d if packed else H * d))
    if packed:
        n.input(None).input(None)
    else:
        n.input(f"{name}.key", dt, (-1, KV * d)).input(f"{name}.value", dt, (-1, KV * d))
    n.input(f"{name}.key_cache", cache_dt, (nb, bs, KV, cw)).input(f"{name}.value_cache", cache_dt, (nb, bs, KV, cw))
    n.input(f"{name}.cum", I32, (B + 1,)).input(f"{name}.past", I32, (B,)).input(f"{name}.block_table", I32, (B, maxb))
    for spec in extra_inputs or []:
        n.input(*spec) if spec else n.input(None)
    n.output(f"{name}.out", dt, (-1, H * d))
    if outputs >= 2:
        n.output(f"{name}.key_cache_out", cache_dt, (nb, bs, KV, cw))
    if outputs >= 3:
        n.output(f"{name}.value_cache_out", cache_dt, (nb, bs, KV, cw))
    n.attr("num_heads", H).attr("kv_num_heads", KV)
    for k, v in (attrs or {}).items():
        n.attr(k, v)
    return n


def gqa_node(graph, name="gqa", *, H=4, KV=2, d=16, dt=F16, B=1, S=1, cap=32, attrs=None, rotary=None,
             present=True):
    """A GroupQueryAttention node: separate Q/K/V, BNSH past caches of capacity `cap`."""
    n = graph.node("GroupQueryAttention", name)
    n.input(f"{name}.query", dt, (B, S, H * d)).input(f"{name}.key", dt, (B, S, KV * d))
    n.input(f"{name}.value", dt, (B, S, KV * d))
    n.input(f"{name}.past_key", dt, (B, KV, cap, d)).input(f"{name}.past_value", dt, (B, KV, cap, d))
    n.input(f"{name}.seqlens_k", I32, (B,)).input(f"{name}.total", I32, (1,))
    if rotary:
        positions, half = rotary
        n.input(f"{name}.cos", dt, (positions, half)).input(f"{name}.sin", dt, (positions, half))
    n.output(f"{name}.out", dt, (B, S, H * d))
    if present:
        n.output(f"{name}.present_key", dt, (B, KV, -1, d)).output(f"{name}.present_value", dt, (B, KV, -1, d))
    n.attr("num_heads", H).attr("kv_num_heads", KV)
    for k, v in (attrs or {}).items():
        n.attr(k, v)
    return n


def ptr_of(a: np.ndarray) -> int:
    return a.ctypes.data
