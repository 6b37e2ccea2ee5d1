"""Python side of the EP host layer (include/b200_ep.h): session options, the KV block pool and
the compiled-node launcher.

These mirror what the ONNX Runtime plugin shell does around each claimed node: parse the
``ep.b200.*`` session options (session value first, then the environment), create one node
state per claimed PagedAttention / GroupQueryAttention node, and run its Compute on the node's
tensors.  The KV block pool owns (or adopts) the paged K/V caches and hands out block ids for the
block tables.
"""

from __future__ import annotations

import ctypes

from . import _capi
from ._capi import LIB, B200Error, check


def parse_options(session: dict | None = None) -> _capi.EpOptions:
    """``ep.b200.*`` options from a session config dict, then the environment (strict parse)."""
    session = session or {}
    n = len(session)
    keys = (ctypes.c_char_p * max(n, 1))(*[k.encode() for k in session])
    vals = (ctypes.c_char_p * max(n, 1))(*[str(v).encode() for v in session.values()])
    out = _capi.EpOptions()
    check(LIB.b200_ep_options_parse(keys, vals, n, ctypes.byref(out)))
    return out


def ort_error_class(status: int) -> str:
    """``"OK"``, ``"ORT_INVALID_ARGUMENT"`` or ``"ORT_EP_FAIL"`` for a B200 status."""
    return {0: "OK", 1: "ORT_INVALID_ARGUMENT", 2: "ORT_EP_FAIL"}[LIB.b200_ort_error_class(status)]


class KvPool:
    """Paged K/V caches ``[num_blocks, block_size, kv_heads, head_size]`` and their free block ids.

    ``KvPool(budget_bytes=..., ...)`` allocates the caches on the device; ``key_cache=`` /
    ``value_cache=`` (device pointers or tensors) adopt caller-owned caches instead."""

    def __init__(self, *, block_size, kv_num_heads, head_size, cache_dtype, num_blocks=0, budget_bytes=0,
                 device=0, key_cache=None, value_cache=None, k_scale=None, v_scale=None):
        d = _capi.KvPoolDesc()
        d.device, d.block_size, d.kv_num_heads, d.head_size = device, block_size, kv_num_heads, head_size
        d.cache_dtype, d.num_blocks, d.budget_bytes = cache_dtype, num_blocks, budget_bytes

        def ptr(x):
            if x is None:
                return None
            return ctypes.c_void_p(x if isinstance(x, int) else x.data_ptr())

        d.key_cache, d.value_cache, d.k_scale, d.v_scale = (ptr(x) for x in (key_cache, value_cache, k_scale, v_scale))
        self._keep = (key_cache, value_cache, k_scale, v_scale)
        handle = ctypes.c_void_p()
        check(LIB.b200_kv_pool_create(ctypes.byref(d), ctypes.byref(handle)))
        self.handle = handle

    def info(self) -> _capi.KvPoolInfo:
        out = _capi.KvPoolInfo()
        check(LIB.b200_kv_pool_info(self.handle, ctypes.byref(out)))
        return out

    def alloc(self, count: int) -> list[int]:
        ids = (ctypes.c_int32 * max(count, 1))()
        check(LIB.b200_kv_pool_alloc(self.handle, count, ids))
        return list(ids[:count])

    def free(self, ids) -> None:
        ids = list(ids)
        arr = (ctypes.c_int32 * max(len(ids), 1))(*ids)
        check(LIB.b200_kv_pool_free(self.handle, arr, len(ids)))

    def blocks_for(self, tokens: int) -> int:
        return LIB.b200_kv_pool_blocks_for(self.handle, tokens)

    def caches(self, torch_dtype):
        """The pool's K and V caches as torch tensors (views of the pool's device memory)."""
        import torch

        info = self.info()
        shape = (info.num_blocks, info.block_size, -1)
        out = []
        for p in (info.key_cache, info.value_cache):
            nbytes = info.num_blocks * info.block_bytes
            buf = _device_buffer(p, nbytes)
            out.append(torch.as_tensor(buf, device="cuda").view(torch.uint8).view(torch_dtype).view(*shape))
        return out

    def close(self) -> None:
        if self.handle:
            check(LIB.b200_kv_pool_destroy(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def _device_buffer(ptr: int, nbytes: int):
    """A ``__cuda_array_interface__`` holder for `nbytes` of device memory at `ptr`."""

    class _Buf:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                    "strides": None}

    return _Buf()


class EpNode:
    """The launcher state of one claimed node (``kind`` "paged" or "gqa")."""

    def __init__(self, node_info, options: _capi.EpOptions | None = None, kind: str = "paged"):
        handle = ctypes.c_void_p()
        opts = ctypes.byref(options) if options is not None else None
        create = LIB.b200_ep_node_create_paged if kind == "paged" else LIB.b200_ep_node_create_gqa
        check(create(ctypes.byref(node_info), opts, ctypes.byref(handle)))
        self.handle, self.kind = handle, kind

    def compute_paged(self, tensors: _capi.PagedTensors, stream) -> None:
        check(LIB.b200_ep_node_compute_paged(self.handle, ctypes.byref(tensors), ctypes.c_void_p(stream)))

    def compute_gqa(self, params: _capi.GqaParams, stream) -> None:
        check(LIB.b200_ep_node_compute_gqa(self.handle, ctypes.byref(params), ctypes.c_void_p(stream)))

    def stats(self):
        ws, n = ctypes.c_uint64(), ctypes.c_uint64()
        check(LIB.b200_ep_node_stats(self.handle, ctypes.byref(ws), ctypes.byref(n)))
        return {"workspace_bytes": ws.value, "computes": n.value}

    def close(self) -> None:
        if self.handle:
            check(LIB.b200_ep_node_destroy(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


__all__ = ["EpNode", "KvPool", "B200Error", "ort_error_class", "parse_options"]
