"""Host-side checks of ``b200_shard_gather`` (include/b200_shard.h): every geometry and pointer
check runs before anything touches a device, with B200_ERR_INVALID_ARGUMENT and its message."""

import ctypes

import pytest

from onnxruntime_ep_b200 import _capi


def params(world=2, rank=0, rows=4, slice_bytes=64):
    p = _capi.ShardGatherParams()
    p.world, p.rank, p.rows, p.slice_bytes = world, rank, rows, slice_bytes
    p.local = 0x1000
    for t in range(world):
        p.outputs[t] = 0x2000 + 0x1000 * t
        p.flags[t] = 0x9000 + 0x100 * t
    p.state = 0x8000
    return p


def call(p):
    return _capi.LIB.b200_shard_gather(ctypes.byref(p), None), _capi.LIB.b200_last_error().decode()


def test_layout_matches_library():
    assert _capi.LIB.b200_shard_gather_params_size() == ctypes.sizeof(_capi.ShardGatherParams)
    assert _capi.LIB.b200_ipc_handle_size() == 64


@pytest.mark.parametrize("mutate,message", [
    (lambda p: setattr(p, "world", 0), "world must be 1..8"),
    (lambda p: setattr(p, "world", 9), "world must be 1..8"),
    (lambda p: setattr(p, "rank", 2), "rank in [0, world)"),
    (lambda p: setattr(p, "slice_bytes", 24), "slice_bytes a positive multiple of 16"),
    (lambda p: setattr(p, "rows", -1), "rows >= 0"),
    (lambda p: setattr(p, "local", None), "local (16-byte aligned) and state are required"),
    (lambda p: setattr(p, "local", 0x1008), "local (16-byte aligned) and state are required"),
    (lambda p: setattr(p, "state", None), "local (16-byte aligned) and state are required"),
    (lambda p: p.outputs.__setitem__(1, None), "every rank's output (16-byte aligned) and flags are required"),
    (lambda p: p.flags.__setitem__(0, None), "every rank's output (16-byte aligned) and flags are required"),
])
def test_invalid_arguments(mutate, message):
    p = params()
    mutate(p)
    rc, msg = call(p)
    assert rc == _capi.B200_ERR_INVALID_ARGUMENT
    assert message in msg


def test_ipc_null_arguments():
    handle = (ctypes.c_uint8 * 64)()
    assert _capi.LIB.b200_ipc_get_handle(None, ctypes.addressof(handle)) == _capi.B200_ERR_INVALID_ARGUMENT
    ptr = ctypes.c_void_p()
    assert _capi.LIB.b200_ipc_open_handle(0, None, ctypes.byref(ptr)) == _capi.B200_ERR_INVALID_ARGUMENT
    assert _capi.LIB.b200_ipc_close_handle(0, None) == _capi.B200_OK
