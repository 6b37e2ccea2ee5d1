"""CPU-only checks of the C ABI: the library loads, exports every declared entry point, its
struct layouts match the binding, and the host-side logic (claim predicate, metadata
validation) behaves like the reference.  No kernel is launched."""

import ctypes
import os
import re

import numpy as np
import pytest

from onnxruntime_ep_b200 import _capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in sorted(os.listdir(os.path.join(ROOT, "include")))
           if h.endswith(".h")]


def declared_symbols():
    text = "".join(open(h).read() for h in HEADERS)
    return sorted(set(re.findall(r"B200_API\s+[\w\s\*]+?\b(b200_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported_and_bound():
    names = declared_symbols()
    assert len(names) >= 30
    for name in names:
        assert hasattr(_capi.LIB, name), name
        assert name in _capi.SIGNATURES, f"{name} lacks a ctypes signature"


def test_struct_layouts_match():
    assert _capi.LIB.b200_params_size() == ctypes.sizeof(_capi.PagedAttentionParams)
    assert _capi.LIB.b200_node_info_size() == ctypes.sizeof(_capi.NodeInfo)
    assert _capi.LIB.b200_version() >= 100


# ---------------------------------------------------------------------------------------------
# host metadata validation (attention.rs:3934-3990), no device memory touched
# ---------------------------------------------------------------------------------------------
DUMMY = ctypes.c_void_p(0x1000)  # never dereferenced by host validation


def host_params(cum, past, bt, nt, slots=None, NB=8, bs=4):
    p = _capi.PagedAttentionParams()
    p.num_heads, p.kv_num_heads, p.head_size = 4, 2, 16
    p.act_dtype = p.cache_dtype = _capi.DTYPE_FLOAT16
    p.num_tokens, p.batch = nt, len(cum) - 1
    p.num_blocks, p.block_size, p.max_blocks_per_seq = NB, bs, bt.shape[1]
    for f in ("query", "key", "value", "key_cache", "value_cache", "cumulative_sequence_length",
              "past_seqlens", "block_table", "output"):
        setattr(p, f, DUMMY)
    keep = [np.ascontiguousarray(a, np.int32) for a in (cum, past, bt)]
    p.host_cumulative_sequence_length = keep[0].ctypes.data
    p.host_past_seqlens = keep[1].ctypes.data
    p.host_block_table = keep[2].ctypes.data
    if slots is not None:
        keep.append(np.ascontiguousarray(slots, np.int32))
        p.host_slot_mapping = keep[-1].ctypes.data
    return p, keep


def validate(*a, **k):
    p, keep = host_params(*a, **k)
    rc = _capi.LIB.b200_paged_attention_validate_host(ctypes.byref(p))
    return rc, _capi.LIB.b200_last_error().decode()


def test_host_validation_accepts_good_metadata():
    bt = np.array([[0, 1], [2, 3]])
    rc, _ = validate([0, 2, 3], [3, 5], bt, 3)
    assert rc == _capi.B200_OK


@pytest.mark.parametrize("cum,past,msg", [
    ([1, 2, 3], [0, 0], "inconsistent cumulative lengths"),   # cum[0] != 0
    ([0, 3, 2], [0, 0], "inconsistent cumulative lengths"),   # not monotone
    ([0, 1, 2], [0, 0], "inconsistent cumulative lengths"),   # cum[B] != nt
    ([0, 2, 3], [-1, 0], "inconsistent cumulative lengths"),  # negative past
    ([0, 2, 3], [7, 0], "sequence exceeds block table capacity"),
])
def test_host_validation_messages(cum, past, msg):
    rc, err = validate(cum, past, np.array([[0, 1], [2, 3]]), 3)
    assert rc == _capi.B200_ERR_FAIL and msg in err


def test_host_validation_bad_block_and_slot():
    rc, err = validate([0, 2, 3], [3, 5], np.array([[0, 9], [2, 3]]), 3)
    assert rc == _capi.B200_ERR_FAIL and "invalid physical block" in err
    rc, err = validate([0, 2, 3], [0, 0], np.array([[0, 1], [2, 3]]), 3, slots=[0, -2, 1])
    assert rc == _capi.B200_ERR_FAIL and "slot_mapping must contain -1" in err
    rc, err = validate([0, 2, 3], [0, 0], np.array([[0, 1], [2, 3]]), 3, slots=[0, 32, 1])
    assert rc == _capi.B200_ERR_FAIL and "slot_mapping must contain -1" in err
    rc, _ = validate([0, 2, 3], [0, 0], np.array([[0, 1], [2, 3]]), 3, slots=[0, -1, 31])
    assert rc == _capi.B200_OK


def test_bad_heads_is_invalid_argument():
    p, keep = host_params([0, 1], [0], np.array([[0]]), 1)
    p.kv_num_heads = 3
    assert _capi.LIB.b200_paged_attention_validate_host(ctypes.byref(p)) == _capi.B200_ERR_INVALID_ARGUMENT
    assert "bad num_heads/kv_num_heads" in _capi.LIB.b200_last_error().decode()


def test_workspace_size_grows_with_tokens():
    sizes = []
    for nt in (1, 1000):
        p, keep = host_params([0, nt], [0], np.array([[0, 1]]), nt)
        n = ctypes.c_size_t(0)
        assert _capi.LIB.b200_paged_attention_workspace_size(ctypes.byref(p), ctypes.byref(n)) == 0
        sizes.append(n.value)
    assert sizes[1] > sizes[0] > 0


# ---------------------------------------------------------------------------------------------
# Python helper: workspace ownership (host only; the params are filled, nothing is launched)
# ---------------------------------------------------------------------------------------------
def _cpu_call_tensors(nt=20, H=8, KV=2, D=128, B=2, bs=16):
    torch = pytest.importorskip("torch")
    q = torch.zeros((nt, H * D), dtype=torch.bfloat16)
    k = torch.zeros((nt, KV * D), dtype=torch.bfloat16)
    kc = torch.zeros((8, bs, KV, D), dtype=torch.bfloat16)
    cum = torch.tensor([0, 12, nt], dtype=torch.int32)
    past = torch.tensor([0, 3], dtype=torch.int32)
    bt = torch.tensor([[0, 1], [2, 3]], dtype=torch.int32)
    return (q, k, k, kc, kc, cum, past, bt), dict(num_heads=H, kv_num_heads=KV)


def test_build_params_keeps_its_shared_workspace(monkeypatch):
    """A later, larger build replaces the shared buffer; params built before it keep theirs
    alive through the keepalive list instead of pointing at freed memory."""
    torch = pytest.importorskip("torch")
    from onnxruntime_ep_b200 import paged
    bufs = []

    def fake_shared(device, nbytes):
        bufs.append(torch.empty(nbytes, dtype=torch.uint8))
        return bufs[-1]

    monkeypatch.setattr(paged, "_shared_workspace", fake_shared)
    args, kw = _cpu_call_tensors()
    p, keep, _ = paged.build_params(*args, **kw)
    assert any(t is bufs[-1] for t in keep)
    assert p.workspace == bufs[-1].data_ptr() and p.workspace_bytes == bufs[-1].numel()


def test_build_params_private_workspace():
    torch = pytest.importorskip("torch")
    from onnxruntime_ep_b200 import paged
    args, kw = _cpu_call_tensors()
    need = ctypes.c_size_t(0)
    p0, _, _ = paged.build_params(*args, **kw, workspace=torch.empty(64 << 20, dtype=torch.uint8))
    _capi.check(_capi.LIB.b200_paged_attention_workspace_size(ctypes.byref(p0), ctypes.byref(need)))
    ws = torch.empty(need.value, dtype=torch.uint8)
    p, keep, _ = paged.build_params(*args, **kw, workspace=ws)
    assert p.workspace == ws.data_ptr() and p.workspace_bytes == need.value
    assert any(t is ws for t in keep)
    for bad in (torch.empty(need.value - 1, dtype=torch.uint8), torch.empty(need.value, dtype=torch.int8),
                torch.empty(2 * need.value, dtype=torch.uint8)[::2]):
        with pytest.raises(_capi.B200Error, match="workspace"):
            paged.build_params(*args, **kw, workspace=bad)
