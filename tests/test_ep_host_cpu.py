"""EP host layer on CPU (include/b200_ep.h): strict session options with session-over-environment
precedence (rust/src/config.rs:18-64, rust/src/memory.rs:10-98), the status -> ORT error class
mapping (rust/src/lib.rs:53-92), the KV block pool's bookkeeping over caller-owned caches (no
device memory is touched), and node creation through the claim predicates."""

import ctypes

import pytest

from onnxruntime_ep_b200 import _capi, ep
from onnxruntime_ep_b200._capi import B200Error

ENV = ["ONNXRUNTIME_EP_B200_KV_POOL_BYTES", "ONNXRUNTIME_EP_B200_NUM_GPUS", "ONNXRUNTIME_EP_B200_DEVICE_ID",
       "ONNXRUNTIME_EP_B200_DECODE_MIN_TILES", "ONNXRUNTIME_EP_B200_FORCE_GENERIC", "ONNXRUNTIME_EP_B200_CHECK_STATUS"]


@pytest.fixture(autouse=True)
def clean_env(monkeypatch):
    for k in ENV:
        monkeypatch.delenv(k, raising=False)


def test_defaults():
    o = ep.parse_options({})
    assert (o.has_kv_pool_bytes, o.kv_pool_bytes, o.num_gpus, o.device_id) == (0, 0, 1, 0)
    assert (o.decode_min_tiles_per_warp, o.force_generic, o.check_status) == (0, 0, 1)


def test_session_values_parse():
    o = ep.parse_options({"ep.b200.kv_pool_bytes": "536870912", "ep.b200.num_gpus": "8",
                          "ep.b200.device_id": "3", "ep.b200.decode_min_tiles_per_warp": "6",
                          "ep.b200.force_generic": "1", "ep.b200.check_status": "0",
                          "session.other_entry": "kept by ORT, ignored here"})
    assert (o.has_kv_pool_bytes, o.kv_pool_bytes) == (1, 512 * 1024 * 1024)
    assert (o.num_gpus, o.device_id, o.decode_min_tiles_per_warp, o.force_generic, o.check_status) == (8, 3, 6, 1, 0)


def test_byte_counts_accept_zero_and_the_64_bit_maximum():
    assert ep.parse_options({"ep.b200.kv_pool_bytes": "0"}).kv_pool_bytes == 0
    assert ep.parse_options({"ep.b200.kv_pool_bytes": str(2**64 - 1)}).kv_pool_bytes == 2**64 - 1


@pytest.mark.parametrize("value", ["", "-1", "1e9", " 1", "1 ", "0x10", "+5", str(2**64), "1.5"])
def test_byte_counts_are_strict(value):
    with pytest.raises(B200Error, match="ep.b200.kv_pool_bytes must be a nonnegative decimal byte count") as e:
        ep.parse_options({"ep.b200.kv_pool_bytes": value})
    assert e.value.code == _capi.B200_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("value", ["", "true", "false", "2", "-1", " 1", "01"])
def test_booleans_accept_only_zero_and_one(value):
    # the reference's boolean rule (config.rs:46-52, its test at :72-80)
    with pytest.raises(B200Error, match="ep.b200.force_generic: expected 0 or 1"):
        ep.parse_options({"ep.b200.force_generic": value})


@pytest.mark.parametrize("key,value", [("ep.b200.num_gpus", "0"), ("ep.b200.num_gpus", "x"),
                                       ("ep.b200.device_id", "-1"), ("ep.b200.decode_min_tiles_per_warp", "0"),
                                       ("ep.b200.num_gpus", str(2**31))])
def test_integers_are_strict(key, value):
    with pytest.raises(B200Error, match=key.replace(".", r"\.")):
        ep.parse_options({key: value})


def test_environment_fills_what_the_session_leaves_unset(monkeypatch):
    monkeypatch.setenv("ONNXRUNTIME_EP_B200_KV_POOL_BYTES", "1024")
    monkeypatch.setenv("ONNXRUNTIME_EP_B200_FORCE_GENERIC", "1")
    o = ep.parse_options({"ep.b200.force_generic": "0"})
    assert (o.has_kv_pool_bytes, o.kv_pool_bytes) == (1, 1024)  # from the environment
    assert o.force_generic == 0  # the session value wins


def test_bad_environment_value_names_the_variable(monkeypatch):
    monkeypatch.setenv("ONNXRUNTIME_EP_B200_KV_POOL_BYTES", "lots")
    with pytest.raises(B200Error, match="ONNXRUNTIME_EP_B200_KV_POOL_BYTES \\(environment\\)"):
        ep.parse_options({})
    # a session value shadows the bad environment entry
    assert ep.parse_options({"ep.b200.kv_pool_bytes": "7"}).kv_pool_bytes == 7


def test_error_classes():
    assert ep.ort_error_class(_capi.B200_OK) == "OK"
    assert ep.ort_error_class(_capi.B200_ERR_INVALID_ARGUMENT) == "ORT_INVALID_ARGUMENT"
    for code in (_capi.B200_ERR_FAIL, _capi.B200_ERR_CUDA, _capi.B200_ERR_UNSUPPORTED, _capi.B200_ERR_WORKSPACE,
                 _capi.B200_ERR_DEVICE):
        assert ep.ort_error_class(code) == "ORT_EP_FAIL"


def test_struct_layouts_match():
    for which, cls in enumerate((_capi.EpOptions, _capi.KvPoolDesc, _capi.KvPoolInfo, _capi.PagedTensors)):
        assert _capi.LIB.b200_ep_struct_size(which) == ctypes.sizeof(cls)


# ---- KV block pool over caller-owned caches (never dereferenced here) -----------------------
FAKE_K, FAKE_V = 0x10000, 0x20000


def pool(nb=10, **kw):
    return ep.KvPool(block_size=16, kv_num_heads=8, head_size=128, cache_dtype=_capi.DTYPE_BFLOAT16,
                     num_blocks=nb, key_cache=FAKE_K, value_cache=FAKE_V, **kw)


def test_block_bytes():
    d = _capi.KvPoolDesc(block_size=16, kv_num_heads=8, head_size=128)
    out = ctypes.c_uint64()
    for dt, want in ((_capi.DTYPE_BFLOAT16, 16 * 8 * 128 * 2), (_capi.DTYPE_INT8, 16 * 8 * 128),
                     (_capi.DTYPE_FLOAT8E4M3FN, 16 * 8 * 128), (_capi.DTYPE_UINT8, 16 * 8 * 64)):
        d.cache_dtype = dt
        assert _capi.LIB.b200_kv_pool_block_bytes(ctypes.byref(d), ctypes.byref(out)) == 0
        assert out.value == want
    d.head_size = 7
    d.cache_dtype = _capi.DTYPE_UINT8
    _capi.LIB.b200_kv_pool_block_bytes(ctypes.byref(d), ctypes.byref(out))
    assert out.value == 16 * 8 * 4  # int4 rows round the head up to whole bytes


def test_pool_hands_out_lowest_ids_first_and_reuses_freed_ones():
    p = pool()
    info = p.info()
    assert (info.num_blocks, info.free_blocks, info.owns_memory, info.key_cache) == (10, 10, 0, FAKE_K)
    a = p.alloc(3)
    assert a == [0, 1, 2]
    b = p.alloc(2)
    assert b == [3, 4]
    p.free([1])
    assert p.alloc(1) == [1]  # the last freed block goes out next
    assert p.info().free_blocks == 5
    p.free(a + b)
    assert p.info().free_blocks == 10


def test_pool_alloc_is_all_or_nothing():
    p = pool(nb=4)
    p.alloc(3)
    with pytest.raises(B200Error, match="out of KV cache blocks") as e:
        p.alloc(2)
    assert ep.ort_error_class(e.value.code) == "ORT_EP_FAIL"
    assert p.info().free_blocks == 1


@pytest.mark.parametrize("bad,reason", [([99], "outside"), ([-1], "outside"), ([5], "not allocated"),
                                        ([0, 0], "freed twice")])
def test_pool_free_checks_every_id_and_changes_nothing_on_error(bad, reason):
    p = pool()
    p.alloc(3)
    with pytest.raises(B200Error, match=reason):
        p.free([2] + bad if bad != [0, 0] else bad)
    assert p.info().free_blocks == 7  # block 2 was not freed either


def test_pool_blocks_for():
    p = pool()
    assert [p.blocks_for(t) for t in (0, 1, 16, 17, 8192)] == [0, 1, 1, 2, 512]


def test_pool_geometry_and_budget_errors():
    with pytest.raises(B200Error, match="num_blocks or a byte budget"):
        ep.KvPool(block_size=16, kv_num_heads=8, head_size=128, cache_dtype=_capi.DTYPE_BFLOAT16)
    with pytest.raises(B200Error, match="holds no block"):
        ep.KvPool(block_size=16, kv_num_heads=8, head_size=128, cache_dtype=_capi.DTYPE_BFLOAT16, budget_bytes=100)
    with pytest.raises(B200Error, match="over the budget"):
        ep.KvPool(block_size=16, kv_num_heads=8, head_size=128, cache_dtype=_capi.DTYPE_BFLOAT16, num_blocks=4,
                  budget_bytes=4 * 65536 - 1)
    with pytest.raises(B200Error, match="both key_cache and value_cache"):
        ep.KvPool(block_size=16, kv_num_heads=8, head_size=128, cache_dtype=_capi.DTYPE_BFLOAT16, num_blocks=4,
                  key_cache=FAKE_K)
    with pytest.raises(B200Error, match="need k_scale and v_scale"):
        ep.KvPool(block_size=16, kv_num_heads=1, head_size=128, cache_dtype=_capi.DTYPE_FLOAT8E4M3FN, num_blocks=4,
                  key_cache=FAKE_K, value_cache=FAKE_V)
    with pytest.raises(B200Error, match="cache dtype"):
        ep.KvPool(block_size=16, kv_num_heads=8, head_size=128, cache_dtype=_capi.DTYPE_FLOAT, num_blocks=4,
                  key_cache=FAKE_K, value_cache=FAKE_V)


# ---- node creation (the claim predicate decides) ---------------------------------------------
def test_paged_node_creation_follows_the_claim():
    from test_claim_cpu import node

    n = ep.EpNode(node(H=32, KV=8, d=128, dt=_capi.DTYPE_BFLOAT16, nb=64, bs=16, B=4, maxb=8))
    assert n.stats() == {"workspace_bytes": 0, "computes": 0}
    n.close()
    bad = node(H=32, KV=8, d=128)
    bad.kv_cache_layout = b"LATENT"
    with pytest.raises(B200Error, match="not claimed: ") as e:
        ep.EpNode(bad)
    assert e.value.code == _capi.B200_ERR_UNSUPPORTED


def test_gqa_node_creation_follows_the_claim():
    from test_gqa_cpu import gnode

    n = ep.EpNode(gnode(), kind="gqa")
    n.close()
    bad = gnode()
    bad.qk_output = 1
    with pytest.raises(B200Error, match="GroupQueryAttention not claimed"):
        ep.EpNode(bad, kind="gqa")


def test_wrong_compute_kind_is_rejected():
    from test_gqa_cpu import gnode

    n = ep.EpNode(gnode(), kind="gqa")
    with pytest.raises(B200Error, match="not a PagedAttention node"):
        n.compute_paged(_capi.PagedTensors(), 0)
    n.close()
