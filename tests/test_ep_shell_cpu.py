"""The ORT plugin-EP glue (csrc/ep_shell.cpp) driven by the fake ORT host, without a GPU.

Covers what ORT's host does before any tensor moves: CreateEpFactories (version check, room for
a factory), the factory's names and ids, GetSupportedDevices (one EP device on the NVIDIA GPU
with the "B200" device memory registered), CreateEp (exactly one device, strict ep.b200.*
session options), GetCapability (PagedAttention / GroupQueryAttention claimed one node per
fusion, declines with the claim predicate's reason), Compile (name-matched input mapping, declined
forms rejected), the allocator choice, the data transfer's CanCopy, and that nothing the fake
host hands out leaks.  A Compute without a GPU must fail loudly rather than fall back.
"""

import pytest

import ort_host as oh
from ort_host import BF16, F16, F32, GPU, CPU, I32, NVIDIA


@pytest.fixture
def host():
    h = oh.Host()
    yield h
    h.close()


@pytest.fixture
def ep(host):
    rc, n, _ = host.devices([(CPU, 0), (GPU, NVIDIA)])
    assert rc == 0 and n == 1
    assert host.create_ep() == 0, oh.last_error()
    return host


def test_factory_identity(host):
    assert host.string("name") == "B200ExecutionProvider"
    assert host.string("vendor") == "onnxruntime-ep-b200"
    assert host.string("version") == "0.31.0"
    assert host.vendor_id() == 0x10DE
    assert not host.stream_aware()


def test_registration_name_is_the_factory_name():
    h = oh.Host(registration_name="MyB200")
    try:
        assert h.string("name") == "MyB200"
    finally:
        h.close()


def test_older_runtime_is_refused():
    with pytest.raises(RuntimeError, match="requires ONNX Runtime 1.31 or newer"):
        oh.Host(max_api_version=30)
    assert oh.last_error()[0] == oh.ORT_INVALID_ARGUMENT


def test_factories_need_room():
    assert oh.create_factories_raw(0) == oh.ORT_INVALID_ARGUMENT
    assert "room for one OrtEpFactory" in oh.last_error()[1]
    assert oh.create_factories_raw(1) == 0


def test_supported_devices_pick_the_nvidia_gpu(host):
    rc, n, infos = host.devices([(CPU, 0), (GPU, 0x1002), (GPU, NVIDIA), (GPU, NVIDIA)])
    assert (rc, n, infos) == (0, 1, 1)
    assert host.device_memory() == ("B200", 1, NVIDIA, 0)


def test_no_gpu_means_no_ep_device(host):
    assert host.devices([(CPU, 0)]) == (0, 0, 0)
    assert host.devices([(GPU, 0x1002)]) == (0, 0, 0)


def test_create_ep_needs_exactly_one_device(host):
    host.devices([(GPU, NVIDIA)])
    assert host.create_ep(num_devices=2) == oh.ORT_INVALID_ARGUMENT
    assert "expects exactly one device" in oh.last_error()[1]


@pytest.mark.parametrize("key,value,needle", [
    ("ep.b200.check_status", "yes", "ep.b200.check_status"),
    ("ep.b200.kv_pool_bytes", "12MB", "ep.b200.kv_pool_bytes"),
    ("ep.b200.force_generic", "2", "expected 0 or 1"),
])
def test_create_ep_rejects_malformed_options(host, key, value, needle):
    host.devices([(GPU, NVIDIA)])
    assert host.create_ep({key: value}) == oh.ORT_INVALID_ARGUMENT
    assert needle in oh.last_error()[1]


def test_create_ep_device_must_match_the_registered_memory(host):
    host.devices([(GPU, NVIDIA)])
    assert host.create_ep({"ep.b200.device_id": "1"}) == oh.ORT_INVALID_ARGUMENT
    assert "differs from the device" in oh.last_error()[1]


def test_ep_identity_and_memory(ep):
    assert ep.ep_name() == "B200ExecutionProvider"
    assert ep.default_memory() == (1, NVIDIA, 0)


def test_capability_claims_attention_nodes_one_per_fusion(ep):
    g = oh.Graph()
    try:
        oh.paged_node(g, "pa0")                                            # claimed
        oh.paged_node(g, "pa1", attrs={"is_causal": 2})                    # declined
        oh.gqa_node(g, "gqa0")                                             # claimed
        oh.gqa_node(g, "gqa1", attrs={"qk_output": 1})                     # declined
        g.node("MatMul", "mm", domain="")                                  # not an attention node
        g.node("PagedAttention", "other_domain", domain="com.example")     # not ours
        oh.paged_node(g, "pa2", dt=BF16, packed=True, outputs=3)           # claimed
        rc, claimed, drop = ep.capability(g)
        assert rc == 0, oh.last_error()
        assert claimed == [0, 2, 6]
        assert drop == 0  # constant initializers stay inputs of the fused node
        report = ep.report().splitlines()
        assert report[0] == "pa0: claimed"
        assert report[1] == "pa1: declined: is_causal must be 0 or 1"
        assert report[2] == "gqa0: claimed"
        assert report[3].startswith("gqa1: declined: qk_output")
        assert report[4] == "pa2: claimed"
        assert len(report) == 5
    finally:
        g.close()


def test_capability_reads_string_and_float_attributes(ep):
    g = oh.Graph()
    try:
        oh.paged_node(g, "latent", attrs={"kv_cache_layout": "LATENT"})
        oh.paged_node(g, "bad_layout", attrs={"kv_cache_layout": "PAGED"})
        oh.paged_node(g, "softcap", attrs={"softcap": 30.0, "scale": 0.125, "local_window_size": 64})
        rc, claimed, _ = ep.capability(g)
        assert rc == 0 and claimed == [2]
        lines = ep.report().splitlines()
        assert "LATENT" in lines[0] and "declined" in lines[0]
        assert lines[1] == "bad_layout: declined: kv_cache_layout must be SEPARATE or LATENT"
    finally:
        g.close()


def test_values_without_type_information_are_declined(ep):
    g = oh.Graph()
    try:
        n = g.node("PagedAttention", "untyped")
        n.input_untyped("q").input("k", F16, (-1, 32)).input("v", F16, (-1, 32))
        n.input("kc", F16, (8, 4, 2, 16)).input("vc", F16, (8, 4, 2, 16))
        n.input("cum", I32, (3,)).input("past", I32, (2,)).input("bt", I32, (2, 4))
        n.output("out", F16, (-1, 64))
        n.attr("num_heads", 4).attr("kv_num_heads", 2)
        rc, claimed, _ = ep.capability(g)
        assert rc == 0 and claimed == []
        assert "untyped: declined" in ep.report()
    finally:
        g.close()


def test_compile_maps_inputs_by_name(ep):
    g = oh.Graph()
    try:
        oh.paged_node(g, "pa")
        oh.gqa_node(g, "gqa", rotary=(64, 8), attrs={"do_rotary": 1})
        assert ep.compile(g, 0) == 0, oh.last_error()
        assert ep.compile(g, 0, reverse=True) == 1, oh.last_error()
        assert ep.compile(g, 1) == 2, oh.last_error()
    finally:
        g.close()


def test_compile_rejects_a_declined_node(ep):
    g = oh.Graph()
    try:
        oh.paged_node(g, "pa", attrs={"is_causal": 5})
        assert ep.compile(g, 0) == -1
        code, msg = oh.last_error()
        assert code == oh.ORT_EP_FAIL and "not claimed" in msg and "is_causal" in msg
    finally:
        g.close()


def test_compute_without_a_gpu_fails_loudly(ep):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; the GPU tests run Compute")
    import numpy as np

    g = oh.Graph()
    ctx = oh.KernelContext()
    try:
        oh.paged_node(g, "pa")
        idx = ep.compile(g, 0)
        q = np.zeros((2, 64), np.float16)
        ctx.input("pa.query", F16, q.shape, oh.ptr_of(q), q.nbytes)
        assert ep.compute(idx, ctx) == oh.ORT_EP_FAIL
        assert "B200" in oh.last_error()[1]
    finally:
        ctx.close()
        g.close()


def test_allocator_only_for_the_b200_memory(host):
    assert host.allocator("Cpu") == 0
    assert host.allocator("B200") == 1
    assert host.allocator_name() == "B200"


def test_data_transfer_copies_between_host_and_the_ep_device(host):
    assert host.transfer() == 0
    assert host.can_copy("b200", "cpu") and host.can_copy("cpu", "b200") and host.can_copy("b200", "b200")
    assert not host.can_copy("cpu", "cpu")
    assert not host.can_copy("other", "b200") and not host.can_copy("b200", "other")
    assert not host.can_copy("b200", "cpu", device=1)  # another ordinal is not this EP's memory


def test_data_transfer_checks_shapes(host):
    import numpy as np

    host.transfer()
    a = np.zeros(8, np.float32)
    b = np.zeros(4, np.float32)
    assert host.copy(F32, (8,), oh.ptr_of(a), a.nbytes, (4,), oh.ptr_of(b), b.nbytes) == oh.ORT_INVALID_ARGUMENT
    assert "matching shapes" in oh.last_error()[1]


def test_nothing_leaks():
    h = oh.Host()
    h.devices([(GPU, NVIDIA)])
    h.create_ep({"ep.b200.check_status": "0"})
    g = oh.Graph()
    oh.paged_node(g, "pa")
    h.capability(g)
    h.compile(g, 0)
    h.allocator("B200")
    h.transfer()
    h.close()
    g.close()
    assert oh.live_counts() == (0, 0)
