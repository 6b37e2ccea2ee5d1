"""b200_paged_attention_static_scratch: the entry point for callers that cannot allocate device
memory.

Some callers of this library may not call cudaMalloc when they run attention: a host runtime
that hands the kernels only the tensors it already owns, a serving loop that forbids device
allocations after start-up (so memory use stays fixed and no allocation can stall or fail
mid-request), or a cgo/JNI binding without a CUDA allocator of its own.  This entry point takes
its scratch from a 32 MiB static device array instead of a caller workspace.

The tests call it through the C ABI, two calls in a row each time (the second reuses what the
first left in the shared array), and check:
* the output against b200_paged_attention with a caller workspace (max-abs 2e-3, the decode
  tolerance; caches bit-exact) and against the CPU oracle (error beyond the bf16 output's own
  rounding at most 2e-3), at a small size, at head size 256 and at the full config-3 size;
* that the second call changes the device's free memory by nothing (it allocates nothing);
* that without a caller status word, b200_read_status_static_scratch still reports device-side
  metadata errors;
* that a call needing more than 32 MiB is rejected with B200_ERR_WORKSPACE.
The file is named to be collected last, and passes alone in a fresh process as well as after
the other tests.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import baseline_cases as bc  # noqa: E402
from onnxruntime_ep_b200 import _capi, paged  # noqa: E402


def _decode_case(seed, B=24, H=32, KV=8, D=128, bs=16, nb=4096):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rng = np.random.default_rng(seed)
    L = rng.integers(1, 3000, size=B, endpoint=True).astype(np.int64)
    maxb = int(-(-int(L.max()) // bs))
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((B, maxb), np.int32)
    off = 0
    for b in range(B):
        n = -(-int(L[b]) // bs)
        bt[b, :n] = perm[off:off + n]
        off += n
    s = 1.0 / np.sqrt(D)
    mk = lambda *shape: (torch.randn(*shape, generator=g, device="cuda") * s).to(torch.bfloat16)
    return dict(H=H, KV=KV, D=D, q=mk(B, H * D), k=mk(B, KV * D), v=mk(B, KV * D),
                kc=mk(nb, bs, KV, D), vc=mk(nb, bs, KV, D), cum=np.arange(B + 1, dtype=np.int32),
                past=(L - 1).astype(np.int32), bt=bt, L=L, fp8=False, tol=2e-3)


def _fresh(case, kc0, vc0):
    """The case with its caches reset to the pre-call snapshots."""
    c = dict(case)
    c["kc"], c["vc"] = kc0.clone(), vc0.clone()
    return c


def _compare(case, sample_n=16):
    """Workspace call once, static-scratch call twice; all against each other and the oracle."""
    kc0, vc0 = case["kc"].clone(), case["vc"].clone()
    ref_case = _fresh(case, kc0, vc0)
    want = bc.run(ref_case).float()
    torch.cuda.synchronize()
    for call in range(2):
        c = _fresh(case, kc0, vc0)
        p, keep, out = bc.prepare(c)  # every tensor of the call exists before the measurement
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        bc.call(p, static_scratch=True)
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        del keep
        if call == 1:  # the first call may load the module that holds the array
            assert free_after == free_before, "the static-scratch call changed the device's free memory"
        assert float((out.float() - want).abs().max()) <= 2e-3
        assert bc.caches_equal(c["kc"], ref_case["kc"]) and bc.caches_equal(c["vc"], ref_case["vc"])
        idx = bc.sample(case["L"], n=sample_n, seed=call)
        bc.check_sampled(c, out, idx, kc0, vc0)
        del c, out


def test_static_scratch_matches_workspace_entry_and_oracle_twice():
    _compare(_decode_case(11))


def test_static_scratch_head_size_256():
    _compare(_decode_case(12, B=16, H=8, KV=2, D=256, nb=2048), sample_n=8)


def test_static_scratch_config3_size():
    _compare(bc.config3())


def test_static_scratch_status_without_device_status():
    """No caller status word: the word lives in the static array, and the static-scratch status
    read turns a bad device-side block id into the reference's message."""
    case = _decode_case(13, B=4)
    out = bc.run(case, static_scratch=True)  # also reads the status: a good call reports OK
    assert out is not None
    bad = dict(case, bt=np.full_like(case["bt"], 10_000))  # pool has 4096 blocks
    dev = case["kc"].device
    p, keep, _ = paged.build_params(
        bad["q"], bad["k"], bad["v"], bad["kc"], bad["vc"], torch.from_numpy(bad["cum"]).to(dev),
        torch.from_numpy(bad["past"]).to(dev), torch.from_numpy(bad["bt"]).to(dev), num_heads=bad["H"],
        kv_num_heads=bad["KV"])  # device metadata only: the checks run on the device
    p.workspace, p.workspace_bytes = None, 0
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _capi.check(_capi.LIB.b200_paged_attention_static_scratch(ctypes.byref(p), stream))
    rc = _capi.LIB.b200_read_status_static_scratch(ctypes.byref(p), stream)
    assert rc == _capi.B200_ERR_FAIL
    assert "invalid physical block" in _capi.LIB.b200_last_error().decode()
    # b200_read_status has no workspace to look in
    assert _capi.LIB.b200_read_status(ctypes.byref(p), stream) == _capi.B200_ERR_INVALID_ARGUMENT
    del keep
    # the next good call clears the word
    bc.run(case, static_scratch=True)


def test_static_scratch_rejects_calls_beyond_its_size():
    # RoPE rows of a long prefill batch (2 x nt x (H + KV) x d bytes) exceed 32 MiB.
    nt, H, KV, D = 8192, 32, 8, 128
    q = torch.zeros(nt, H * D, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(nt, KV * D, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(nt // 16 + 1, 16, KV, D, dtype=torch.bfloat16, device="cuda")
    cos = torch.ones(nt, D // 2, dtype=torch.bfloat16, device="cuda")
    p, keep, out = paged.build_params(
        q, k, k, kc, kc.clone(), torch.tensor([0, nt], dtype=torch.int32),
        torch.tensor([0], dtype=torch.int32),
        torch.arange(nt // 16 + 1, dtype=torch.int32).reshape(1, -1),
        num_heads=H, kv_num_heads=KV, do_rotary=1, cos_cache=cos, sin_cache=cos)
    rc = _capi.LIB.b200_paged_attention_static_scratch(
        ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _capi.B200_ERR_WORKSPACE
    assert "static scratch" in _capi.LIB.b200_last_error().decode()
