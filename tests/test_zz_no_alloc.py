"""b200_paged_attention_static_scratch: the entry point for callers that cannot allocate device
memory (a runtime that hands over only the tensors it owns, a serving loop that forbids device
allocations after start-up, a cgo/JNI binding without a CUDA allocator).

Its scratch is a 32 MiB static device array instead of a caller workspace.  The test calls it
through the C ABI twice in a row and checks each result against b200_paged_attention with a
caller workspace, within the decode tolerance used by the other parity tests (max-abs 2e-3,
caches bit-exact).  The file is named to be collected last and passes alone in a fresh
process as well as after the other tests.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from onnxruntime_ep_b200 import _capi, paged  # noqa: E402


def _decode_case(seed, B=24, H=32, KV=8, D=128, bs=16, nb=4096):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rng = np.random.default_rng(seed)
    L = rng.integers(1, 3000, size=B, endpoint=True)
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
    return dict(
        q=mk(B, H * D), k=mk(B, KV * D), v=mk(B, KV * D),
        kc=mk(nb, bs, KV, D), vc=mk(nb, bs, KV, D),
        cum=torch.arange(B + 1, dtype=torch.int32),
        past=torch.from_numpy((L - 1).astype(np.int32)),
        bt=torch.from_numpy(bt), H=H, KV=KV)


def _run(case, static):
    kc, vc = case["kc"].clone(), case["vc"].clone()
    p, keep, out = paged.build_params(
        case["q"], case["k"], case["v"], kc, vc, case["cum"], case["past"], case["bt"],
        num_heads=case["H"], kv_num_heads=case["KV"])
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    p.device_status = ctypes.c_void_p(status.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if static:
        p.workspace = None  # ignored by the static-scratch entry point
        p.workspace_bytes = 0
        _capi.check(_capi.LIB.b200_paged_attention_static_scratch(ctypes.byref(p), stream))
    else:
        _capi.check(_capi.LIB.b200_paged_attention(ctypes.byref(p), stream))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    del keep
    return out.float().cpu(), kc.cpu(), vc.cpu()


def test_static_scratch_matches_workspace_entry_twice():
    case = _decode_case(11)
    want, wkc, wvc = _run(case, static=False)
    for _ in range(2):  # the second call reuses the scratch left by the first
        got, kc, vc = _run(case, static=True)
        assert float((got - want).abs().max()) <= 2e-3
        assert torch.equal(kc.view(torch.int16), wkc.view(torch.int16))
        assert torch.equal(vc.view(torch.int16), wvc.view(torch.int16))


def test_static_scratch_rejects_calls_beyond_its_size():
    # RoPE scratch for a long prefill batch (nt x (H + KV) x d x 2 bytes) exceeds 32 MiB.
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
