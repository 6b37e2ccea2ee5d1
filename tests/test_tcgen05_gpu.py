"""Known-answer test of the tcgen05 building blocks (TMA, shared-memory matrix descriptors in
K-major and MN-major 128B-swizzled layouts, tcgen05.mma into tensor memory with the A operand
in shared or in tensor memory, tcgen05.st / tcgen05.ld) against torch.matmul."""

import ctypes

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from onnxruntime_ep_b200 import _capi  # noqa: E402


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tcgen05_products(dtype):
    g = torch.Generator(device="cuda").manual_seed(0)
    a, b, v = (torch.randn(128, 128, generator=g, device="cuda").to(dtype) for _ in range(3))
    c_qk = torch.zeros(128, 128, device="cuda")
    c_pv = torch.zeros(128, 128, device="cuda")
    c_ts = torch.zeros(128, 128, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    dt = _capi.DTYPE_BFLOAT16 if dtype == torch.bfloat16 else _capi.DTYPE_FLOAT16
    s = torch.cuda.current_stream()
    _capi.check(_capi.LIB.b200_selftest_tcgen05(
        dt, a.data_ptr(), b.data_ptr(), v.data_ptr(), c_qk.data_ptr(), c_pv.data_ptr(),
        c_ts.data_ptr(), status.data_ptr(), ctypes.c_void_p(s.cuda_stream)))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    want_qk = a.float() @ b.float().T
    want_pv = a.float() @ v.float()
    torch.testing.assert_close(c_qk, want_qk, rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(c_pv, want_pv, rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(c_ts, want_pv, rtol=1e-4, atol=1e-3)
