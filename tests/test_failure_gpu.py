"""Failure detection on the GPU without a fault: a bounded wait that runs out.

noise_selftest_wait_timeout launches the GEMM engine with a producer that arms its operand barrier
but issues no copy and a wait budget of about 10 ms. The MMA warp's wait runs out; the kernel must
record NOISE_WAIT_TIMEOUT in the status word and end through its abort path (no role left waiting,
tensor memory freed), so that the call finishes within a bound and the context stays usable: a
normal GEMM launched afterwards on the same stream must give the right product.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_timeout_sets_status_and_context_survives():
    from noise_b200 import _lib
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    a = torch.zeros(128, 64, dtype=torch.bfloat16, device='cuda')
    b = torch.zeros(256, 64, dtype=torch.bfloat16, device='cuda')
    status = torch.zeros(1, dtype=torch.int32, device='cuda')
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert lib.noise_selftest_wait_timeout(a.data_ptr(), b.data_ptr(), status.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(status.item()) == 3, 'NOISE_WAIT_TIMEOUT expected'
    assert elapsed < 5.0, elapsed
    # the context is intact: a normal product on the same stream
    g = torch.Generator(device='cuda').manual_seed(1)
    A = torch.randn(256, 128, device='cuda', generator=g).bfloat16()
    B = torch.randn(256, 128, device='cuda', generator=g).bfloat16()
    C = torch.empty(256, 256, device='cuda')
    st = torch.zeros(1, dtype=torch.int32, device='cuda')
    _lib.call('noise_gemm_bf16', A.data_ptr(), B.data_ptr(), C.data_ptr(), 256, 256, 128, 1.0, 0, st.data_ptr(),
              stream)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    torch.testing.assert_close(C, A.float() @ B.float().t(), rtol=1e-3, atol=1e-3)
