"""The tcgen05 GEMM engine on its own, against torch's fp32 matmul of the same bf16 operands."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def run_gemm(A, B, out_bf16=False, alpha=1.0):
    from noise_b200 import _lib
    M, K = A.shape
    N = B.shape[0]
    C = torch.empty(M, N, device=A.device, dtype=torch.bfloat16 if out_bf16 else torch.float32)
    status = torch.zeros(1, dtype=torch.int32, device=A.device)
    _lib.call('noise_gemm_bf16', A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, alpha, int(out_bf16),
              status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert status.item() == 0, f'device status {status.item()}'
    return C


@pytest.mark.parametrize('M,N,K', [(128, 256, 64), (256, 512, 512), (128 * 150, 1536, 512), (4096, 512, 2048),
                                   (1024, 4096, 512)])
def test_gemm_matches_fp32(M, N, K):
    g = torch.Generator(device='cuda').manual_seed(M + N + K)
    A = torch.randn(M, K, device='cuda', generator=g).bfloat16()
    B = torch.randn(N, K, device='cuda', generator=g).bfloat16()
    C = run_gemm(A, B)
    ref = A.float() @ B.float().t()
    err = (C - ref).abs()
    if not torch.allclose(C, ref, rtol=1e-4, atol=1e-3):
        bad = (err > 1e-3 + 1e-4 * ref.abs()).nonzero()
        print('mismatches', bad.shape[0], 'first', bad[:8].tolist())
        print('C[:2,:8]', C[:2, :8].tolist())
        print('ref[:2,:8]', ref[:2, :8].tolist())
    torch.testing.assert_close(C, ref, rtol=1e-4, atol=1e-3)


def test_gemm_bf16_out_and_alpha():
    g = torch.Generator(device='cuda').manual_seed(7)
    A = torch.randn(512, 512, device='cuda', generator=g).bfloat16()
    B = torch.randn(256, 512, device='cuda', generator=g).bfloat16()
    C = run_gemm(A, B, out_bf16=True, alpha=0.5)
    ref = (0.5 * (A.float() @ B.float().t())).bfloat16()
    torch.testing.assert_close(C.float(), ref.float(), rtol=1e-2, atol=1e-2)
