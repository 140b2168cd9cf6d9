"""noise_reassemble (DUST.reassemble, train/val/run.py:465-471: g = einsum('btd,bti->di', err, x)) against
a float64 product of the same inputs.

Tolerances: tile-aligned shapes run on tf32 tensor cores, as the reference's float32 einsum does
under set_float32_matmul_precision('high'): relative L2 error <= 2e-3 and cosine >= 0.99999 (tf32
keeps 10 of fp32's 23 mantissa bits of each operand); the 8 x 32 ve_gate shape runs in fp32 on CUDA
cores: relative error <= 1e-5. Inputs normalised by the kernel (x_norm) are compared against the
float64 RMS norm of the same rows.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('K,out,inp,x_ld,dtype,norm', [
    (16384, 512, 512, 512, torch.float32, True),     # attention projections / mlp.c_fc input shape
    (16384, 2048, 512, 512, torch.float32, True),    # mlp.c_fc
    (4096, 512, 2048, 2048, torch.bfloat16, False),  # mlp.c_proj from the bf16 hidden
    (2048, 4096, 512, 512, torch.float32, True),     # lm_head
    (16384, 8, 32, 512, torch.float32, True),        # ve_gate: first 32 channels of the normalised row
    (1024, 512, 512, 512, torch.bfloat16, False),    # attn.c_proj from the bf16 attention output
])
def test_reassemble_matches_float64(K, out, inp, x_ld, dtype, norm):
    from noise_b200.dust import contract
    g = torch.Generator(device='cuda').manual_seed(K + out + inp)
    err = torch.randn(K, out, device='cuda', generator=g) * 1e-2
    x = (torch.randn(K, x_ld, device='cuda', generator=g) * 3).to(dtype)
    got = contract(err, x, norm, inp if inp != x_ld else None).double()
    xd = x.double()
    if norm:
        xd = xd * torch.rsqrt(xd.pow(2).mean(-1, keepdim=True) + torch.finfo(torch.float32).eps)
    want = err.double().t() @ xd[:, :inp]
    rel = ((got - want).norm() / want.norm()).item()
    cos = torch.nn.functional.cosine_similarity(got.reshape(-1), want.reshape(-1), dim=0).item()
    print(K, out, inp, dtype, norm, 'rel', rel, 'cos', cos)
    tc = out % 128 == 0 and inp % 256 == 0
    assert rel <= (2e-3 if tc else 1e-5) and cos >= 0.99999
