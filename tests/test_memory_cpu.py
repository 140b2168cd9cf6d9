"""The credit memory's host logic on CPU (noise_b200.dust.CreditMemory, train/val/run.py:281-330).

- every site's M = S (P + ridge mean(diag P) I)^-1 comes from one solve over all sites' right-hand
  sides; each equals a solve of its own site to fp32 rounding (rtol 1e-5);
- the solved matrices follow remember(): after new estimates P and S change, and so does M;
- DUST.step's matmul-precision scope restores the caller's setting, also when the step raises.
"""
import pytest
import torch


def _memory(seed=0, sites=(('a', 8), ('b', 16), ('c', 4)), keys=64, tokens=256):
    from noise_b200.dust import CreditMemory
    g = torch.Generator().manual_seed(seed)
    mem = CreditMemory()
    credit = torch.randn(tokens, keys, generator=g)
    mem.estimates = {n: torch.randn(tokens, d, generator=g) for n, d in sites}
    mem.remember(credit, float(tokens))
    return mem, credit, g


def _own_solve(mem, name):
    P = mem.P.double()
    A = P + mem.ridge * P.diagonal().mean() * torch.eye(len(P), dtype=torch.float64)
    return torch.linalg.solve(A, mem.S[name].double().T).T


def test_batched_solve_matches_each_site():
    mem, _, _ = _memory()
    for name in ('a', 'b', 'c'):
        got = mem.matrix(name)
        assert got.shape == mem.S[name].shape
        torch.testing.assert_close(got.double(), _own_solve(mem, name), rtol=1e-5, atol=1e-6)
    assert mem.matrix('missing') is None


def test_matrices_follow_remember():
    mem, credit, g = _memory()
    before = mem.matrix('a').clone()
    mem.estimates = {'a': torch.randn(credit.shape[0], 8, generator=g), 'd': torch.randn(credit.shape[0], 2, generator=g)}
    mem.remember(credit * 1.5, float(credit.shape[0]))
    after = mem.matrix('a')
    assert not torch.allclose(before, after)
    torch.testing.assert_close(after.double(), _own_solve(mem, 'a'), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(mem.matrix('d').double(), _own_solve(mem, 'd'), rtol=1e-5, atol=1e-6)


def test_retrieve_uses_the_solved_matrices():
    mem, credit, _ = _memory()
    out = mem.retrieve(credit, ['a', 'b', 'missing'])
    assert set(out) == {'a', 'b'}
    for name in ('a', 'b'):
        torch.testing.assert_close(out[name].double(), credit.double() @ _own_solve(mem, name).T, rtol=1e-4,
                                   atol=1e-5)


def test_precision_scope_restores_the_callers_setting():
    from noise_b200.dust import reference_matmul_precision
    prev = torch.get_float32_matmul_precision()
    try:
        torch.set_float32_matmul_precision('highest')
        with reference_matmul_precision():
            assert torch.get_float32_matmul_precision() == 'high'
        assert torch.get_float32_matmul_precision() == 'highest'
        with pytest.raises(RuntimeError):
            with reference_matmul_precision():
                raise RuntimeError('step failed')
        assert torch.get_float32_matmul_precision() == 'highest'
    finally:
        torch.set_float32_matmul_precision(prev)
