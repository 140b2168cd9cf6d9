"""Population forward on the GPU against the CPU oracle (same seeded inputs, same counter-based draws).

Tolerance: per-member loss relative error <= 1e-3 (the parity bar for the population forward), and in practice the
bf16-operand / fp32-accumulate path lands within a few 1e-5 of the fp32 oracle.
"""
import numpy as np
import pytest
import torch

from noise_b200.data import zipf_tokens

pytestmark = pytest.mark.gpu

SEED, STEP = 0, 3


@pytest.fixture(scope='module')
def weights():
    from noise_b200.model import Weights
    return Weights('cuda', seed=0)


@pytest.fixture(scope='module')
def params_cpu():
    from oracle import model as om
    return om.make_params(0)


def oracle_losses(params, members, pairs, sigma, rows):
    from oracle import eggroll as oe
    from oracle import model as om
    draws, sign = oe.member_draws(members, pairs, sigma, SEED, STEP)
    with torch.no_grad():
        return om.population_losses(params, draws, sign, rows[:, :-1], rows[:, 1:]).numpy()


@pytest.mark.parametrize('B,T,members,pairs,sigma', [
    (1, 128, 4, 2, 1e-3),
    (2, 256, 4, 2, 2e-3),
    (1, 1152, 2, 1, 1e-3),   # the 1024-token windows bind
    (1, 128, 6, 4, 0.05),    # a large sigma
])
def test_population_matches_oracle(weights, params_cpu, B, T, members, pairs, sigma):
    from noise_b200.population import population_losses
    rows = zipf_tokens(B, T + 1, seed=11 + T)
    got = population_losses(weights, rows[:, :-1], rows[:, 1:], 0, members, pairs, sigma, SEED, STEP).cpu().numpy()
    want = oracle_losses(params_cpu, np.arange(members), pairs, sigma, rows)
    print('gpu', got, 'oracle', want, 'rel', np.abs(got - want) / want)
    np.testing.assert_allclose(got, want, rtol=1e-3)


def test_member_offset_and_chunking(weights):
    """A member range evaluated in one call, in pieces, or with a tiny workspace gives the same losses."""
    from noise_b200.population import population_losses, workspace_bytes
    rows = zipf_tokens(1, 129, seed=5)
    x, y = rows[:, :-1], rows[:, 1:]
    full = population_losses(weights, x, y, 0, 8, 4, 1e-3, SEED, STEP).cpu()
    part = torch.cat([population_losses(weights, x, y, m0, 2, 4, 1e-3, SEED, STEP).cpu() for m0 in range(0, 8, 2)])
    small = population_losses(weights, x, y, 0, 8, 4, 1e-3, SEED, STEP, max_workspace=workspace_bytes(3 * 128)).cpu()
    assert torch.equal(full, part)
    assert torch.equal(full, small)


def test_chunks_wrap_and_odd_starts(weights, params_cpu):
    """Members past 2P wrap onto earlier directions. Pieces that start on odd members, and a workspace
    that forces three-member chunks, give the losses of one call bit for bit (each chunk's draw table
    maps the directions it spans to its own slots). The one call matches the oracle."""
    from noise_b200.population import population_losses, workspace_bytes
    rows = zipf_tokens(1, 129, seed=7)
    x, y = rows[:, :-1], rows[:, 1:]
    members, pairs, sigma = 11, 3, 1e-2
    full = population_losses(weights, x, y, 0, members, pairs, sigma, SEED, STEP).cpu()
    part = torch.cat([population_losses(weights, x, y, m0, n, pairs, sigma, SEED, STEP).cpu()
                      for m0, n in ((0, 3), (3, 5), (8, 3))])
    small = population_losses(weights, x, y, 0, members, pairs, sigma, SEED, STEP,
                              max_workspace=workspace_bytes(3 * 128)).cpu()
    assert torch.equal(full, part)
    assert torch.equal(full, small)
    want = oracle_losses(params_cpu, np.arange(members), pairs, sigma, rows)
    np.testing.assert_allclose(full.numpy(), want, rtol=1e-3)


def test_deterministic(weights):
    from noise_b200.population import population_losses
    rows = zipf_tokens(2, 257, seed=6)
    a = population_losses(weights, rows[:, :-1], rows[:, 1:], 0, 4, 2, 1e-3, SEED, STEP).cpu()
    b = population_losses(weights, rows[:, :-1], rows[:, 1:], 0, 4, 2, 1e-3, SEED, STEP).cpu()
    assert torch.equal(a, b)
