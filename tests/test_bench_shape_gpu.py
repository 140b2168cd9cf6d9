"""Parity at the benchmarked shape, and rank agreement of near-tied members.

1. The bench configuration: 1,024 rank-1 members (512 directions, sigma 1e-3),
   every member on the same 8 sequences of 2048 tokens, the default 32 GiB workspace, so members run
   in 6 equal chunks of 171 and each chunk's draw table spans 86 directions. Members at a chunk's
   first and last rows, in the middle of a chunk and at the end of the population are checked
   against the float32 CPU oracle (train/val/eggroll.py:66-103 restated; pinned to the reference by
   tests/golden/population.npz). Tolerance: relative 1e-3 per member loss (the parity bar).
2. Rank agreement (the fitness ranks are exact functions of the losses, so what must hold is that
   the bf16-operand losses order members as the float32 losses do): 64 members (32 antithetic pairs)
   at sigma 1e-3 on one sequence of 512 tokens. Spearman rho of the member losses >= 0.99, and a pair's
   antithetic difference L[2i+1] - L[2i] may change sign only when the oracle's |difference| is below
   5e-5 (a near tie within the bf16 rounding of the two losses); the flip rate is printed.
"""
import numpy as np
import pytest
import torch

from noise_b200.data import zipf_tokens

pytestmark = pytest.mark.gpu

SEED, STEP = 0, 1


@pytest.fixture(scope='module')
def setup():
    from noise_b200.model import Weights
    from oracle import model as om
    return Weights('cuda', seed=0), om.make_params(0)


def _oracle(params, members, pairs, sigma, x, y):
    from oracle import eggroll as oe
    from oracle import model as om
    draws, sign = oe.member_draws(np.asarray(members), pairs, sigma, SEED, STEP)
    with torch.no_grad():
        return om.population_losses(params, draws, sign, x, y).numpy()


def test_bench_shape_members_match_oracle(setup):
    from noise_b200 import population
    w, params = setup
    rows = zipf_tokens(8, 2049, seed=1)
    x, y = rows[:, :-1], rows[:, 1:]
    members, pairs, sigma = 1024, 512, 1e-3
    budget = 32 << 30
    chunk = population.units_that_fit(8 * 2048, members, budget, pairs)
    assert chunk == 171
    got = population.population_losses(w, x, y, 0, members, pairs, sigma, SEED, STEP, max_workspace=budget)
    got = got.cpu().numpy()
    picks = [0, chunk - 1, chunk, 2 * chunk + 85, members - 1]
    want = _oracle(params, picks, pairs, sigma, x, y)
    rel = np.abs(got[picks] - want) / want
    print('members', picks, 'gpu', got[picks], 'oracle', want, 'rel', rel)
    assert np.all(rel <= 1e-3)


def test_rank_agreement_near_ties(setup):
    from noise_b200.population import population_losses
    w, params = setup
    rows = zipf_tokens(1, 513, seed=17)
    x, y = rows[:, :-1], rows[:, 1:]
    members, pairs, sigma = 64, 32, 1e-3
    got = population_losses(w, x, y, 0, members, pairs, sigma, SEED, STEP).cpu().double().numpy()
    want = _oracle(params, list(range(members)), pairs, sigma, x, y).astype(np.float64)
    rg, rw = np.argsort(np.argsort(got)), np.argsort(np.argsort(want))
    rho = 1 - 6 * np.sum((rg - rw) ** 2) / (members * (members ** 2 - 1))
    dg, dw = got[1::2] - got[0::2], want[1::2] - want[0::2]
    flips = np.sign(dg) != np.sign(dw)
    print(f'spearman {rho:.5f}; pair flips {flips.sum()}/{len(flips)}; |diff| oracle median {np.median(np.abs(dw)):.2e}, '
          f'gpu-oracle loss error max {np.max(np.abs(got - want)):.2e}; flipped |diff| {np.abs(dw[flips])}')
    assert rho >= 0.99
    assert np.all(np.abs(dw[flips]) < 5e-5)
