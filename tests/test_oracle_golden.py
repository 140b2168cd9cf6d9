"""The CPU oracle against the reference's own outputs (tests/golden/*.npz, made by make_golden.py)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import eggroll as oe
from oracle import model as om
from oracle import philox

GOLDEN = Path(__file__).resolve().parent / 'golden'


@pytest.fixture(scope='module')
def params():
    return om.make_params(0)


def test_philox_known_answers():
    """Random123's published Philox4x32-10 known-answer vectors."""
    cases = [((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
             ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
             ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
              (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1))]
    for ctr, key, want in cases:
        got = tuple(int(x) for x in philox.philox4x32_10(*ctr, *key))
        assert got == want


def test_gaussian_stream_moments():
    z = philox.gaussians(0, 1, 5, 0, np.arange(64), 4096)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1) < 0.01
    assert not np.allclose(z[0], z[1])
    z2 = philox.gaussians(0, 1, 5, 0, [3], 10)
    np.testing.assert_array_equal(z2[0], z[3, :10])


def test_param_specs_match_reference():
    f = np.load(GOLDEN / 'forward.npz')
    assert list(f['param_names']) == [n for n, _ in om.PARAM_SPECS]
    assert om.N_PARAMS == 37_749_776


def test_init_matches_reference(params):
    f = np.load(GOLDEN / 'forward.npz')
    for (name, _), ref in zip(om.PARAM_SPECS, f['param_checksums']):
        t = params[name].double()
        got = np.array([t.sum().item(), t.abs().sum().item(), t.pow(2).sum().item()])
        np.testing.assert_allclose(got, ref, rtol=1e-9, atol=1e-9, err_msg=name)


def test_forward_matches_reference(params):
    f = np.load(GOLDEN / 'forward.npz')
    rows = torch.from_numpy(f['tokens'].astype(np.int64))
    with torch.no_grad():
        ce = om.forward(params, rows[:, :-1], rows[:, 1:], reduction='none')
    np.testing.assert_allclose(ce.numpy(), f['ce'], rtol=0, atol=2e-5)


def test_population_matches_reference(params):
    f = np.load(GOLDEN / 'population.npz')
    row = torch.from_numpy(f['tokens'].astype(np.int64))
    draws, sign = oe.member_draws(f['members'], int(f['pairs']), float(f['sigma']), int(f['seed']), int(f['step']))
    with torch.no_grad():
        losses = om.population_losses(params, draws, sign, row[None, :-1], row[None, 1:])
    np.testing.assert_allclose(losses.numpy(), f['losses'], rtol=1e-6, atol=0)


def test_eggroll_step_matches_reference(params):
    """Losses -> z-scored fitness -> sum f eps -> AdamW, against Eggroll.step with injected draws."""
    f = np.load(GOLDEN / 'eggroll_step.npz')
    pairs, sigma, seed, step = int(f['pairs']), float(f['sigma']), int(f['seed']), int(f['step'])
    batch = torch.from_numpy(f['tokens'].astype(np.int64))
    # reference layout with CHUNK = 1: members (2c, 2c+1) run on sequence c
    losses = []
    with torch.no_grad():
        for c in range(2):
            members = np.array([2 * c, 2 * c + 1])
            draws, sign = oe.member_draws(members, pairs, sigma, seed, step)
            losses.append(om.population_losses(params, draws, sign, batch[c:c + 1, :-1], batch[c:c + 1, 1:]))
    losses = torch.cat(losses).numpy()
    np.testing.assert_allclose(losses, f['losses'], rtol=1e-6)
    # the reconstruction from the reference's own losses isolates the update arithmetic
    w = oe.fitness_zscore(f['losses'].astype(np.float32), pairs)
    grads = oe.sum_fe(w, n_fitness=len(f['losses']) // 2, seed=seed, step=step)
    for i, (name, shape) in enumerate(om.PARAM_SPECS):
        g = grads[name]
        ref_sums = f[f'g{i}_sums']
        np.testing.assert_allclose(g.sum().item(), ref_sums[0], rtol=1e-4, atol=1e-4, err_msg=name)
        np.testing.assert_allclose(g.abs().sum().item(), ref_sums[1], rtol=1e-5, err_msg=name)
        if f'g{i}_full' in f:
            np.testing.assert_allclose(g.numpy(), f[f'g{i}_full'], rtol=1e-5, atol=1e-7, err_msg=name)
        else:
            got = g.reshape(-1)[torch.from_numpy(f[f'g{i}_idx'])].numpy()
            np.testing.assert_allclose(got, f[f'g{i}_val'], rtol=1e-5, atol=1e-7, err_msg=name)
    # AdamW's first step from zero state
    lr = float(f['lr'])
    for i, (name, shape) in enumerate(om.PARAM_SPECS):
        p = params[name].double().clone()
        m, v = torch.zeros_like(p), torch.zeros_like(p)
        p0 = p.clone()
        oe.adamw_step(p, grads[name], m, v, 1, lr, betas=tuple(f['betas']))
        d = (p - p0)
        if f'd{i}_full' in f:
            np.testing.assert_allclose(d.numpy(), f[f'd{i}_full'], rtol=2e-3, atol=2e-7, err_msg=name)
        else:
            got = d.reshape(-1)[torch.from_numpy(f[f'g{i}_idx'])].numpy()
            np.testing.assert_allclose(got, f[f'd{i}_val'], rtol=2e-3, atol=2e-7, err_msg=name)


def test_centered_ranks_exact():
    rng = np.random.default_rng(0)
    x = rng.normal(size=1000).astype(np.float32)
    x[10] = x[20]  # a tie: the lower member index ranks first
    x[30] = np.nan
    r = oe.centered_ranks(x)
    assert sorted(r.tolist()) == list(range(1000))
    assert r[30] == 999
    assert r[10] == r[20] - 1
    finite = np.delete(np.arange(1000), 30)
    order = finite[np.argsort(x[finite], kind='stable')]
    np.testing.assert_array_equal(r[order], np.arange(999))
