"""The oracle's credit memory (memory_matrix, retrieve, remember, calibrate) and prior-corrected
direct_errors against the reference's DUST (tests/golden/memory.npz). Float64 oracle vs the float32
reference: relative tolerance 1e-4 on the memory and 1e-3 on the rerun-based errors."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import dust as od
from oracle import model as om

GOLDEN = Path(__file__).resolve().parent / 'golden'
SEED, STEP = 0, 1
SITES = ['transformer.h.1.attn.c_proj', 'transformer.h.1.mlp.c_proj', 'transformer.h.6.mlp.c_fc', 'o@0']


def estimates(b, t, round_, seed=31):
    g = torch.Generator().manual_seed(seed + round_)
    width = {'transformer.h.6.mlp.c_fc': 2048}
    return {s: torch.randn(b, t, width.get(s, 512), generator=g) * 0.01 for s in SITES}


def check(f, key, got, rtol, atol):
    got = np.asarray(got, dtype=np.float64)
    if key in f:
        np.testing.assert_allclose(got, f[key], rtol=rtol, atol=atol, err_msg=key)
        return
    flat = got.reshape(-1)
    np.testing.assert_allclose(flat[f[key + '__idx']], f[key + '__val'], rtol=rtol, atol=atol, err_msg=key)
    sums = np.array([flat.sum(), np.abs(flat).sum(), (flat ** 2).sum()])
    np.testing.assert_allclose(sums[1:], f[key + '__sums'][1:], rtol=max(rtol, 1e-6), err_msg=key)


@pytest.fixture(scope='module')
def memory():
    from noise_b200.data import zipf_tokens
    f = np.load(GOLDEN / 'memory.npz')
    p = om.make_params(0)
    rows = zipf_tokens(2, 129, seed=4)
    x, y = rows[:, :-1].contiguous(), rows[:, 1:].contiguous()
    y[1, 5] = -1
    b, t = x.shape
    with torch.no_grad():
        cap = od.capture(p, x)
        c = od.coordinate_differences(cap['raw'].double(), y, 0.1)
    valid = int((y >= 0).sum())
    P, S = None, {}
    for r in range(2):
        P, S = od.remember(P, S, c, estimates(b, t, r), valid, 0.9)
    M = {s: od.memory_matrix(S[s], P, 0.1) for s in SITES}
    return f, p, cap, x, y, c, P, S, M


def test_memory_writes_and_reads_match_reference(memory):
    f, p, cap, x, y, c, P, S, M = memory
    check(f, 'P', P.numpy(), 1e-4, 1e-9)
    for k, s in enumerate(SITES):
        check(f, f'S_{k}', S[s].numpy(), 1e-4, 1e-9)
        check(f, f'M_{k}', M[s].numpy(), 1e-3, 1e-7)
        check(f, f'r_{k}', (c @ M[s].T).numpy(), 1e-3, 1e-8)


def test_calibration_matches_reference(memory):
    f = memory[0]
    cal = {}
    for r in range(2):
        fits = {s: tuple(v) for s, v in zip(SITES, f[f'fits_{r}'].astype(np.float64))}
        cal, alpha = od.calibrate(cal, fits, 0.8)
    np.testing.assert_allclose([alpha[s] for s in SITES], f['alpha'], rtol=1e-5)


CASES = {
    'writers': (['transformer.h.1.attn.c_proj', 'transformer.h.1.mlp.c_proj'], ['attn', 'mlp']),
    'hidden': (['transformer.h.6.mlp.c_fc'], ['fc']),
    'hub': (['o@0'], ['o']),
}


@pytest.mark.parametrize('name', list(CASES))
def test_prior_direct_errors_match_reference(memory, name):
    f, p, cap, x, y, c, P, S, M = memory
    alpha = dict(zip(SITES, f['alpha']))
    sites, keys = CASES[name]
    draws, sigma, entry, gamma = f[f'pe_{name}_meta']
    draws, entry = int(draws), int(entry)
    b, t = x.shape
    a, priors, ret = {}, {}, {}
    with torch.no_grad():
        logits = om.soft_cap(cap['raw'])
        clean = torch.nn.functional.cross_entropy(logits.reshape(-1, om.VOCAB), y.reshape(-1), ignore_index=-1,
                                                  reduction='none').view_as(y)
        for site, key in zip(sites, keys):
            d = 2048 if key == 'fc' else 512
            a[site] = od.site_draws(SEED, STEP, site, np.arange(draws), b, t, d, draws)
            ret[site] = c @ M[site].T
            priors[site] = alpha[site] * ret[site]
            if key == 'fc':
                live = (cap['fc_pre'][entry] > 0).double()
                a[site] = a[site] * live.float()
                priors[site] = priors[site] * live
        jitter = {key: sigma * a[site] for site, key in zip(sites, keys)}
        perturbed = od.rerun(p, cap, x, y.clamp(min=0), draws, entry, jitter) * (y >= 0)
    errs = od.direct_errors(clean, perturbed, a, float(sigma), n=16, gamma=float(gamma), priors=priors)
    kept = 1 - 1 / 16
    for k, site in enumerate(sites):
        check(f, f'pe_{name}_{k}', errs[site].numpy(), 1e-3, 1e-5)
        target = errs[site] / kept
        fit = [float((ret[site] * target).sum()), float((ret[site] * ret[site]).sum())]
        np.testing.assert_allclose(fit, f[f'pf_{name}_{k}'], rtol=2e-3)
