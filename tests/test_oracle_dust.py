"""The DUST oracle against the reference's own outputs (tests/golden/dust.npz)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import dust as od
from oracle import model as om

GOLDEN = Path(__file__).resolve().parent / 'golden'
SEED, STEP = 0, 1


def golden():
    return np.load(GOLDEN / 'dust.npz')


def check(f, key, got, rtol, atol):
    """Compare against a full fixture array or its sampled entries + checksums."""
    got = np.asarray(got, dtype=np.float64)
    if key in f:
        np.testing.assert_allclose(got, f[key], rtol=rtol, atol=atol, err_msg=key)
        return
    flat = got.reshape(-1)
    np.testing.assert_allclose(flat[f[key + '__idx']], f[key + '__val'], rtol=rtol, atol=atol, err_msg=key)
    sums = np.array([flat.sum(), np.abs(flat).sum(), (flat ** 2).sum()])
    np.testing.assert_allclose(sums[1:], f[key + '__sums'][1:], rtol=max(rtol, 1e-6), err_msg=key)


def test_hadamard_rows_orthogonal():
    H = od.hadamard(64)
    torch.testing.assert_close(H @ H.t(), 64 * torch.eye(64))
    assert H[0].eq(1).all()


def test_orthogonal_draws_match_reference():
    f = golden()
    sid = od.site_id('transformer.h.1.mlp.c_fc')
    pats, offs = od.frame(SEED, STEP, sid, 1, 2048, 2, 128)
    idx = 16 + np.arange(16)
    signs = od.draw_signs(SEED, STEP, sid, idx, 2, 128)
    a = od.orthogonal_draws(pats, offs, signs, idx, 2048)
    check(f, 'ortho_fc', a.numpy(), 0, 0)


def test_coordinate_differences_and_reward_to_go():
    f = golden()
    g = torch.Generator().manual_seed(9)  # the inputs make_golden.py drew
    raw = torch.randn(2, 16, 4096, generator=g) * 3
    tg = torch.randint(0, 4096, (2, 16), generator=g)
    tg[0, 3] = -1
    check(f, 'cd_raw', raw.numpy(), 0, 0)
    got = od.coordinate_differences(raw.double(), tg, 0.1)
    check(f, 'cd', got.numpy(), 2e-4, 1e-6)
    got = od.reward_to_go(torch.from_numpy(f['rtg_in']).double(), 0.3)
    np.testing.assert_allclose(got.numpy(), f['rtg'], rtol=1e-5, atol=1e-6)


@pytest.fixture(scope='module')
def setup():
    f = golden()
    p = om.make_params(0)
    rows = torch.from_numpy(f['tokens'].astype(np.int64))
    x, y = rows[:, :-1], torch.from_numpy(f['targets'])
    with torch.no_grad():
        cap = od.capture(p, x)
        logits = om.soft_cap(cap['raw'])
        clean = torch.nn.functional.cross_entropy(logits.reshape(-1, om.VOCAB), y.reshape(-1), ignore_index=-1,
                                                  reduction='none').view_as(y)
    np.testing.assert_allclose(clean.numpy(), f['clean_loss'], rtol=1e-5, atol=1e-6)
    return f, p, cap, x, y, clean


CASES = {
    'writers': (['transformer.h.1.attn.c_proj', 'transformer.h.1.mlp.c_proj'], ['attn', 'mlp']),
    'hidden': (['transformer.h.6.mlp.c_fc'], ['fc']),
    'embed': (['transformer.wte'], ['transformer.wte']),
    'hub': (['o@0'], ['o']),
}


@pytest.mark.parametrize('name', list(CASES))
def test_direct_errors_match_reference(setup, name):
    f, p, cap, x, y, clean = setup
    sites, keys = CASES[name]
    draws, sigma, entry, gamma = f[f'de_{name}_meta']
    draws, entry = int(draws), (None if entry < 0 else int(entry))
    b, t = x.shape
    width = {'attn': 512, 'mlp': 512, 'o': 512, 'transformer.wte': 512, 'fc': 2048}
    a = {}
    for site, key in zip(sites, keys):
        d = width[key]
        a[site] = od.site_draws(SEED, STEP, site, np.arange(draws), b, t, d, draws)
        if key == 'fc':
            a[site] = a[site] * (cap['fc_pre'][entry] > 0).float()
    jitter = {key: sigma * a[site] for site, key in zip(sites, keys)}
    with torch.no_grad():
        perturbed = od.rerun(p, cap, x, y.clamp(min=0), draws, entry, jitter)
        perturbed = perturbed * (y >= 0)  # ignored targets score zero, like the clean loss
    errs = od.direct_errors(clean, perturbed, a, sigma, n=16, gamma=gamma)
    for k, site in enumerate(sites):
        check(f, f'de_{name}_{k}', errs[site].numpy(), 1e-3, 1e-4)
        if site.startswith('o@'):
            continue
        if site == 'transformer.wte':
            g = od.reassemble_embedding(errs[site], x)
        else:
            inp = {'attn': cap['proj_in'], 'mlp': cap['mlp_in'], 'fc': cap['fc_in']}[keys[k]][entry]
            g = od.reassemble(errs[site], inp)
        check(f, f'ra_{name}_{k}', g.numpy(), 2e-3, 1e-3)
