"""The oracle's local_errors (attention-internal estimates) against the reference's DUST.local_errors
run with the same injected draws and seeded hub targets (tests/golden/local.npz). Both are float32
CPU computations; tolerance: relative L2 1e-4 over the sampled entries and checksums rtol 1e-4."""
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / 'golden'
SEED, STEP = 0, 1
KINDS = ['q', 'k', 'v', 'gate', 've']


def targets(b, t, layers=8, seed=21):
    g = torch.Generator().manual_seed(seed)
    return {i: torch.randn(b, t, 512, generator=g) * 0.01 for i in range(layers)}


def local_case(kind, f):
    from noise_b200.data import zipf_tokens
    from oracle import dust as od
    from oracle import model as om
    b, t, draws = (int(v) for v in f[f'le_{kind}_meta'])
    rows = zipf_tokens(b, t + 1, seed=5)
    x = rows[:, :-1].contiguous()
    p = om.make_params(0)
    with torch.no_grad():
        cap = od.capture(p, x)
        a = {i: od.site_draws(SEED, STEP, od.local_site(kind, i), np.arange(draws), b, t, od.local_width(kind), draws)
             for i in od.local_layers(kind)}
        errs = od.local_errors(p, cap, x, kind, a, targets(b, t))
    return p, cap, x, errs


def unpack(f, key):
    if key in f:
        return None, torch.from_numpy(f[key]).reshape(-1).double()
    return torch.from_numpy(f[key + '__idx']), torch.from_numpy(f[key + '__val'])


@pytest.mark.parametrize('kind', KINDS)
def test_local_errors_match_reference(kind):
    from oracle import dust as od
    f = np.load(GOLDEN / 'local.npz')
    p, cap, x, errs = local_case(kind, f)
    for k, (site, e) in enumerate(errs.items()):
        idx, want = unpack(f, f'le_{kind}_{k}')
        got = e.reshape(-1) if idx is None else e.reshape(-1)[idx]
        rel = ((got - want).norm() / want.norm()).item()
        assert rel < 1e-4, (site, rel)
        if f'le_{kind}_{k}__sums' in f:
            np.testing.assert_allclose(e.abs().sum().item(), f[f'le_{kind}_{k}__sums'][1], rtol=1e-4)
    site, e = next(iter(errs.items()))
    i = od.local_layers(kind)[0]
    if kind == 've':
        g = od.reassemble_embedding(e, x)
    else:
        g = od.reassemble(e, od.local_input(cap, kind, i))
    idx, want = unpack(f, f'lr_{kind}')
    got = g.reshape(-1) if idx is None else g.reshape(-1)[idx]
    assert ((got - want).norm() / want.norm()).item() < 1e-4
