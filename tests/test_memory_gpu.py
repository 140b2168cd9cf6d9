"""The credit memory and prior-corrected direct errors on the GPU.

- the prior correction inside the contraction kernel (one Walsh-Hadamard transform per token and
  draw cycle) against the oracle's explicit sigma a . mu on identical perturbed losses: rtol 1e-4;
- the memory (P, S, M, retrievals, alpha) and the whole prior-corrected estimates against the
  reference (tests/golden/memory.npz). The key c comes from the GPU's bf16-GEMM logits, so the memory
  is compared by relative L2 (<= 3e-2 for P and S, 5e-2 for M, retrievals and estimates) and cosine.
  The memory's products run on TF32, the precision DUST.step gives them (the reference's run sets
  set_float32_matmul_precision('high'), train/val/run.py:676; the fixture was made on the CPU in fp32).
  The MLP hidden site is held to the oracle run with the GPU's own live-unit mask (same bounds); against
  the reference only its cosine is checked, since ~0.2% of units are live in one forward and not the
  other and the prior's predicted drop sums over all of a token's units.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / 'golden'
SEED, STEP = 0, 1
SITES = ['transformer.h.1.attn.c_proj', 'transformer.h.1.mlp.c_proj', 'transformer.h.6.mlp.c_fc', 'o@0']
WIDTH = {'transformer.h.6.mlp.c_fc': 2048}


def _estimates(b, t, round_, seed=31):
    g = torch.Generator().manual_seed(seed + round_)
    return {s: torch.randn(b, t, WIDTH.get(s, 512), generator=g) * 0.01 for s in SITES}


def _rel(got, want):
    got, want = torch.as_tensor(got).reshape(-1).double(), torch.as_tensor(want).reshape(-1).double()
    return ((got - want).norm() / want.norm()).item(), torch.nn.functional.cosine_similarity(got, want, dim=0).item()


def _pick(f, key, flat):
    if key in f:
        return flat, torch.from_numpy(f[key]).reshape(-1).double()
    return flat[torch.from_numpy(f[key + '__idx'])], torch.from_numpy(f[key + '__val'])


@pytest.fixture(scope='module', autouse=True)
def _reference_precision():
    from noise_b200.dust import reference_matmul_precision
    with reference_matmul_precision():
        yield


@pytest.fixture(scope='module')
def env():
    from noise_b200.data import zipf_tokens
    from noise_b200.dust import Capture, CreditMemory, head_error
    from noise_b200.model import Weights
    f = np.load(GOLDEN / 'memory.npz')
    rows = zipf_tokens(2, 129, seed=4)
    x, y = rows[:, :-1].contiguous(), rows[:, 1:].contiguous()
    y[1, 5] = -1
    w = Weights('cuda', seed=0)
    cap = Capture(w, x, y)
    credit = head_error(cap).view(-1, 4096)
    valid = float((y >= 0).sum())
    mem = CreditMemory()
    for r in range(2):
        mem.estimates = {s: e.cuda() for s, e in _estimates(2, 128, r).items()}
        mem.remember(credit, valid)
    return dict(f=f, x=x, y=y, w=w, cap=cap, credit=credit, mem=mem)


def test_prior_correction_matches_oracle(env):
    """Identical perturbed losses and priors in: only the kernel's prediction and centring differ."""
    from noise_b200.dust import accumulate_errors, prior_struct, site
    from oracle import dust as od
    cap = env['cap']
    names = ['transformer.h.1.attn.c_proj', 'transformer.h.1.mlp.c_proj']
    draws, sigma, n = 32, 0.4, 16
    g = torch.Generator().manual_seed(5)
    clean = cap.clean_loss.cpu().view(2, 128)
    perturbed = clean.unsqueeze(0) + 1e-2 * torch.randn(draws, 2, 128, generator=g)
    mus = {s: torch.randn(2, 128, 512, generator=g) * 0.02 for s in names}
    a = {s: od.site_draws(SEED, STEP, s, np.arange(draws), 2, 128, 512, draws) for s in names}
    want = od.direct_errors(clean, perturbed, a, sigma, n=n, gamma=0.0, priors=mus)
    sites = [site(s) for s in names]
    priors = {s: m.reshape(256, 512).cuda().contiguous() for s, m in mus.items()}
    ps = prior_struct(sites, priors)
    for s in sites:
        err = accumulate_errors(cap, perturbed.cuda().contiguous(), s, 0, n, sigma, 0.0, SEED, STEP, prior=ps)
        got = (err / draws + (1 - 1 / n) * priors[s.name]).view(2, 128, -1).cpu().double()
        torch.testing.assert_close(got, want[s.name], rtol=1e-4, atol=1e-6)


def test_memory_matches_reference(env):
    f, mem, credit = env['f'], env['mem'], env['credit']
    rel, cos = _rel(*_pick(f, 'P', mem.P.cpu().double().reshape(-1)))
    print('P', rel, cos)
    assert rel < 3e-2 and cos > 0.999
    for k, s in enumerate(SITES):
        rel, cos = _rel(*_pick(f, f'S_{k}', mem.S[s].cpu().double().reshape(-1)))
        assert rel < 3e-2 and cos > 0.999, (s, 'S', rel, cos)
        rel, cos = _rel(*_pick(f, f'M_{k}', mem.matrix(s).cpu().double().reshape(-1)))
        assert rel < 5e-2 and cos > 0.998, (s, 'M', rel, cos)
        r = mem.retrieve(credit, [s])[s]
        rel, cos = _rel(*_pick(f, f'r_{k}', r.cpu().double().reshape(-1)))
        print(s, 'retrieval', rel, cos)
        assert rel < 5e-2 and cos > 0.998, (s, 'r', rel, cos)


def test_calibration_matches_reference(env):
    from noise_b200.dust import CreditMemory
    f = env['f']
    mem = CreditMemory()
    for r in range(2):
        fits = torch.from_numpy(f[f'fits_{r}']).float().cuda()
        mem.fits = {s: fits[k] for k, s in enumerate(SITES)}
        mem.calibrate()
    np.testing.assert_allclose([mem.alpha[s] for s in SITES], f['alpha'], rtol=1e-5)


CASES = {
    'writers': ['transformer.h.1.attn.c_proj', 'transformer.h.1.mlp.c_proj'],
    'hidden': ['transformer.h.6.mlp.c_fc'],
    'hub': ['o@0'],
}


@pytest.mark.parametrize('name', list(CASES))
def test_prior_direct_errors_match_reference(env, name):
    from noise_b200.dust import chunk_size, direct_errors
    f, mem, cap, credit = env['f'], env['mem'], env['cap'], env['credit']
    mem.alpha = dict(zip(SITES, (float(a) for a in f['alpha'])))
    names = CASES[name]
    draws, sigma, entry, gamma = f[f'pe_{name}_meta']
    draws, entry = int(draws), int(entry)
    retrieved = mem.retrieve(credit, names)
    live = {s: (cap.hidden[entry] > 0).float() for s in names if s.endswith('mlp.c_fc')}
    errs = direct_errors(env['w'], cap, names, draws, float(sigma), entry, float(gamma), SEED, STEP,
                         priors=mem.priors(retrieved, live))
    kept = 1 - 1 / chunk_size(draws, 16)
    loose = bool(live)  # see below
    for k, s in enumerate(names):
        rel, cos = _rel(*_pick(f, f'pe_{name}_{k}', errs[s].cpu().double().reshape(-1)))
        print(name, s, 'rel', rel, 'cos', cos)
        if loose:
            # The prior enters every draw's predicted drop as a sum over all 2048 units, so the units
            # that the bf16 forward and the fp32 reference disagree are live (~0.2%, pre-activation at
            # zero within rounding) shift whole tokens. Against the reference: cosine only; the tight
            # check is against the oracle given the GPU's own live mask, below.
            assert cos >= 0.99, (s, rel, cos)
        else:
            assert rel <= 5e-2 and cos >= 0.995, (s, rel, cos)
            mem.fit(s, retrieved[s], errs[s], kept)
            rel, _ = _rel(mem.fits[s].cpu(), torch.from_numpy(f[f'pf_{name}_{k}']))
            assert rel <= 5e-2, (s, 'fit', rel)
    if loose:
        from oracle import dust as od
        from oracle import model as om
        s = names[0]
        p = om.make_params(0)
        x, y = env['x'], env['y']
        with torch.no_grad():
            ocap = od.capture(p, x)
            mask = (cap.hidden[entry] > 0).float().cpu().view(2, 128, -1)
            a = {s: od.site_draws(SEED, STEP, s, np.arange(draws), 2, 128, 2048, draws) * mask}
            mu = {s: mem.priors(retrieved, live)[s].cpu().double().view(2, 128, -1)}
            perturbed = od.rerun(p, ocap, x, y.clamp(min=0), draws, entry, {'fc': float(sigma) * a[s]}) * (y >= 0)
            logits = om.soft_cap(ocap['raw'])
            clean = torch.nn.functional.cross_entropy(logits.reshape(-1, om.VOCAB), y.reshape(-1), ignore_index=-1,
                                                      reduction='none').view_as(y)
        want = od.direct_errors(clean, perturbed, a, float(sigma), n=16, gamma=float(gamma), priors=mu)[s]
        rel, cos = _rel(errs[s].cpu(), want)
        print(name, s, 'vs oracle with the same live mask: rel', rel, 'cos', cos)
        assert rel <= 5e-2 and cos >= 0.995, (s, rel, cos)
