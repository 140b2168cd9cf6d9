"""DUST's direct-draw path on the GPU against the CPU oracle and the reference's fixtures.

Tolerances: per-token rerun losses rel 2e-3 (bf16 GEMM operands in the blocks, fp32 head on tf32
MMAs, vs the fp32 oracle); the error contraction and coordinate differences on identical inputs rtol
1e-4; the full estimate (rerun + contraction) against the reference's float32 direct_errors
(tests/golden/dust.npz): cosine >= 0.999 and relative L2 error <= 2e-2, unless the reference's own
GPU precision (the same estimator with bfloat16 draws, rewards and autocast, float32 rerun head:
tests/golden/dust_bf16.npz) is itself further from its float32 result, in which case this path must
be at least as close as the reference's: cosine >= that floor's and relative error <= its. Only the
MLP-hidden site (block 6, live units) has such a floor (cosine 0.9968, relative error 0.080); this
path measures 0.9985 and 0.056 there, and 0.9999 / <= 0.016 in every other case."""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / 'golden'
SEED, STEP = 0, 1


@pytest.fixture(scope='module')
def env():
    from noise_b200.dust import Capture
    from noise_b200.model import Weights
    from oracle import dust as od
    from oracle import model as om
    f = np.load(GOLDEN / 'dust.npz')
    rows = torch.from_numpy(f['tokens'].astype(np.int64))
    x, y = rows[:, :-1], torch.from_numpy(f['targets'])
    w = Weights('cuda', seed=0)
    cap = Capture(w, x, y)
    p = om.make_params(0)
    with torch.no_grad():
        ocap = od.capture(p, x)
    return dict(f=f, x=x, y=y, w=w, cap=cap, p=p, ocap=ocap)


def test_capture_matches_oracle(env):
    cap, ocap, f = env['cap'], env['ocap'], env['f']
    np.testing.assert_allclose(cap.clean_loss.cpu().numpy().reshape(2, -1), f['clean_loss'], rtol=2e-4, atol=1e-5)
    # bf16 GEMM operands across several blocks: compare whole tensors by relative L2 error
    for i in range(8):
        rel, cos = _rel(cap.blocks[i].cpu(), ocap['blocks'][i])
        assert rel < 1e-2 and cos > 0.9999, (i, rel, cos)
    rel, cos = _rel(cap.logits.cpu(), ocap['raw'])
    assert rel < 2e-2 and cos > 0.9998, (rel, cos)


CASES = {
    'writers': (['transformer.h.1.attn.c_proj', 'transformer.h.1.mlp.c_proj'], ['attn', 'mlp']),
    'hidden': (['transformer.h.6.mlp.c_fc'], ['fc']),
    'embed': (['transformer.wte'], ['transformer.wte']),
    'hub': (['o@0'], ['o']),
    'deep': (['transformer.h.7.attn.c_proj', 'transformer.h.7.mlp.c_proj'], ['attn', 'mlp']),
}


def _oracle_draws(env, name, gpu_mask=False):
    """The oracle's draws for a case; MLP-hidden draws masked by the oracle's live units, or by the
    GPU capture's (gpu_mask) when the two paths must see identical inputs."""
    from oracle import dust as od
    f, ocap = env['f'], env['ocap']
    sites, keys = CASES[name]
    draws, sigma, entry, gamma = f[f'de_{name}_meta']
    draws, entry = int(draws), (None if entry < 0 else int(entry))
    width = {'attn': 512, 'mlp': 512, 'o': 512, 'transformer.wte': 512, 'fc': 2048}
    a = {}
    for s, k in zip(sites, keys):
        a[s] = od.site_draws(SEED, STEP, s, np.arange(draws), 2, 128, width[k], draws)
        if k == 'fc':
            live = env['cap'].hidden[entry].cpu().float().view(2, 128, -1) > 0 if gpu_mask else ocap['fc_pre'][entry] > 0
            a[s] = a[s] * live.float()
    return sites, keys, draws, float(sigma), entry, float(gamma), a


@pytest.mark.parametrize('name', list(CASES))
def test_rerun_matches_oracle(env, name):
    from noise_b200.dust import rerun, site
    from oracle import dust as od
    sites, keys, draws, sigma, entry, gamma, a = _oracle_draws(env, name)
    got = rerun(env['w'], env['cap'], [site(s) for s in sites], draws, 0, sigma, entry, SEED, STEP).cpu()
    jitter = {k: sigma * a[s] for s, k in zip(sites, keys)}
    with torch.no_grad():
        want = od.rerun(env['p'], env['ocap'], env['x'], env['y'].clamp(min=0), draws, entry, jitter)
        want = want * (env['y'] >= 0)
    torch.testing.assert_close(got, want, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize('name', ['writers', 'hidden', 'hub'])
def test_error_contraction_matches_oracle(env, name):
    """Identical per-token losses in, so only the contraction is compared."""
    from noise_b200.dust import accumulate_errors, site
    from oracle import dust as od
    sites, keys, draws, sigma, entry, gamma, a = _oracle_draws(env, name, gpu_mask=True)
    g = torch.Generator().manual_seed(5)
    clean = env['cap'].clean_loss.cpu().view(2, 128)
    perturbed = clean.unsqueeze(0) + 1e-2 * torch.randn(draws, 2, 128, generator=g)
    want = od.direct_errors(clean, perturbed, a, sigma, n=16, gamma=gamma)
    for s in sites:
        err = accumulate_errors(env['cap'], perturbed.cuda().contiguous(), site(s), 0, 16, sigma, gamma, SEED, STEP)
        got = (err / draws).view(2, 128, -1).cpu().double()
        torch.testing.assert_close(got, want[s], rtol=1e-4, atol=1e-6)


def test_coordinate_differences_match_oracle(env):
    from noise_b200.dust import head_error
    from oracle import dust as od
    got = head_error(env['cap']).cpu().double()
    want = od.coordinate_differences(env['cap'].logits.cpu().double().view(2, 128, -1), env['y'], 0.1)
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-6)


def _rel(got, want):
    got, want = got.reshape(-1).double(), want.reshape(-1).double()
    return ((got - want).norm() / want.norm()).item(), torch.nn.functional.cosine_similarity(got, want, dim=0).item()


@pytest.mark.parametrize('name', list(CASES))
def test_direct_errors_match_reference(env, name):
    """The whole estimate (GPU reruns + contraction) against the reference's direct_errors, on the
    sampled entries the fixture keeps."""
    from noise_b200.dust import direct_errors
    f = env['f']
    sites, keys, draws, sigma, entry, gamma, a = _oracle_draws(env, name)
    errs = direct_errors(env['w'], env['cap'], sites, draws, sigma, entry, gamma, SEED, STEP)
    fb = np.load(GOLDEN / 'dust_bf16.npz')
    for k, s in enumerate(sites):
        key = f'de_{name}_{k}'
        got = errs[s].cpu().double().reshape(-1)[torch.from_numpy(f[key + '__idx'])]
        want = torch.from_numpy(f[key + '__val'])
        rel, cos = _rel(got, want)
        frel, fcos = _rel(torch.from_numpy(fb[key + '__val']), want)
        grel, gcos = _rel(got, torch.from_numpy(fb[key + '__val']))
        print(f'{name} {s}: vs fp32 ref rel {rel:.4f} cos {cos:.5f}; ref bf16 vs fp32 rel {frel:.4f} cos {fcos:.5f}; '
              f'vs bf16 ref rel {grel:.4f} cos {gcos:.5f}')
        assert cos >= min(0.999, fcos) and rel <= max(2e-2, frel), (rel, cos, frel, fcos)
