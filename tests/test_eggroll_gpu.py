"""Fitness shaping, Sigma f eps + AdamW and a whole Eggroll.step on the GPU, against the oracle and the
reference's golden vectors. Tolerances: ranks bit-exact; update cosine >= 0.999 (the parity bar for the update) and
elementwise rtol 1e-4 on the reconstructed gradient; AdamW deltas rtol 2e-3."""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / 'golden'


def _losses(n, seed=0):
    rng = np.random.default_rng(seed)
    x = (8.3 + 1e-3 * rng.standard_normal(n)).astype(np.float32)
    x[5] = x[17]   # exact tie
    x[40] = x[41]  # a tie inside one antithetic pair
    return x


@pytest.mark.parametrize('n,pairs', [(1024, 512), (4096, 2048), (2000, 700)])
def test_fitness_ranks_and_weights(n, pairs):
    from noise_b200.eggroll import fitness_weights
    from oracle import eggroll as oe
    x = _losses(n, n)
    if n == 2000:
        x[100] = np.nan
    t = torch.from_numpy(x).cuda()
    ranks = torch.empty(n, dtype=torch.int32, device='cuda')
    w_rank = fitness_weights(t, pairs, 'centered_rank', ranks).cpu().numpy()
    np.testing.assert_array_equal(ranks.cpu().numpy(), oe.centered_ranks(x))
    np.testing.assert_array_equal(w_rank, oe.fitness_centered_rank(x, pairs).astype(np.float32))
    if n != 2000:
        w_z = fitness_weights(t, pairs, 'zscore').cpu().numpy()
        np.testing.assert_allclose(w_z, oe.fitness_zscore(x, pairs), rtol=1e-5, atol=1e-6)


def _grad(weights, fw, scale, seed, step):
    from noise_b200 import _lib
    g = torch.empty_like(weights.flat)
    _lib.call('noise_update_sum_fe_adamw', weights.flat.data_ptr(), None, None, None, fw.data_ptr(), fw.numel(),
              float(scale), seed, step, None, 0.0, 0.0, 0.0, 0.0, 0.0, 0, g.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return g


def test_update_matches_reference_gradients():
    """Reference losses -> noise_fitness -> reconstructed gradient vs the gradient Eggroll.step handed to AdamW."""
    from noise_b200.eggroll import fitness_weights
    from noise_b200.model import PARAM_SPECS, Weights
    f = np.load(GOLDEN / 'eggroll_step.npz')
    w = Weights('cuda', seed=0)
    losses = torch.from_numpy(f['losses']).cuda()
    fw = fitness_weights(losses, int(f['pairs']), 'zscore')
    g = _grad(w, fw, 1.0 / (len(f['losses']) // 2), int(f['seed']), int(f['step']))
    off = 0
    dots = np.zeros(3)
    for i, (name, shape) in enumerate(PARAM_SPECS):
        k = int(np.prod(shape))
        gi = g[off:off + k].double().cpu()
        off += k
        np.testing.assert_allclose(gi.abs().sum().item(), f[f'g{i}_sums'][1], rtol=1e-4, err_msg=name)
        if f'g{i}_full' in f:
            ref = f[f'g{i}_full'].reshape(-1)
            got = gi.numpy()
        else:
            ref = f[f'g{i}_val']
            got = gi[torch.from_numpy(f[f'g{i}_idx'])].numpy()
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-6 * np.abs(ref).max(), err_msg=name)
        dots += [np.dot(got, ref), np.dot(got, got), np.dot(ref, ref)]
    cos = dots[0] / np.sqrt(dots[1] * dots[2])
    assert cos >= 0.999, cos


def test_update_matches_oracle_at_bench_scale():
    """512 directions, as in the 1xB200 configuration: kernel vs the float64 oracle on a few tensors."""
    from noise_b200.model import Weights, PARAM_SPECS
    from oracle import eggroll as oe
    w = Weights('cuda', seed=0)
    rng = np.random.default_rng(3)
    fw_np = rng.standard_normal(512).astype(np.float32)
    fw = torch.from_numpy(fw_np).cuda()
    g = _grad(w, fw, 1.0 / 512, 0, 7)
    names = ['resid_lambdas', 'transformer.h.1.attn.ve_gate.weight', 'transformer.h.2.attn.c_k.weight',
             'transformer.h.5.mlp.c_proj.weight']
    ref = oe.sum_fe(fw_np.astype(np.float64), 512, 0, 7, names=names)
    off = 0
    for name, shape in PARAM_SPECS:
        k = int(np.prod(shape))
        if name in ref:
            got = g[off:off + k].view(shape).double().cpu()
            want = ref[name]
            cos = torch.nn.functional.cosine_similarity(got.reshape(-1), want.reshape(-1), dim=0).item()
            assert cos > 0.999999, (name, cos)
            torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-6 * want.abs().max().item())
        off += k


def test_adamw_first_step_matches_reference():
    from noise_b200.eggroll import AdamW, fitness_weights
    from noise_b200.model import PARAM_SPECS, Weights
    f = np.load(GOLDEN / 'eggroll_step.npz')
    w = Weights('cuda', seed=0)
    before = w.flat.clone()
    opt = AdamW(w, lr=float(f['lr']), betas=tuple(f['betas']))
    fw = fitness_weights(torch.from_numpy(f['losses']).cuda(), int(f['pairs']), 'zscore')
    opt.set_sum_fe(fw, 1.0 / (len(f['losses']) // 2), int(f['seed']), int(f['step']))
    opt.step()
    torch.cuda.synchronize()
    delta = (w.flat - before).double().cpu()
    off = 0
    for i, (name, shape) in enumerate(PARAM_SPECS):
        k = int(np.prod(shape))
        d = delta[off:off + k]
        off += k
        if f'd{i}_full' in f:
            np.testing.assert_allclose(d.numpy(), f[f'd{i}_full'].reshape(-1), rtol=2e-3, atol=2e-7, err_msg=name)
        else:
            got = d[torch.from_numpy(f[f'g{i}_idx'])].numpy()
            np.testing.assert_allclose(got, f[f'd{i}_val'], rtol=2e-3, atol=2e-7, err_msg=name)
    # the packed bf16 copy follows the master weights
    from noise_b200 import _lib
    ref_packed = torch.empty_like(w.packed)
    _lib.call('noise_pack_weights', w.flat.data_ptr(), ref_packed.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(ref_packed, w.packed)


def test_eggroll_step_losses_match_reference():
    """Eggroll.step end to end, reference layout (CHUNK = 1, one sequence per member block)."""
    from noise_b200.eggroll import AdamW, Eggroll
    from noise_b200.model import Weights
    f = np.load(GOLDEN / 'eggroll_step.npz')
    w = Weights('cuda', seed=0)
    opt = AdamW(w, lr=float(f['lr']), betas=tuple(f['betas']))
    es = Eggroll(w, int(f['pairs']), sigma=float(f['sigma']), seed=int(f['seed']), chunk=1)
    batch = torch.from_numpy(f['tokens'].astype(np.int64)).cuda()
    mean = es.step(batch[:, :-1], batch[:, 1:], opt, int(f['step']))
    np.testing.assert_allclose(es.last_losses.cpu().numpy(), f['losses'], rtol=2e-5)
    np.testing.assert_allclose(mean, float(f['mean_loss']), rtol=2e-5)
