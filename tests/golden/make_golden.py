"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the reference's own functions (imported from a checkout of pculaf/noise given by --reference)
on CPU in float32 and saves their outputs as small .npz fixtures beside this script:

  forward.npz      utils/model.py GPT.forward, per-token CE, seed-0 model, Zipf tokens, T = 1100
                   (long enough that the 1024-token windows bind), plus per-parameter init checksums.
  population.npz   train/val/eggroll.py population_loss with injected counter-based draws:
                   4 members (2 antithetic directions), one sequence, T = 1100.
  eggroll_step.npz train/val/eggroll.py Eggroll.step end to end with injected draws: 2 directions,
                   CHUNK = 1, two sequences of T = 384, step 1 -> member losses, the gradients handed
                   to AdamW (full for small tensors, checksums and sampled entries for matrices) and
                   the parameter change after AdamW.

Only the attention primitive is swapped, for the mathematically identical masked SDPA
(`(q >= k) & (q - k <= window)`), because torch.compile(flex_attention) does not lower on CPU here;
population_loss is called uncompiled. Usage:
    python tests/golden/make_golden.py --reference /path/to/noise
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch
from torch.nn import functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from noise_b200.data import zipf_tokens  # noqa: E402
from oracle import eggroll as oe  # noqa: E402
from oracle import model as om  # noqa: E402

SEED, STEP = 0, 1


def sdpa_window(q, k, v, window):
    t = q.shape[1]
    i = torch.arange(t, device=q.device)
    mask = (i[:, None] >= i[None, :]) & (i[:, None] - i[None, :] <= window)
    return F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                          attn_mask=mask).transpose(1, 2)


def checksums(t: torch.Tensor) -> np.ndarray:
    t = t.double()
    return np.array([t.sum().item(), t.abs().sum().item(), t.pow(2).sum().item()])


def sample_entries(t: torch.Tensor, n: int = 64, seed: int = 0):
    flat = t.reshape(-1)
    g = torch.Generator().manual_seed(seed)
    idx = torch.randperm(flat.numel(), generator=g)[:n]
    return idx.numpy(), flat[idx].double().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', type=Path, required=True)
    args = ap.parse_args()
    sys.path.insert(0, str(args.reference))
    import utils.model as um
    import train.val.eggroll as eg
    um.attention = sdpa_window
    eg.attention = sdpa_window
    torch.set_num_threads(8)

    # ---- forward ----
    model = eg.make_model(torch.device('cpu'), SEED)
    rows = zipf_tokens(2, 1101, seed=1)
    with torch.no_grad():
        ce = model(rows[:, :-1].contiguous(), rows[:, 1:].contiguous(), loss_reduction='none')
    names = [n for n, _ in model.named_parameters()]
    sums = np.stack([checksums(p) for _, p in model.named_parameters()])
    np.savez_compressed(HERE / 'forward.npz', tokens=rows.numpy().astype(np.int16), ce=ce.numpy(),
                        param_names=np.array(names), param_checksums=sums)
    print('forward', ce.mean().item())

    # ---- population_loss with injected draws ----
    sigma, pairs = 0.002, 2
    members = np.arange(4)
    draws, sign = oe.member_draws(members, pairs, sigma, SEED, STEP)
    params = dict(model.named_parameters())
    row = zipf_tokens(1, 1101, seed=2)[0]
    with torch.no_grad():
        losses = eg.population_loss(model, params, draws, sign, row[:-1].contiguous(), row[1:].contiguous())
    np.savez_compressed(HERE / 'population.npz', tokens=row.numpy().astype(np.int16), losses=losses.numpy(),
                        sigma=sigma, pairs=pairs, seed=SEED, step=STEP, members=members)
    print('population', losses.tolist())

    # ---- Eggroll.step end to end ----
    eg.CHUNK = 1
    eg.NOISE = 2 ** 20  # the buffer is bypassed by the injected draws; keep it small
    model = eg.make_model(torch.device('cpu'), SEED)
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    opt = torch.optim.AdamW(model.parameters(), lr=eg.LR, betas=eg.BETAS, eps=1e-8, weight_decay=0.0)
    es = eg.Eggroll(model, pairs, 0, 1)
    es.loss = eg.population_loss

    def injected_noise(offsets, directions):
        return oe.draws_for(directions.numpy(), SEED, STEP)

    es.noise = injected_noise
    seen_losses, grads = [], {}
    inner = es.loss

    def recording_loss(*a):
        out = inner(*a)
        seen_losses.append(out.clone())
        return out

    es.loss = recording_loss
    orig_step = opt.step

    def recording_step(*a, **k):
        for n, p in model.named_parameters():
            grads[n] = p.grad.detach().clone()
        return orig_step(*a, **k)

    opt.step = recording_step
    batch = zipf_tokens(2, 385, seed=3)
    mean_loss = es.step(batch[:, :-1].contiguous(), batch[:, 1:].contiguous(), opt, STEP)
    out = dict(tokens=batch.numpy().astype(np.int16), losses=torch.cat(seen_losses).numpy(), mean_loss=mean_loss,
               sigma=eg.SIGMA, pairs=pairs, seed=SEED, step=STEP, lr=eg.LR, betas=np.array(eg.BETAS),
               param_names=np.array(names))
    for i, (n, p) in enumerate(model.named_parameters()):
        g = grads[n]
        delta = (p.detach() - before[n])
        out[f'g{i}_sums'] = checksums(g)
        out[f'd{i}_sums'] = checksums(delta)
        if g.numel() <= 4096:
            out[f'g{i}_full'] = g.double().numpy()
            out[f'd{i}_full'] = delta.double().numpy()
        else:
            idx, vals = sample_entries(g, seed=i)
            out[f'g{i}_idx'], out[f'g{i}_val'] = idx, vals
            out[f'd{i}_val'] = delta.reshape(-1)[torch.from_numpy(idx)].double().numpy()
    np.savez_compressed(HERE / 'eggroll_step.npz', **out)
    print('eggroll step', mean_loss, torch.cat(seen_losses).tolist())


if __name__ == '__main__':
    main()
