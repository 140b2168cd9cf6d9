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
  optim.npz        train/val/run.py make_optimizer (ANVIL II on block matrices, AdamW x1/x30/x300
                   elsewhere), three steps on seeded dense gradients (torch.Generator seed 11, N(0, 0.01^2),
                   drawn in named_parameters order each step): parameter deltas per tensor as checksums
                   and 512 sampled entries.
  dust.npz         train/val/run.py DUST pieces on two sequences of T = 128: orthogonal_noise with
                   injected frames and signs, coordinate_differences, reward_to_go, and
                   direct_errors (real capture + rerun + centring + contraction) for a writers group,
                   an MLP hidden site (live-unit mask), the embedding (rerun from the embedding) and
                   an attention-output hub with reward-to-go, each with its reassembled gradient.
  local.npz        train/val/run.py DUST.local_errors for each kind (q, k, v, gate, ve) with injected
                   draws and seeded hub targets (LOCAL_CASES), plus the first block's reassembled
                   gradient per kind.
  dust_bf16.npz,   the direct_errors and local_errors cases again with the reference's estimator set
  local_bf16.npz   to its GPU precision (bfloat16 draws, rewards and autocast; float32 rerun head):
                   the spread between the reference's own two precisions, the floor for any bf16 path.
  memory.npz       train/val/run.py credit memory: remember / memory_matrix / retrieve / calibrate on
                   seeded estimates keyed by the real head error, and direct_errors with retrievals
                   (MEMORY_SITES), sampled.

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
    ap.add_argument('--only-dust', action='store_true')
    ap.add_argument('--only-optim', action='store_true')
    ap.add_argument('--only-local', action='store_true')
    ap.add_argument('--only-memory', action='store_true')
    ap.add_argument('--only-bf16', action='store_true',
                    help='dust_bf16.npz and local_bf16.npz: the reference at its GPU precision')
    args = ap.parse_args()
    sys.path.insert(0, str(args.reference))
    if args.only_dust:
        dust_golden(args.reference)
        raise SystemExit
    if args.only_bf16:
        dust_golden(args.reference, bf16=True)
        local_golden(args.reference, bf16=True)
        raise SystemExit
    if args.only_optim:
        optim_golden()
        raise SystemExit
    if args.only_local:
        local_golden(args.reference)
        raise SystemExit
    if args.only_memory:
        memory_golden(args.reference)
        raise SystemExit
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


def pack(out: dict, limit: int = 8192, samples: int = 4096) -> dict:
    """Large arrays become checksums + sampled entries (key__sums, __idx, __val, __shape)."""
    packed = {}
    for k, v in out.items():
        v = np.asarray(v)
        if v.size > limit:
            t_ = torch.from_numpy(v.astype(np.float64))
            idx, vals = sample_entries(t_, n=samples, seed=len(k))
            packed[k + '__sums'] = checksums(t_)
            packed[k + '__idx'], packed[k + '__val'] = idx, vals
            packed[k + '__shape'] = np.array(v.shape)
        else:
            packed[k] = v
    return packed


def injector(run, est):
    """A stand-in for DUST.orthogonal_noise that runs the reference's own function on frames and
    signs taken from the counter-based stream (world 1)."""
    from oracle import dust as od

    def inject(site, draws, chunk, n, b_, t_, d, dtype=None):
        sid = od.site_id(site)
        cycles = -(-draws // d)
        pats, offs = od.frame(SEED, STEP, sid, cycles, d, b_, t_)
        idx = chunk * n + np.arange(n)
        signs = od.draw_signs(SEED, STEP, sid, idx, b_, t_)
        # frames and signs in the estimator's draw dtype, as DUST.signs makes them (float32 on CPU)
        est.frames[site] = (torch.as_tensor(pats).to(est.dtype), offs)
        sg = torch.as_tensor(signs).to(est.dtype)
        orig = est.signs
        est.signs = lambda *shape, shared=False: sg[..., None] if shape == (n, b_, t_, 1) else orig(*shape, shared=shared)
        try:
            a = run.DUST.orthogonal_noise(est, site, draws, chunk, n, b_, t_, d, dtype)
        finally:
            est.signs = orig
        return a

    return inject


# (kind, sequences, length, draws): windows bind at T = 1152; T = 256, 512 and 1152 cover the GPU
# kernel's 2-, 4- and 1-tile CTAs
LOCAL_CASES = [('q', 2, 256, 32), ('k', 1, 1152, 16), ('v', 2, 256, 16), ('gate', 2, 256, 16), ('ve', 1, 512, 16)]
LOCAL_TARGET_SEED = 21


def local_targets(b: int, t: int, layers: int = 8) -> dict:
    """Seeded stand-ins for the hub targets, [b, t, 512] per block, 0.01 N(0, 1)."""
    g = torch.Generator().manual_seed(LOCAL_TARGET_SEED)
    return {i: torch.randn(b, t, 512, generator=g) * 0.01 for i in range(layers)}


def local_golden(reference, bf16: bool = False):
    """DUST.local_errors (train/val/run.py:391-463) per kind with injected draws and seeded targets,
    and each kind's reassembled gradient of its first block. bf16: the same at the reference's GPU
    precision (bf16_precision), into local_bf16.npz."""
    torch._dynamo.config.disable = True
    import train.val.run as run
    run.attention = sdpa_window
    torch.set_num_threads(8)
    out = {}
    for kind, b, t, draws in LOCAL_CASES:
        model = run.make_model(torch.device('cpu'), SEED)
        est = run.DUST(model, run.recipe(0.01), SEED, 0, 1)
        if bf16:
            bf16_precision(est)
        rows = zipf_tokens(b, t + 1, seed=5)
        x, y = rows[:, :-1].contiguous(), rows[:, 1:].contiguous()
        est.capture(x, y)
        est.orthogonal_noise = injector(run, est)
        with torch.no_grad():
            errs = est.local_errors(kind, draws, local_targets(b, t))
        for k, (site, e) in enumerate(errs.items()):
            out[f'le_{kind}_{k}'] = e.float().numpy()
        site, e = next(iter(errs.items()))
        if not bf16:
            out[f'lr_{kind}'] = est.reassemble(site, e).numpy()
        out[f'le_{kind}_meta'] = np.array([b, t, draws])
        print('local', kind, {s: float(v.abs().mean()) for s, v in errs.items()})
    np.savez_compressed(HERE / ('local_bf16.npz' if bf16 else 'local.npz'), **pack(out, samples=1024))


MEMORY_SITES = ['transformer.h.1.attn.c_proj', 'transformer.h.1.mlp.c_proj', 'transformer.h.6.mlp.c_fc', 'o@0']
MEMORY_SEED = 31


def memory_estimates(b: int, t: int, round_: int) -> dict:
    """Seeded stand-ins for a step's site estimates, [b, t, d], 0.01 N(0, 1)."""
    g = torch.Generator().manual_seed(MEMORY_SEED + round_)
    width = {'transformer.h.6.mlp.c_fc': 2048}
    return {s: torch.randn(b, t, width.get(s, 512), generator=g) * 0.01 for s in MEMORY_SITES}


def memory_golden(reference):
    """The credit memory (train/val/run.py:281-330) and direct_errors with its prior (:332-378): two
    remember() writes of seeded estimates keyed by the real head error, the memory matrices and
    retrievals, two calibrations, and direct_errors with retrievals for a writers group, an MLP hidden
    site and a hub with reward-to-go."""
    torch._dynamo.config.disable = True
    import train.val.run as run
    run.attention = sdpa_window
    torch.set_num_threads(8)
    model = run.make_model(torch.device('cpu'), SEED)
    est = run.DUST(model, run.recipe(0.01), SEED, 0, 1)
    rows = zipf_tokens(2, 129, seed=4)
    x, y = rows[:, :-1].contiguous(), rows[:, 1:].contiguous()
    y[1, 5] = -1
    b, t = x.shape
    with torch.no_grad():
        est.capture(x, y)
        est.head_credit = est.head_error()[..., :4096]
        valid = (y != -1).sum()
        est.prior_sites = list(MEMORY_SITES)
        out = {}
        for round_ in range(2):
            est.estimates = memory_estimates(b, t, round_)
            est.remember(valid)
        out['P'] = est.shared['P'].numpy()
        for k, site in enumerate(MEMORY_SITES):
            out[f'S_{k}'] = est.memory[site]['S'].numpy()
            out[f'M_{k}'] = est.memory_matrix(site).numpy()
        retrieved = est.retrieve(MEMORY_SITES)
        for k, site in enumerate(MEMORY_SITES):
            out[f'r_{k}'] = retrieved[site].numpy()
        # calibration from two rounds of seeded fits
        g = torch.Generator().manual_seed(MEMORY_SEED + 7)
        for round_ in range(2):
            est.fits = {s: torch.stack([torch.randn((), generator=g), torch.rand((), generator=g) + 0.5])
                        for s in MEMORY_SITES}
            out[f'fits_{round_}'] = torch.stack([est.fits[s] for s in MEMORY_SITES]).numpy()
            est.calibrate()
        out['alpha'] = np.array([est.alpha[s] for s in MEMORY_SITES])
        # direct errors with the prior
        est.orthogonal_noise = injector(run, est)
        cases = [
            ('writers', ['transformer.h.1.attn.c_proj', 'transformer.h.1.mlp.c_proj'], 32, 0.4, 1, 0.0),
            ('hidden', ['transformer.h.6.mlp.c_fc'], 16, 0.4, 6, 0.0),
            ('hub', ['o@0'], 16, 0.4, 0, 0.3),
        ]
        for name, sites, draws, sigma, entry, gamma in cases:
            est.frames.clear()
            est.fits.clear()
            errs = est.direct_errors(sites, draws, sigma, entry, gamma, est.retrieve(sites))
            for k, site in enumerate(sites):
                out[f'pe_{name}_{k}'] = errs[site].numpy()
                out[f'pf_{name}_{k}'] = est.fits[site].numpy()
            out[f'pe_{name}_meta'] = np.array([draws, sigma, -1 if entry is None else entry, gamma])
    np.savez_compressed(HERE / 'memory.npz', **pack(out, samples=1024))
    print('memory', out['alpha'], {k: float(np.abs(v).mean()) for k, v in out.items() if k.startswith('pe_') and 'meta' not in k})


def bf16_precision(est):
    """Run a DUST estimator on CPU at the reference's GPU precision: draws and rewards in bfloat16
    (DUST.dtype) and the capture and reruns under bfloat16 autocast (DUST.autocast), the rerun head
    still float32 as the reference's own code keeps it (train/val/run.py:272-278)."""
    est.dtype = torch.bfloat16
    est.autocast = lambda: torch.autocast('cpu', dtype=torch.bfloat16)


DUST_CASES = [
    ('writers', ['transformer.h.1.attn.c_proj', 'transformer.h.1.mlp.c_proj'], 32, 0.4, 1, 0.0),
    ('hidden', ['transformer.h.6.mlp.c_fc'], 16, 0.4, 6, 0.0),
    ('embed', ['transformer.wte'], 16, 0.8, None, 0.0),
    ('hub', ['o@0'], 16, 0.4, 0, 0.3),
    ('deep', ['transformer.h.7.attn.c_proj', 'transformer.h.7.mlp.c_proj'], 32, 0.4, 7, 0.0),
]


def dust_golden(reference, bf16: bool = False):
    """DUST fixtures; only orthogonal_noise's random frames and signs are injected. bf16: the
    direct_errors cases again at the reference's GPU precision (bf16_precision), into dust_bf16.npz:
    the spread between the reference's own two precisions."""
    from oracle import dust as od
    torch._dynamo.config.disable = True
    import train.val.run as run
    run.attention = sdpa_window
    torch.manual_seed(0)
    model = run.make_model(torch.device('cpu'), SEED)
    est = run.DUST(model, run.recipe(0.01), SEED, 0, 1)
    if bf16:
        bf16_precision(est)
    rows = zipf_tokens(2, 129, seed=4)
    x, y = rows[:, :-1].contiguous(), rows[:, 1:].contiguous()
    y[1, 5] = -1  # an ignored target
    est.capture(x, y)
    b, t = x.shape
    out = dict(tokens=rows.numpy().astype(np.int16), targets=y.numpy().astype(np.int64),
               clean_loss=est.clean_loss.float().numpy())

    inject = injector(run, est)
    if bf16:
        est.orthogonal_noise = lambda site, draws, chunk, n, b_, t_, d, dtype=None: inject(site, draws, chunk, n, b_, t_, d, dtype)
        for name, sites, draws, sigma, entry, gamma in DUST_CASES:
            est.frames.clear()
            errs = est.direct_errors(sites, draws, sigma, entry, gamma, {})
            for k, site in enumerate(sites):
                out[f'de_{name}_{k}'] = errs[site].float().numpy()
            out[f'de_{name}_meta'] = np.array([draws, sigma, -1 if entry is None else entry, gamma])
        np.savez_compressed(HERE / 'dust_bf16.npz', **pack(out))
        print('dust bf16', {k: v.shape for k, v in out.items() if k.startswith('de_')})
        return

    # orthogonal_noise itself
    a = inject('transformer.h.1.mlp.c_fc', 96, 1, 16, b, t, 2048)
    out['ortho_fc'] = a.numpy().astype(np.int8)
    est.frames.clear()
    # coordinate differences and reward-to-go
    g = torch.Generator().manual_seed(9)
    raw = torch.randn(2, 16, 4096, generator=g) * 3
    tg = torch.randint(0, 4096, (2, 16), generator=g)
    tg[0, 3] = -1
    out['cd_raw'], out['cd_targets'] = raw.numpy(), tg.numpy()
    out['cd'] = run.coordinate_differences(raw, tg, 0.1).numpy()
    rw = torch.randn(3, 2, 40, generator=g)
    out['rtg_in'], out['rtg'] = rw.numpy(), run.reward_to_go(rw, 0.3).numpy()
    # direct errors through the reference's own reruns
    est.orthogonal_noise = lambda site, draws, chunk, n, b_, t_, d, dtype=None: inject(site, draws, chunk, n, b_, t_, d, dtype)
    for name, sites, draws, sigma, entry, gamma in DUST_CASES:
        est.frames.clear()
        errs = est.direct_errors(sites, draws, sigma, entry, gamma, {})
        for k, site in enumerate(sites):
            out[f'de_{name}_{k}'] = errs[site].numpy()
            if not site.startswith('o@'):
                out[f'ra_{name}_{k}'] = est.reassemble(site, errs[site]).numpy()
        out[f'de_{name}_meta'] = np.array([draws, sigma, -1 if entry is None else entry, gamma])
    np.savez_compressed(HERE / 'dust.npz', **pack(out))
    print('dust', {k: v.shape for k, v in out.items() if k.startswith('de_')})


def optim_golden():
    torch._dynamo.config.disable = True
    import train.val.run as run
    model = run.make_model(torch.device('cpu'), SEED)
    opt = run.make_optimizer(model, run.recipe(0.01), 100)
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    g = torch.Generator().manual_seed(11)
    for _ in range(3):
        for _, prm in model.named_parameters():
            prm.grad = torch.randn(prm.shape, generator=g) * 0.01
        opt.step()
    out = {}
    for i, (n, prm) in enumerate(model.named_parameters()):
        d = (prm.detach() - before[n]).double()
        out[f'd{i}_sums'] = checksums(d)
        idx, vals = sample_entries(d, n=512, seed=100 + i)
        out[f'd{i}_idx'], out[f'd{i}_val'] = idx.astype(np.int32), vals.astype(np.float32)
    np.savez_compressed(HERE / 'optim.npz', **out)
    print('optim', out['d3_sums'], out['d2_sums'])


if __name__ == '__main__':
    main()
    dust_golden(None)
    optim_golden()
