"""DUST's direct-draw estimator pieces, restated on CPU (test infrastructure; see oracle/__init__.py).

Reference: `train/val/run.py` — hadamard :143-152, orthogonal_noise :223-238, reward_to_go :81-86,
head_loss :89-94, block_forward :102-117, coordinate_differences :120-137, rerun :256-279,
direct_errors :332-378 (with or without the credit-memory prior), local_errors :391-463, reassemble
:465-471, and the credit memory :281-330 (memory_matrix, retrieve, remember, calibrate).

Frames and signs of the orthogonal draws come from the counter-based stream (noise_b200's
`csrc/dust.cuh` generates the same bits); parity with the reference is shown by injecting them into
its `orthogonal_noise` (tests/golden/make_golden.py).
"""
from __future__ import annotations

import math

import numpy as np
import torch
from torch.nn import functional as F

from . import model as om
from .philox import DOMAIN_DIRECT, philox4x32_10

# site ids of the direct-draw stream (one frame per site and step)
SITE_WTE = 2


def site_id(site: str) -> int:
    """Stable id of a jitter site: the parameter tensor id whose output is jittered; hubs o@i -> 64 + i."""
    if site.startswith('o@'):
        return 64 + int(site[2:])
    if site == 'transformer.wte':
        return SITE_WTE
    return om.TENSOR_ID[site + '.weight']


def hadamard(d: int) -> torch.Tensor:
    """Sylvester Hadamard matrix of order d (run.py:143-152): H[r, c] = (-1)^popcount(r & c)."""
    r = np.arange(d)[:, None] & np.arange(d)[None, :]
    bits = np.zeros_like(r)
    while r.any():
        bits ^= r & 1
        r >>= 1
    return torch.from_numpy(1 - 2 * bits).float()


def _bits(seed, step, blocks, kind, direction, site):
    """128 sign bits per Philox block of the direct stream: counter (block, site << 2 | kind, direction)."""
    x = philox4x32_10(np.asarray(blocks, dtype=np.uint64), (site << 2) | kind, direction, DOMAIN_DIRECT, seed, step)
    words = np.stack(x, axis=-1).astype(np.uint64)  # [..., 4]
    return words


def frame(seed: int, step: int, site: int, cycles: int, d: int, b: int, t: int):
    """(patterns [cycles, d] +-1, offsets [b, t] in [0, d)) of a site's orthogonal draws this step."""
    nblk = (d + 127) // 128
    pats = np.empty((cycles, d), dtype=np.float32)
    for c in range(cycles):
        w = _bits(seed, step, np.arange(nblk), 1, c, site)  # [nblk, 4]
        k = np.arange(d)
        bit = (w[k // 128, (k % 128) // 32] >> (k % 32).astype(np.uint64)) & np.uint64(1)
        pats[c] = 1.0 - 2.0 * bit.astype(np.float32)
    e = np.arange(b * t)
    x = philox4x32_10((e // 4).astype(np.uint64), (site << 2) | 2, 0, DOMAIN_DIRECT, seed, step)
    words = np.stack(x, axis=-1)
    offs = (words[e, e % 4] & np.uint32(d - 1)).astype(np.int64).reshape(b, t)
    return torch.from_numpy(pats), torch.from_numpy(offs)


def draw_signs(seed: int, step: int, site: int, draws, b: int, t: int) -> torch.Tensor:
    """Per-draw, per-token sign s [n, b, t] of global draw indices `draws`."""
    draws = np.asarray(draws)
    e = np.arange(b * t)
    out = np.empty((len(draws), b * t), dtype=np.float32)
    for i, idx in enumerate(draws):
        w = _bits(seed, step, e // 128, 3, int(idx), site)  # [bt, 4]
        bit = (w[np.arange(b * t), (e % 128) // 32] >> (e % 32).astype(np.uint64)) & np.uint64(1)
        out[i] = 1.0 - 2.0 * bit.astype(np.float32)
    return torch.from_numpy(out.reshape(len(draws), b, t))


def orthogonal_draws(patterns, offsets, signs, draws, d: int) -> torch.Tensor:
    """a[i, b, t, :] = H[(offset[b, t] + idx_i) mod d, :] * pattern[idx_i // d, :] * s[i, b, t]
    (run.py:235-237), for global draw indices `draws`."""
    H = hadamard(d)
    idx = torch.as_tensor(np.asarray(draws), dtype=torch.long)
    rows = (offsets.unsqueeze(0) + idx[:, None, None]) % d
    return H[rows] * patterns[idx // d][:, None, None, :] * signs[..., None]


def site_draws(seed, step, site: str, draws, b, t, d, total_draws):
    sid = site_id(site)
    cycles = -(-total_draws // d)
    pats, offs = frame(seed, step, sid, cycles, d, b, t)
    signs = draw_signs(seed, step, sid, draws, b, t)
    return orthogonal_draws(pats, offs, signs, draws, d)


def coordinate_differences(raw: torch.Tensor, y: torch.Tensor, sigma: float) -> torch.Tensor:
    """Central difference of each token's soft-capped CE along each of its own raw logits (run.py:120-137)."""
    cap = lambda v: 15 * torch.tanh(v / 15)
    z, up, down = cap(raw), cap(raw + sigma), cap(raw - sigma)
    weight = torch.softmax(z, -1)
    moved = lambda new: torch.log1p(weight * torch.expm1(new - z))
    change = moved(up) - moved(down)
    target = y.clamp(min=0).unsqueeze(-1)
    change = change.scatter_add(-1, target, -(up - down).gather(-1, target))
    return change / (2 * sigma) * (y >= 0).unsqueeze(-1)


def reward_to_go(reward: torch.Tensor, gamma: float) -> torch.Tensor:
    """Discounted sum of future rewards along t, truncated where gamma^lag < 1e-6 (run.py:81-86)."""
    lags = math.ceil(math.log(1e-6) / math.log(gamma))
    out = torch.zeros_like(reward)
    t = reward.shape[-1]
    for k in range(lags):
        out[..., :t - k] += gamma ** k * reward[..., k:]
    return out


def direct_errors(clean_loss, perturbed, draws_by_site: dict, sigma: float, n: int, gamma: float = 0.0,
                  priors: dict | None = None):
    """Sum over chunks of n draws of -(centred reward) . a / sigma, divided by the draw count
    (run.py:347-378). perturbed [N, b, t]; draws_by_site[site] = a [N, b, t, d]. With priors
    {site: mu [b, t, d]} (already masked like the draws), each reward gains the centred loss drop the
    prior predicts, sigma sum_s a_s . mu_s, after the reward-to-go, and the estimate gains
    (1 - 1/n) mu."""
    priors = priors or {}
    total = perturbed.shape[0]
    errors = {s: torch.zeros(a.shape[1:], dtype=torch.float64) for s, a in draws_by_site.items()}
    for c0 in range(0, total, n):
        reward = clean_loss.unsqueeze(0).double() - perturbed[c0:c0 + n].double()
        if n > 1:
            reward = reward - reward.mean(0, keepdim=True)
        if gamma:
            reward = reward_to_go(reward, gamma)
        if priors:
            predicted = sigma * sum(torch.einsum('nbtd,btd->nbt', draws_by_site[s][c0:c0 + n].double(), mu.double())
                                    for s, mu in priors.items())
            reward = reward + (predicted - predicted.mean(0, keepdim=True) if n > 1 else predicted)
        for s, a in draws_by_site.items():
            errors[s] -= torch.einsum('nbt,nbtd->btd', reward, a[c0:c0 + n].double()) / sigma
    kept = 1 - 1 / n if n > 1 else 1.0
    return {s: e / total + kept * priors[s].double() if s in priors else e / total for s, e in errors.items()}


def memory_matrix(S: torch.Tensor, P: torch.Tensor, ridge: float) -> torch.Tensor:
    """M = S (P + ridge mean(diag P) I)^-1 through a Cholesky factor (run.py:281-292)."""
    lam = ridge * P.diagonal().mean()
    L = torch.linalg.cholesky(P + lam * torch.eye(len(P), dtype=P.dtype))
    return torch.cholesky_solve(S.T, L).T


def remember(P, S: dict, c: torch.Tensor, estimates: dict, valid, beta: float):
    """EMA writes of the key covariance P and each site's S (run.py:304-314), single rank:
    C = c^T c / valid, G = sum_t delta_t c_t^T / valid."""
    cf = c.reshape(-1, c.shape[-1]).double()
    C = cf.T @ cf / valid
    P = beta * (P if P is not None else torch.zeros_like(C)) + (1 - beta) * C
    out = {}
    for site, e in estimates.items():
        G = torch.einsum('btd,btk->dk', e.double(), c.double()) / valid
        out[site] = beta * S.get(site, torch.zeros_like(G)) + (1 - beta) * G
    return P, out


def calibrate(calibration: dict, fits: dict, beta: float):
    """alpha per site from EMAs of <r, estimate> and |r|^2 (run.py:316-330); returns (calibration, alpha)."""
    cal, alpha = dict(calibration), {}
    for site, (dot, ret) in fits.items():
        if ret > 0:
            od, orr = cal.get(site, (dot, ret))
            cal[site] = (beta * od + (1 - beta) * dot, beta * orr + (1 - beta) * ret)
            alpha[site] = cal[site][0] / cal[site][1]
    return cal, alpha


def block_forward(p: dict, i: int, x, ve, cos, sin, jitter: dict):
    """Block i with optional additive jitter at o / attn / fc / mlp (run.py:102-117), fp32 [N, T, d]."""
    pre = f'transformer.h.{i}.'
    n, t, _ = x.shape
    h = om.rms_norm(x)
    q = (h @ p[pre + 'attn.c_q.weight'].t()).view(n, t, om.HEADS, om.HEAD_DIM)
    k = (h @ p[pre + 'attn.c_k.weight'].t()).view(n, t, om.HEADS, om.HEAD_DIM)
    v = (h @ p[pre + 'attn.c_v.weight'].t()).view(n, t, om.HEADS, om.HEAD_DIM)
    if ve is not None:
        gate = 2 * torch.sigmoid(h[..., :om.GATE_CHANNELS] @ p[pre + 'attn.ve_gate.weight'].t())
        v = v + gate.unsqueeze(-1) * ve.view(n, t, om.HEADS, om.HEAD_DIM)
    q, k = om.rms_norm(om.rope(q, cos, sin)), om.rms_norm(om.rope(k, cos, sin))
    y = om.window_attention(q, k, v, om.WINDOWS[i]).reshape(n, t, om.WIDTH)
    if 'o' in jitter:
        y = y + jitter['o']
    a = y @ p[pre + 'attn.c_proj.weight'].t()
    if 'attn' in jitter:
        a = a + jitter['attn']
    x = x + a
    hidden = om.rms_norm(x) @ p[pre + 'mlp.c_fc.weight'].t()
    if 'fc' in jitter:
        hidden = hidden + jitter['fc']
    m = F.relu(hidden).square() @ p[pre + 'mlp.c_proj.weight'].t()
    if 'mlp' in jitter:
        m = m + jitter['mlp']
    return x + m


def capture(p: dict, idx: torch.Tensor):
    """Clean forward keeping what the reruns and reassembly need (run.py:189-209, :244-254): the
    embedding rows, x0, block inputs (after mixing), value-embedding lookups, and per block the
    inputs of c_proj (y), c_fc (norm of the mid stream) and mlp.c_proj (relu^2), the MLP
    pre-activation, and the raw logits with the head's input."""
    b, t = idx.shape
    cos, sin = om.rotary_tables(t)
    emb = p['transformer.wte.weight'][idx]
    x = x0 = om.rms_norm(emb)
    cap = dict(emb=emb, x0=x0, blocks=[], ves=[], proj_in=[], fc_in=[], fc_pre=[], mlp_in=[])
    for i in range(om.LAYERS):
        pre = f'transformer.h.{i}.'
        x = p['resid_lambdas'][i] * x + p['x0_lambdas'][i] * x0
        cap['blocks'].append(x)
        ve = p[f'value_embeds.{i}.weight'][idx] if i in om.VE_LAYERS else None
        cap['ves'].append(ve)
        h = om.rms_norm(x)
        q = (h @ p[pre + 'attn.c_q.weight'].t()).view(b, t, om.HEADS, om.HEAD_DIM)
        k = (h @ p[pre + 'attn.c_k.weight'].t()).view(b, t, om.HEADS, om.HEAD_DIM)
        v = (h @ p[pre + 'attn.c_v.weight'].t()).view(b, t, om.HEADS, om.HEAD_DIM)
        if ve is not None:
            gate = 2 * torch.sigmoid(h[..., :om.GATE_CHANNELS] @ p[pre + 'attn.ve_gate.weight'].t())
            v = v + gate.unsqueeze(-1) * ve.view(b, t, om.HEADS, om.HEAD_DIM)
        q, k = om.rms_norm(om.rope(q, cos, sin)), om.rms_norm(om.rope(k, cos, sin))
        y = om.window_attention(q, k, v, om.WINDOWS[i]).reshape(b, t, om.WIDTH)
        cap['proj_in'].append(y)
        x = x + y @ p[pre + 'attn.c_proj.weight'].t()
        fc_in = om.rms_norm(x)
        fc_pre = fc_in @ p[pre + 'mlp.c_fc.weight'].t()
        mlp_in = F.relu(fc_pre).square()
        cap['fc_in'].append(fc_in)
        cap['fc_pre'].append(fc_pre)
        cap['mlp_in'].append(mlp_in)
        x = x + mlp_in @ p[pre + 'mlp.c_proj.weight'].t()
    cap['head_in'] = om.rms_norm(x)
    cap['raw'] = cap['head_in'] @ p['lm_head.weight'].t()
    return cap


def rerun(p: dict, cap: dict, idx, targets, n: int, entry, jitter: dict) -> torch.Tensor:
    """Per-token losses [n, b, t] of n jittered copies rerun from block `entry` (None: from the
    embedding, jitter['transformer.wte'] added before the norm), fp32 head (run.py:256-279).
    jitter maps 'o' / 'attn' / 'fc' / 'mlp' (or 'transformer.wte') to [n, b, t, d]."""
    b, t = idx.shape
    cos, sin = om.rotary_tables(t)
    flat = lambda a: a.reshape(n * b, t, -1)
    if entry is None:
        x = x0 = om.rms_norm(flat(cap['emb'].unsqueeze(0) + jitter['transformer.wte']))
        start = 0
    else:
        x = flat(cap['blocks'][entry].unsqueeze(0).expand(n, -1, -1, -1))
        x0 = flat(cap['x0'].unsqueeze(0).expand(n, -1, -1, -1))
        start = entry
    for i in range(start, om.LAYERS):
        if entry is None or i > entry:
            x = p['resid_lambdas'][i] * x + p['x0_lambdas'][i] * x0
        ve = cap['ves'][i]
        ve = None if ve is None else flat(ve.unsqueeze(0).expand(n, -1, -1, -1))
        sites = {k: flat(v) for k, v in jitter.items() if k != 'transformer.wte'} if i == entry else {}
        x = block_forward(p, i, x, ve, cos, sin, sites)
    logits = om.soft_cap(om.rms_norm(x) @ p['lm_head.weight'].t())
    tg = targets.unsqueeze(0).expand(n, -1, -1).reshape(-1)
    return F.cross_entropy(logits.reshape(-1, om.VOCAB), tg, reduction='none').view(n, b, t)


def reassemble(error: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """Weight gradient from output error and cached input: einsum('btd,bti->di') (run.py:465-471)."""
    return torch.einsum('btd,bti->di', error.double(), x.double())


def reassemble_embedding(error: torch.Tensor, idx: torch.Tensor, vocab: int = om.VOCAB) -> torch.Tensor:
    """Embedding gradient: rows of the error summed per token id (run.py:468-470, index_add)."""
    out = torch.zeros(vocab, error.shape[-1], dtype=torch.float64)
    return out.index_add_(0, idx.reshape(-1), error.reshape(-1, error.shape[-1]).double())


LOCAL_SITES = {'q': 'attn.c_q', 'k': 'attn.c_k', 'v': 'attn.c_v', 'gate': 'attn.ve_gate'}


def local_layers(kind: str):
    """Blocks with an estimate of `kind` (run.py:398): value embeddings and gates exist on VE blocks only."""
    return [i for i in range(om.LAYERS) if kind not in ('ve', 'gate') or i in om.VE_LAYERS]


def local_site(kind: str, i: int) -> str:
    return f'value_embeds.{i}' if kind == 've' else f'transformer.h.{i}.{LOCAL_SITES[kind]}'


def local_width(kind: str) -> int:
    return om.HEADS if kind == 'gate' else om.WIDTH


def attention_inputs(p: dict, cap: dict, idx, i: int):
    """Block i's raw q, k, v [b, t, h, d], gate logits z [b, t, h] and value-embedding rows (None off
    the VE blocks), recomputed from the captured block input (run.py:418-425)."""
    b, t = idx.shape
    pre = f'transformer.h.{i}.'
    h = om.rms_norm(cap['blocks'][i])
    q, k, v = ((h @ p[pre + f'attn.c_{n}.weight'].t()).view(b, t, om.HEADS, om.HEAD_DIM) for n in 'qkv')
    z = ve = None
    if i in om.VE_LAYERS:
        z = h[..., :om.GATE_CHANNELS] @ p[pre + 'attn.ve_gate.weight'].t()
        ve = p[f'value_embeds.{i}.weight'][idx].view(b, t, om.HEADS, om.HEAD_DIM)
    return q, k, v, z, ve


def local_credit(t: int, window: int, gamma: float) -> torch.Tensor:
    """credit[t', s] = gamma^(s - t') for 0 <= s - t' <= window (run.py:428-430)."""
    pos = torch.arange(t)
    lag = pos[None, :] - pos[:, None]
    return ((lag >= 0) & (lag <= window)).double() * gamma ** lag.clamp(min=0).double()


def local_errors(p: dict, cap: dict, idx, kind: str, draws_by_layer: dict, targets: dict, sigma: float = 0.1,
                 gamma: float = 0.98, n: int = 16) -> dict:
    """Attention-internal errors of one kind (run.py:391-463) for every block that has it, from the
    draws a [N, b, t, width] given per block, scored against the hub targets [b, t, 512]:
      q, k   delta = attention with the perturbed (RoPE'd, normed) side minus the clean attention
      v, ve  delta = attention of the value change sigma a (ve: x 2 sigmoid(z))
      gate   delta = attention of (2 sigmoid(z + sigma a) - 2 sigmoid(z - sigma a)) ve, divisor 2 sigma
    score = <target, delta> per head; all kinds but q spread it back over earlier tokens by the lag
    credit; errors = sum_draws score a / divisor / N. Returns {site: [b, t, width]} in float64."""
    b, t = idx.shape
    cos, sin = om.rotary_tables(t)
    h, d = om.HEADS, om.HEAD_DIM
    processed = lambda raw: om.rms_norm(om.rope(raw, cos, sin))  # noqa: E731
    out = {}
    for i in local_layers(kind):
        q, k, v, z, ve = attention_inputs(p, cap, idx, i)
        values = v if z is None else v + (2 * torch.sigmoid(z)).unsqueeze(-1) * ve
        qp, kp = processed(q), processed(k)
        window = om.WINDOWS[i]
        baseline = om.window_attention(qp, kp, values, window)
        credit = local_credit(t, window, gamma)
        tgt = targets[i].view(b, t, h, d).double()
        a_all = draws_by_layer[i].float()
        total = a_all.shape[0]
        err = torch.zeros(b, t, local_width(kind), dtype=torch.float64)
        rep = lambda x, m: x.unsqueeze(0).expand(m, *x.shape).reshape(m * b, t, h, d)  # noqa: E731
        for c0 in range(0, total, n):
            a = a_all[c0:c0 + n]
            m = a.shape[0]
            divisor = sigma
            if kind in ('q', 'k'):
                raw = q if kind == 'q' else k
                moved = processed((raw.unsqueeze(0) + sigma * a.view(m, b, t, h, d)).reshape(m * b, t, h, d))
                qa, ka = (moved, rep(kp, m)) if kind == 'q' else (rep(qp, m), moved)
                delta = om.window_attention(qa, ka, rep(values, m), window).view(m, b, t, h, d) - baseline
            else:
                if kind == 'gate':
                    dv = (2 * torch.sigmoid(z + sigma * a) - 2 * torch.sigmoid(z - sigma * a)).unsqueeze(-1) * ve
                    divisor = 2 * sigma
                else:
                    dv = sigma * a.view(m, b, t, h, d)
                    if kind == 've':
                        dv = dv * (2 * torch.sigmoid(z)).unsqueeze(-1)
                delta = om.window_attention(rep(qp, m), rep(kp, m), dv.reshape(m * b, t, h, d),
                                            window).view(m, b, t, h, d)
            score = torch.einsum('bthd,nbthd->nbth', tgt, delta.double())
            if kind != 'q':
                score = torch.einsum('nbsh,ts->nbth', score, credit)
            est = torch.einsum('nbth,nbthd->bthd', score, a.double().view(m, b, t, h, -1))
            err += est.reshape(b, t, -1) / divisor
        out[local_site(kind, i)] = err / total
    return out


def local_input(cap: dict, kind: str, i: int) -> torch.Tensor:
    """The cached input of a local site's module: the block's normed input (its first 32 channels for
    the gate); value embeddings reassemble by token id instead."""
    h = om.rms_norm(cap['blocks'][i])
    return h[..., :om.GATE_CHANNELS] if kind == 'gate' else h
