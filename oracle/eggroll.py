"""EGGROLL bookkeeping, fitness shaping, update reconstruction and AdamW, restated on CPU
(test infrastructure; see oracle/__init__.py).

Reference: `train/val/eggroll.py` (member indexing :134-146, fitness :151-154, reconstruction
:155-166, AdamW :205) and torch's AdamW arithmetic for the optimizer step.
"""
from __future__ import annotations

import numpy as np
import torch

from . import model as om
from .philox import gaussians

BETAS = (0.5, 0.95)   # train/val/eggroll.py:32
ADAM_EPS = 1e-8       # train/val/eggroll.py:205


def member_direction(j, pairs: int):
    """Member j evaluates direction (j mod 2P) // 2 (train/val/eggroll.py:140)."""
    return (np.asarray(j) % (2 * pairs)) // 2


def member_sign(j, sigma: float):
    """+sigma for even members, -sigma for odd ones (train/val/eggroll.py:138)."""
    return np.where(np.asarray(j) % 2 == 0, sigma, -sigma)


def draws_for(directions, seed: int, step: int, dtype=torch.float32) -> dict:
    """The noise dict `population_loss` consumes (train/val/eggroll.py:122-128), built from the
    counter-based stream instead of the reference's 2^28 buffer: name -> (a [n, rows], b [n, cols])
    for matrices and embeddings, eps [n, 8] for the mixing scalars."""
    directions = np.asarray(directions, dtype=np.uint64)
    out = {}
    for tid, (name, shape) in enumerate(om.PARAM_SPECS):
        if len(shape) == 1:
            out[name] = torch.from_numpy(gaussians(seed, step, tid, 0, directions, shape[0])).to(dtype)
        else:
            a = torch.from_numpy(gaussians(seed, step, tid, 0, directions, shape[0])).to(dtype)
            b = torch.from_numpy(gaussians(seed, step, tid, 1, directions, shape[1])).to(dtype)
            out[name] = (a, b)
    return out


def member_draws(members, pairs: int, sigma: float, seed: int, step: int, dtype=torch.float32):
    """(draws dict, sign [n]) for a list of member indices."""
    members = np.asarray(members)
    dirs = member_direction(members, pairs)
    return draws_for(dirs, seed, step, dtype), torch.tensor(member_sign(members, sigma), dtype=dtype)


def fitness_zscore(losses: np.ndarray, pairs: int) -> np.ndarray:
    """Per-direction weights of train/val/eggroll.py:151-154: antithetic difference
    L(minus) - L(plus) over its unbiased std (+1e-8), summed over the members that share a direction."""
    losses = np.asarray(losses, dtype=np.float64)
    f = losses[1::2] - losses[0::2]
    f = f / (f.std(ddof=1) + 1e-8)
    w = np.zeros(pairs)
    np.add.at(w, np.arange(len(f)) % pairs, f)
    return w


def centered_ranks(losses: np.ndarray) -> np.ndarray:
    """Rank of each loss in ascending order (ties by member index, NaN last) mapped to
    rank / (N - 1) - 0.5. Ranks are integers and bit-exact by construction."""
    losses = np.asarray(losses, dtype=np.float32)
    key = np.where(np.isnan(losses), np.float32(np.inf), losses)
    nan_last = np.isnan(losses).astype(np.int8)
    order = np.lexsort((np.arange(len(losses)), key, nan_last))
    ranks = np.empty(len(losses), dtype=np.int64)
    ranks[order] = np.arange(len(losses))
    return ranks


def fitness_centered_rank(losses: np.ndarray, pairs: int) -> np.ndarray:
    """Direction weights from centred ranks: cr(minus) - cr(plus), summed per direction."""
    n = len(losses)
    r = centered_ranks(losses).astype(np.float64)
    cr = r / max(n - 1, 1) - 0.5
    f = cr[1::2] - cr[0::2]
    w = np.zeros(pairs)
    np.add.at(w, np.arange(len(f)) % pairs, f)
    return w


def sum_fe(weights: np.ndarray, n_fitness: int, seed: int, step: int, chunk: int = 64,
           names=None, dtype=torch.float64) -> dict:
    """g = -sum_p w_p a_p b_p^T / n_fitness per matrix, -sum_p w_p eps_p / n_fitness per scalar
    vector (train/val/eggroll.py:155-166), regenerating the draws chunk by chunk."""
    pairs = len(weights)
    specs = [(n, s) for n, s in om.PARAM_SPECS if names is None or n in names]
    grads = {n: torch.zeros(s, dtype=dtype) for n, s in specs}
    w_all = torch.tensor(weights, dtype=dtype)
    for c0 in range(0, pairs, chunk):
        dirs = np.arange(c0, min(pairs, c0 + chunk))
        w = w_all[c0:c0 + len(dirs)]
        for name, shape in specs:
            tid = om.TENSOR_ID[name]
            if len(shape) == 1:
                eps = torch.from_numpy(gaussians(seed, step, tid, 0, dirs, shape[0])).to(dtype)
                grads[name] -= w @ eps
            else:
                a = torch.from_numpy(gaussians(seed, step, tid, 0, dirs, shape[0])).to(dtype)
                b = torch.from_numpy(gaussians(seed, step, tid, 1, dirs, shape[1])).to(dtype)
                grads[name] -= (w[:, None] * a).t() @ b
    return {n: g / n_fitness for n, g in grads.items()}


def adamw_step(p, g, m, v, t: int, lr: float, betas=BETAS, eps=ADAM_EPS, weight_decay=0.0):
    """One AdamW step in torch's arithmetic order (decoupled decay, then m lerp, v update, bias
    corrections on the step size and on sqrt(v)). Updates p, m, v in place."""
    b1, b2 = betas
    if weight_decay:
        p.mul_(1 - lr * weight_decay)
    m.lerp_(g, 1 - b1)
    v.mul_(b2).addcmul_(g, g, value=1 - b2)
    bc1 = 1 - b1 ** t
    bc2 = 1 - b2 ** t
    denom = (v.sqrt() / (bc2 ** 0.5)).add_(eps)
    p.addcdiv_(m, denom, value=-lr / bc1)
    return p, m, v
