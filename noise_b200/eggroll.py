"""EGGROLL on B200: the host-side mirror of `train/val/eggroll.py` (Eggroll :106-168, AdamW :205).

Same knobs and the same control flow as the reference, with the work in CUDA:
  - population evaluation  -> noise_pop_forward_lowrank (one launch sequence per member block)
  - loss all-gather        -> torch.distributed (NCCL) when world > 1, as in the reference
  - fitness                -> noise_fitness (z-score as in the reference, or centred ranks)
  - reconstruction + AdamW -> noise_update_sum_fe_adamw (draws regenerated in-kernel)
The reference slices each direction's draws out of a fixed 2^28 Gaussian buffer at random offsets;
here a direction's draws are the counter-based stream keyed by (seed, step, direction, tensor), so
every rank regenerates any direction without communication, as in the reference.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .model import Weights
from .population import population_losses

BATCH = 8            # train/val/eggroll.py:28
SEED = 0
PAIRS = 131072
SIGMA = 0.002
LR, BETAS = 0.001, (0.5, 0.95)
WARMDOWN = 0.3
CHUNK = 256          # pairs per member block (2 * CHUNK members per population call)

FITNESS_MODES = {'zscore': 0, 'centered_rank': 1}


@dataclass
class CounterNoise:
    """The draws of members [begin, begin + count): direction (j mod 2P) // 2, sign +sigma for even j.
    Stands in for the reference's `noise` dict; kernels regenerate the values."""
    begin: int
    count: int
    pairs: int
    sigma: float
    seed: int
    step: int


def population_loss(model: Weights, p, noise: CounterNoise, sign, idx, targets) -> torch.Tensor:
    """Drop-in for train/val/eggroll.py:66 population_loss: mean CE [m] of the noise's members on one
    sequence idx/targets [T] (or every row of [B, T]). `p` and `sign` are implied by `model` and `noise`."""
    del p, sign
    return population_losses(model, idx, targets, noise.begin, noise.count, noise.pairs, noise.sigma,
                             noise.seed, noise.step)


class AdamW:
    """torch.optim.AdamW's duck type over the flat master buffer (`param_groups`, `zero_grad`, `step`).

    The gradient is not a dense tensor: the estimator hands over the fitness weights and the draw
    key, and `step()` reconstructs sum_d w_d eps_d and applies AdamW in one kernel."""

    def __init__(self, weights: Weights, lr=LR, betas=BETAS, eps=1e-8, weight_decay=0.0, lr_mult=None):
        self.w = weights
        self.param_groups = [dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay)]
        self.exp_avg = torch.zeros_like(weights.flat)
        self.exp_avg_sq = torch.zeros_like(weights.flat)
        self.lr_mult = None if lr_mult is None else torch.as_tensor(lr_mult, dtype=torch.float32,
                                                                    device=weights.device)
        self.t = 0
        self._pending = None

    def zero_grad(self, set_to_none=True):
        self._pending = None

    def set_sum_fe(self, fitness_weights: torch.Tensor, grad_scale: float, seed: int, step: int):
        self._pending = (fitness_weights, grad_scale, seed, step)

    def step(self):
        if self._pending is None:
            return
        fw, scale, seed, step = self._pending
        g = self.param_groups[0]
        self.t += 1
        _lib.call('noise_update_sum_fe_adamw', self.w.flat.data_ptr(), self.w.packed.data_ptr(),
                  self.exp_avg.data_ptr(), self.exp_avg_sq.data_ptr(), fw.data_ptr(), fw.numel(), float(scale),
                  seed & 0xFFFFFFFF, step & 0xFFFFFFFF,
                  None if self.lr_mult is None else self.lr_mult.data_ptr(), float(g['lr']), float(g['betas'][0]),
                  float(g['betas'][1]), float(g['eps']), float(g['weight_decay']), self.t, None,
                  torch.cuda.current_stream(self.w.device).cuda_stream)
        self._pending = None


def fitness_weights(losses: torch.Tensor, pairs: int, mode: str = 'zscore', ranks: torch.Tensor | None = None):
    """Per-direction weights [pairs] from member losses [2 * n] (noise_fitness)."""
    n = losses.numel()
    lib = _lib.load()
    ws = torch.empty(lib.noise_fitness_workspace_bytes(n), dtype=torch.uint8, device=losses.device)
    out = torch.empty(pairs, dtype=torch.float32, device=losses.device)
    _lib.call('noise_fitness', losses.data_ptr(), n, pairs, FITNESS_MODES[mode], out.data_ptr(),
              None if ranks is None else ranks.data_ptr(), ws.data_ptr(), ws.numel(),
              torch.cuda.current_stream(losses.device).cuda_stream)
    return out


class Eggroll:
    """Mirror of train/val/eggroll.py:106-168.

    all_sequences=False keeps the reference's layout: members = max(2P, 2B), member j evaluates
    sequence j // (members / B). all_sequences=True makes every member evaluate all B sequences
    (members = 2P), the configuration the B200 benchmark is quoted on."""

    def __init__(self, model: Weights, pairs: int, rank: int = 0, world: int = 1, sigma: float = SIGMA,
                 seed: int = SEED, fitness: str = 'zscore', all_sequences: bool = False, chunk: int = CHUNK):
        self.model, self.pairs, self.rank, self.world = model, pairs, rank, world
        self.sigma, self.seed, self.fitness, self.all_sequences, self.chunk = sigma, seed, fitness, all_sequences, chunk
        self.device = model.device
        self.loss = population_loss
        self.last_losses = None

    def members(self, batch: int) -> int:
        return 2 * self.pairs if self.all_sequences else max(2 * self.pairs, 2 * batch)

    def evaluate(self, x: torch.Tensor, y: torch.Tensor, step: int) -> torch.Tensor:
        """This rank's member losses [members / world] (device)."""
        members = self.members(len(x))
        begin, end = self.member_range(len(x))
        per_rank = end - begin
        if self.all_sequences:
            noise = CounterNoise(begin, per_rank, self.pairs, self.sigma, self.seed, step)
            return self.loss(self.model, None, noise, None, x, y)
        per_seq = members // len(x)
        losses = torch.empty(per_rank, device=self.device)
        start = begin
        while start < end:  # blocks of up to 2 * chunk members, never straddling two sequences
            seq = start // per_seq
            count = min(2 * self.chunk, end - start, (seq + 1) * per_seq - start)
            noise = CounterNoise(start, count, self.pairs, self.sigma, self.seed, step)
            losses[start - begin:start - begin + count] = self.loss(self.model, None, noise, None, x[seq], y[seq])
            start += count
        return losses

    def member_range(self, batch: int) -> tuple[int, int]:
        """[begin, end) of the members this rank evaluates (train/val/eggroll.py:134-139)."""
        members = self.members(batch)
        if members % self.world:
            raise ValueError(f'{members} members do not split over {self.world} ranks')
        per_rank = members // self.world
        return self.rank * per_rank, (self.rank + 1) * per_rank

    def gather(self, losses: torch.Tensor) -> torch.Tensor:
        """All ranks' member losses in member order (train/val/eggroll.py:147-150)."""
        if self.world == 1:
            return losses
        gathered = [torch.empty_like(losses) for _ in range(self.world)]
        torch.distributed.all_gather(gathered, losses)
        return torch.cat(gathered)

    @torch.no_grad()
    def step(self, x, y, optimizer: AdamW, step: int) -> float:
        """Evaluate this rank's share of the population, gather the losses, rebuild the update everywhere."""
        losses = self.gather(self.evaluate(x, y, step))
        self.last_losses = losses
        w = fitness_weights(losses, self.pairs, self.fitness)
        optimizer.zero_grad(set_to_none=True)
        optimizer.set_sum_fe(w, 1.0 / (losses.numel() // 2), self.seed, step)
        optimizer.step()
        return losses.mean().item()
