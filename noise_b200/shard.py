"""Sharded ES update: partial reconstruction, reduce-scatter, a sharded optimizer step, parameter
all-gather.

The reference rebuilds every direction on every rank (train/val/eggroll.py:155-163), so each rank
does O(P x params) work per update whatever the world size. Here rank r contracts only its own
directions [r P / W, (r + 1) P / W) (noise_sum_fe_partial), the W partial sums meet in one NCCL
reduce-scatter that leaves each rank the summed gradient of the tensors it owns, the optimizer steps
those tensors only (its moments and ANVIL rails exist for them alone), and an all-gather of the
updated parameters restores the full model on every rank.

Ownership is a `ShardPlan`: the 60 parameter tensors in named_parameters order cut into W contiguous
runs of whole tensors with balanced sizes, so that every ANVIL matrix sits whole on one rank (its
polar maps need the whole matrix). Each run is padded to the plan's common size S, which is the unit
NCCL's reduce-scatter and all-gather exchange: the partial sums are written straight into that padded
layout (tensor t at out_offsets[t]), rank r's region is [r S, r S + count_r).

`ShardedOptimizer` keeps the duck type of `noise_b200.eggroll.AdamW` (param_groups, zero_grad,
set_sum_fe, step), so `Eggroll.step` drives it unchanged; `kind='anvil'` applies ANVIL II to the block
matrices and AdamW (lr x 300 / 30 / 1) elsewhere, the split of train/val/run.py:643-656.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .model import PARAM_SPECS, Weights
from .optim import AdamWDense, Anvil, adam_scale, is_anvil_matrix

ALIGN = 64  # floats: regions start on 256-byte boundaries


class ShardPlan:
    """Balanced contiguous partition of the parameter tensors over `world` ranks."""

    def __init__(self, world: int):
        if world < 1:
            raise ValueError('world must be >= 1')
        self.world = world
        self.sizes = [math.prod(s) for _, s in PARAM_SPECS]
        self.offsets = [0]
        for n in self.sizes:
            self.offsets.append(self.offsets[-1] + n)
        self.bounds = self._partition()
        self.begin = [self.offsets[self.bounds[r]] for r in range(world)]
        self.count = [self.offsets[self.bounds[r + 1]] - self.begin[r] for r in range(world)]
        self.size = -(-max(self.count) // ALIGN) * ALIGN
        self.owner = [0] * len(self.sizes)
        for r in range(world):
            for t in range(self.bounds[r], self.bounds[r + 1]):
                self.owner[t] = r
        # where tensor t's partial sum goes in the padded [world * size] layout
        self.out_offsets = [self.owner[t] * self.size + self.offsets[t] - self.begin[self.owner[t]]
                            for t in range(len(self.sizes))]

    def _partition(self) -> list[int]:
        """Tensor boundaries [0 = b_0 <= ... <= b_W = 60] minimising the largest run (greedy fill at the
        smallest feasible capacity, found by bisection)."""
        def cuts(cap):
            b, run = [0], 0
            for t, n in enumerate(self.sizes):
                if run + n > cap and run > 0:
                    b.append(t)
                    run = 0
                run += n
            return b

        lo, hi = max(self.sizes), sum(self.sizes)
        while lo < hi:
            mid = (lo + hi) // 2
            if len(cuts(mid)) <= self.world:
                hi = mid
            else:
                lo = mid + 1
        b = cuts(lo)
        b += [len(self.sizes)] * (self.world + 1 - len(b))
        return b

    def region(self, rank: int) -> _lib.NoiseRegion:
        return _lib.NoiseRegion(self.bounds[rank], self.bounds[rank + 1], self.begin[rank])

    def directions(self, rank: int, pairs: int) -> tuple[int, int]:
        """[begin, count) of the directions rank `rank` contracts."""
        lo, hi = rank * pairs // self.world, (rank + 1) * pairs // self.world
        return lo, hi - lo

    def offsets_array(self):
        return (ctypes.c_int64 * len(self.out_offsets))(*self.out_offsets)


class LibraryKernels:
    """The CUDA library calls the sharded update makes (a CPU stand-in replaces them in host tests)."""

    def partial(self, fw: torch.Tensor, pairs: int, d0: int, dn: int, scale: float, seed: int, step: int, offsets,
                out: torch.Tensor):
        _lib.call('noise_sum_fe_partial', fw.data_ptr(), pairs, d0, dn, float(scale), seed & 0xFFFFFFFF,
                  step & 0xFFFFFFFF, ctypes.addressof(offsets), out.data_ptr(),
                  torch.cuda.current_stream(out.device).cuda_stream)


class ShardedOptimizer:
    """The sharded update behind the AdamW duck type of noise_b200.eggroll (set_sum_fe + step).

    kind 'adamw': torch.optim.AdamW on every tensor (the EGGROLL reference's optimizer); 'anvil':
    ANVIL II on the block matrices and AdamW x300 / x30 / x1 elsewhere (train/val/run.py:643-656).
    Collectives run on the default process group when world > 1; every rank makes the same calls in
    the same order. `kernels` and `optimizers` (objects with step(region_grad)) replace the library
    calls and the region optimizers, for host-logic tests."""

    def __init__(self, weights: Weights, rank: int = 0, world: int = 1, kind: str = 'adamw', lr: float = 1e-3,
                 betas=(0.5, 0.95), eps: float = 1e-8, weight_decay: float = 0.0, anvil_lr: float = 0.02,
                 anvil_wd: float = 0.0, steps: int = 610, lr_mult=None, kernels=None, optimizers=None):
        if kind not in ('adamw', 'anvil'):
            raise ValueError(kind)
        self.w, self.rank, self.world, self.kind = weights, rank, world, kind
        self.kernels = kernels or LibraryKernels()
        self.plan = ShardPlan(world)
        self.region = self.plan.region(rank)
        dev = weights.device
        # the padding after each region is never written, so it stays zero through every reduce-scatter
        self.partial = torch.zeros(world * self.plan.size, dtype=torch.float32, device=dev)
        self.grad = self.partial[:self.plan.size] if world == 1 else \
            torch.empty(self.plan.size, dtype=torch.float32, device=dev)
        if world > 1:
            self.send = torch.empty(self.plan.size, dtype=torch.float32, device=dev)
            self.gathered = torch.empty(world * self.plan.size, dtype=torch.float32, device=dev)
        self.param_groups = []
        if optimizers is not None:
            self.optimizers = list(optimizers)
        else:
            owned = {PARAM_SPECS[t][0] for t in range(self.region.tensor_begin, self.region.tensor_end)}
            if kind == 'adamw':
                mult = None if lr_mult is None else {PARAM_SPECS[t][0]: float(lr_mult[t])
                                                     for t in range(len(PARAM_SPECS))}
                adam = AdamWDense(weights, lr, betas, eps, weight_decay, region=self.region, names=owned,
                                  scale=(lambda n: 1.0) if mult is None else mult.__getitem__)
                self.optimizers = [adam]
            else:
                anvil = Anvil(weights, anvil_lr, anvil_wd, steps, region=self.region)
                adam_names = {n for n, s in PARAM_SPECS if not is_anvil_matrix(n, s)}
                adam = AdamWDense(weights, lr, betas, eps, weight_decay, region=self.region, names=owned & adam_names,
                                  scale=adam_scale)
                self.optimizers = [anvil, adam]
                self.param_groups += anvil.param_groups
            self.param_groups += adam.param_groups
            if not adam.param_groups:  # a rank owning only ANVIL matrices still exposes the Adam lr
                self.param_groups.append(dict(names=[], lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay))
            self.optimizers = [o for o in self.optimizers if not isinstance(o, AdamWDense) or o.param_groups]
        self._pending = None
        self._offsets = self.plan.offsets_array()

    def zero_grad(self, set_to_none=True):
        self._pending = None

    def set_sum_fe(self, fitness_weights: torch.Tensor, grad_scale: float, seed: int, step: int):
        self._pending = (fitness_weights, grad_scale, seed, step)

    @torch.no_grad()
    def step(self):
        if self._pending is None:
            return
        fw, scale, seed, step = self._pending
        self._pending = None
        self.reconstruct(fw, scale, seed, step)
        self.exchange_gradients()
        for opt in self.optimizers:
            opt.step(self.grad)
        self.exchange_parameters()

    @torch.no_grad()
    def step_dense(self, flat: torch.Tensor, scale: float = 1.0) -> bool:
        """One update from this rank's share of a dense gradient in the flat layout (DUST's estimate,
        whose draws are split over the ranks): the shares are summed by the reduce-scatter, times
        `scale` (1 / world for the reference's average, train/val/run.py:536, average_ranks at :154-158), each rank steps its
        region and the all-gather restores the model. The reference checks the averaged gradient for
        non-finite values before stepping (:537-538); here every rank checks its summed region and the
        result is all-reduced, so all ranks skip together. Returns False (nothing stepped) on a
        non-finite gradient."""
        plan = self.plan
        for r in range(self.world):
            if plan.count[r]:
                self.partial[r * plan.size:r * plan.size + plan.count[r]].copy_(
                    flat[plan.begin[r]:plan.begin[r] + plan.count[r]])
        self.exchange_gradients()
        n = plan.count[self.rank]
        if scale != 1.0:
            self.grad[:n].mul_(scale)
        bad = (~torch.isfinite(self.grad[:n])).any().to(torch.float32).reshape(1)
        if self.world > 1:
            torch.distributed.all_reduce(bad)
        if bad.item():
            return False
        for opt in self.optimizers:
            opt.step(self.grad)
        self.exchange_parameters()
        return True

    def reconstruct(self, fw: torch.Tensor, scale: float, seed: int, step: int):
        """This rank's directions, contracted into the padded layout of every tensor."""
        pairs = fw.numel()
        d0, dn = self.plan.directions(self.rank, pairs)
        self.kernels.partial(fw, pairs, d0, dn, scale, seed, step, self._offsets, self.partial)

    def exchange_gradients(self):
        """Sum the ranks' partials; this rank keeps its region (self.grad)."""
        if self.world > 1:
            torch.distributed.reduce_scatter_tensor(self.grad, self.partial)

    def exchange_parameters(self):
        """Every rank's updated region into every rank's parameters, then the packed bf16 copy."""
        if self.world == 1:
            return
        plan, flat = self.plan, self.w.flat
        b, n = plan.begin[self.rank], plan.count[self.rank]
        self.send[:n].copy_(flat[b:b + n])
        torch.distributed.all_gather_into_tensor(self.gathered, self.send)
        for r in range(self.world):
            if r != self.rank and plan.count[r]:
                flat[plan.begin[r]:plan.begin[r] + plan.count[r]].copy_(
                    self.gathered[r * plan.size:r * plan.size + plan.count[r]])
        self.w.pack()
