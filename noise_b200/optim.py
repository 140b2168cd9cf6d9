"""Optimizers for dense gradients: ANVIL II on the block matrices and AdamW elsewhere, the
`make_optimizer` split of train/val/run.py:629-656, on noise_b200's kernels.

ANVIL's elementwise and reduction passes run in noise_anvil_region_prepare / _finish, batched over
the block matrices of a region (all 48 by default); its six quintic maps (`polar`, run.py:572-580)
run between them in noise_anvil_region_polar: each matrix's wide form (a tall c_fc transposed, as
polar does) through X <- a X + (b S + c S S) X, S = X X^T, as batched tcgen05 GEMMs in bf16 storage
with fp32 accumulation.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .model import PARAM_SPECS, Weights

# The six (a, b, c) quintic maps of ANVIL II (train/val/run.py:560-567): tuned constants that define
# the method, kept identical.
MAPS = (
    (3.923798038567, -6.095026865488, 3.905234618423),
    (3.278126713798, -3.328923386476, 0.989127286973),
    (3.505298394150, -5.137358782410, 1.968325560615),
    (2.815058591845, -3.685181239622, 1.417196497642),
    (2.245503932403, -2.443826979899, 0.963091710461),
    (2.256537145403, -2.166840097229, 0.929501253245),
)
RUN = (1194, 240, 50, 514)  # total, warmup, cooldown, engage steps of the schedule (run.py:568-569)


def is_anvil_matrix(name: str, shape) -> bool:
    return name.startswith('transformer.h.') and len(shape) == 2 and 've_gate' not in name


def adam_scale(name: str) -> float:
    return 300.0 if ('wte' in name or 'value_embeds' in name) else 30.0 if 'lambdas' in name else 1.0


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


class DenseGrad:
    """A flat gradient buffer with the parameter layout, filled tensor by tensor."""

    def __init__(self, w: Weights):
        self.flat = torch.zeros_like(w.flat)
        self.views, off = {}, 0
        for n, s in PARAM_SPECS:
            k = 1
            for d in s:
                k *= d
            self.views[n] = self.flat[off:off + k].view(s)
            off += k


def whole_region() -> _lib.NoiseRegion:
    """The region of every tensor: the flat buffer itself."""
    return _lib.NoiseRegion(0, len(PARAM_SPECS), 0)


def region_numel(region: _lib.NoiseRegion) -> int:
    """Elements a region buffer needs: from `base` to the end of its last tensor."""
    end = sum(math.prod(s) for _, s in PARAM_SPECS[:region.tensor_end])
    return end - region.base


class AdamWDense:
    """AdamW on dense gradients for the non-ANVIL tensors, lr = base lr x adam_scale(name).

    On a region (noise_b200.shard), only the region's tensors are stepped and the moments are region
    buffers; `names` limits the tensors (all non-ANVIL ones by default)."""

    def __init__(self, w: Weights, lr: float, betas, eps=1e-8, weight_decay=0.0, region=None, names=None,
                 scale=adam_scale):
        self.w = w
        self.region = region or whole_region()
        n = region_numel(self.region)
        self.m = torch.zeros(n, dtype=torch.float32, device=w.device)
        self.v = torch.zeros(n, dtype=torch.float32, device=w.device)
        self.t = 0
        self.param_groups = []
        groups = {}
        for nm, sh in PARAM_SPECS:
            if (names is None and not is_anvil_matrix(nm, sh)) or (names is not None and nm in names):
                groups.setdefault(scale(nm), []).append(nm)
        for sc, group in groups.items():
            self.param_groups.append(dict(names=group, lr=lr * sc, betas=tuple(betas), eps=eps,
                                          weight_decay=weight_decay))

    def step(self, grad):
        """grad: a DenseGrad (whole buffer) or a region buffer tensor."""
        flat = grad.flat if isinstance(grad, DenseGrad) else grad
        self.t += 1
        lrs = [-1.0] * len(PARAM_SPECS)
        index = {n: i for i, (n, _) in enumerate(PARAM_SPECS)}
        for g in self.param_groups:
            for n in g['names']:
                lrs[index[n]] = float(g['lr'])
        lr_arr = (ctypes.c_float * len(lrs))(*lrs)
        g0 = self.param_groups[0]
        _lib.call('noise_adamw_region', self.w.flat.data_ptr(), self.w.packed.data_ptr(), self.m.data_ptr(),
                  self.v.data_ptr(), flat.data_ptr(), ctypes.byref(self.region), ctypes.addressof(lr_arr),
                  float(g0['betas'][0]), float(g0['betas'][1]), float(g0['eps']), float(g0['weight_decay']), self.t,
                  _stream(self.w.device))


class Anvil:
    """ANVIL II (modded-nanogpt PR #360) as in train/val/run.py:583-626, on the block matrices of a
    region (all 48 by default)."""

    def __init__(self, w: Weights, lr: float, weight_decay: float, steps: int, lane_beta=0.9, beta_min=0.85,
                 beta_max=0.93, slow_beta=0.98, fast_beta=0.85, fast_weight=0.4385, region=None):
        self.w = w
        self.region = region or whole_region()
        self.param_groups = [dict(lr=lr, weight_decay=weight_decay)]
        self.total, self.warmup, self.cooldown, self.engage = (round(k * steps / RUN[0]) for k in RUN)
        self.lane_beta, self.beta_min, self.beta_max = lane_beta, beta_min, beta_max
        self.slow_beta, self.fast_beta, self.fast_weight = slow_beta, fast_beta, fast_weight
        self.t = 0
        dev = w.device
        tiles, lanes, mats = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int()
        _lib.call('noise_anvil_region_sizes', ctypes.byref(self.region), ctypes.addressof(tiles),
                  ctypes.addressof(lanes), ctypes.addressof(mats))
        self.matrices = mats.value
        n = region_numel(self.region)
        self.fast = torch.zeros(n, dtype=torch.float32, device=dev)
        self.slow = torch.zeros(n, dtype=torch.float32, device=dev)
        self.scratch = torch.zeros(n, dtype=torch.float32, device=dev)
        self.x = torch.zeros(n, dtype=torch.bfloat16, device=dev)
        self.energy = torch.zeros(max(1, lanes.value), dtype=torch.float32, device=dev)
        self.partials = torch.zeros(max(1, 2 * tiles.value), dtype=torch.float32, device=dev)
        self.scalars = torch.zeros(max(1, mats.value), dtype=torch.float32, device=dev)
        self._polar_ws = None

    def rail_beta(self):
        lo, hi, cool = self.beta_min, self.beta_max, self.total - self.cooldown
        if self.t < self.warmup:
            return lo + (hi - lo) * self.t / self.warmup
        if self.t > cool:
            return hi - (hi - lo) * (self.t - cool) / self.cooldown
        return hi

    def _polar_maps(self):
        dev = self.w.device
        if self._polar_ws is None:
            n = int(_lib.load().noise_anvil_polar_workspace_bytes(ctypes.byref(self.region)))
            self._polar_ws = torch.empty(max(1, n), dtype=torch.uint8, device=dev)
            self._maps = torch.tensor([v for m in MAPS for v in m], dtype=torch.float32)
        _lib.call('noise_anvil_region_polar', ctypes.byref(self.region), self.x.data_ptr(), self._maps.data_ptr(),
                  len(MAPS), self._polar_ws.data_ptr(), self._polar_ws.numel(), None, _stream(dev))

    @torch.no_grad()
    def step(self, grad):
        """grad: a DenseGrad (whole buffer) or a region buffer tensor."""
        flat = grad.flat if isinstance(grad, DenseGrad) else grad
        beta, engaged = self.rail_beta(), self.t >= self.engage
        fast_beta, weight = (self.fast_beta, self.fast_weight) if engaged else (beta, 1.0)
        dev = self.w.device
        g = self.param_groups[0]
        if self.matrices:
            _lib.call('noise_anvil_region_prepare', ctypes.byref(self.region), flat.data_ptr(), self.fast.data_ptr(),
                      self.slow.data_ptr(), self.scratch.data_ptr(), self.x.data_ptr(), self.partials.data_ptr(),
                      self.scalars.data_ptr(), float(fast_beta), float(self.slow_beta), float(beta), float(weight),
                      _stream(dev))
            self._polar_maps()
            _lib.call('noise_anvil_region_finish', ctypes.byref(self.region), self.w.flat.data_ptr(),
                      self.w.packed.data_ptr(), self.slow.data_ptr(), self.x.data_ptr(), self.energy.data_ptr(),
                      self.partials.data_ptr(), self.scalars.data_ptr(), float(self.lane_beta), float(g['lr']),
                      float(g['weight_decay']), _stream(dev))
        self.t += 1


class Optimizers:
    """run.py:629-640: both optimizers behind one step(); param_groups concatenated for set_rate."""

    def __init__(self, *optimizers):
        self.optimizers = optimizers
        self.param_groups = [g for o in optimizers for g in o.param_groups]

    def zero_grad(self, set_to_none=True):
        pass

    def step(self, grad: DenseGrad):
        for o in self.optimizers:
            o.step(grad)


def make_optimizer(w: Weights, lr: float, betas, anvil_lr: float, anvil_wd: float, steps: int) -> Optimizers:
    """ANVIL II on block matrices, AdamW elsewhere (run.py:643-656)."""
    return Optimizers(Anvil(w, anvil_lr, anvil_wd, steps), AdamWDense(w, lr, betas, eps=1e-8, weight_decay=0.0))


def make_sharded_optimizer(w: Weights, lr: float, betas, anvil_lr: float, anvil_wd: float, steps: int, rank: int = 0,
                           world: int = 1):
    """The same split on the sharded update (noise_b200.shard): each rank owns a run of whole tensors,
    the gradient is reduce-scattered instead of all-reduced, and the parameters are all-gathered."""
    from .shard import ShardedOptimizer
    return ShardedOptimizer(w, rank, world, kind='anvil', lr=lr, betas=betas, eps=1e-8, weight_decay=0.0,
                            anvil_lr=anvil_lr, anvil_wd=anvil_wd, steps=steps)
