"""Population forward: per-member losses of rank-1 perturbed models, on the CUDA kernels.

`population_losses` is the kernel-level call behind `Eggroll` (noise_b200/eggroll.py); its
semantics are those of `population_loss` (train/val/eggroll.py:66-103) with the draws regenerated
from the counter-based stream instead of being passed in as tensors.
"""
from __future__ import annotations

import torch

from . import _lib
from .model import Weights

_WORKSPACES: dict = {}

DEFAULT_WORKSPACE_BYTES = 16 << 30


def workspace(device, nbytes: int) -> torch.Tensor:
    """A cached uint8 device buffer of at least nbytes (grown, never shrunk)."""
    key = torch.device(device)
    buf = _WORKSPACES.get(key)
    if buf is None or buf.numel() < nbytes:
        _WORKSPACES.pop(key, None)
        buf = torch.empty(nbytes, dtype=torch.uint8, device=key)
        _WORKSPACES[key] = buf
    return buf


def workspace_bytes(rows: int) -> int:
    return int(_lib.load().noise_pop_workspace_bytes(rows))


def units_that_fit(rows_per_unit: int, units: int, max_workspace: int, pairs: int = 1) -> int:
    """Members (or draws) per chunk the library will use for `units` units of rows_per_unit rows under a
    max_workspace budget: noise_pop_chunk_members, the library's own chunking (largest fitting chunk,
    capped by the draw table and 32-bit row indices, then evened out), at least 1. pairs: the
    population's antithetic directions (1 for direct draws)."""
    n = int(_lib.load().noise_pop_chunk_members(rows_per_unit, max(1, units), max(1, pairs), max_workspace))
    return max(1, n)


def population_losses(w: Weights, tokens: torch.Tensor, targets: torch.Tensor, member_begin: int, members: int,
                      pairs: int, sigma: float, seed: int, step: int, out: torch.Tensor | None = None,
                      status: torch.Tensor | None = None, max_workspace: int | None = None) -> torch.Tensor:
    """Mean CE of members [member_begin, member_begin + members) on every row of tokens/targets [B, T]."""
    if tokens.dim() == 1:
        tokens, targets = tokens[None], targets[None]
    B, T = tokens.shape
    dev = w.device
    tok = tokens.to(dev, torch.int32).contiguous()
    tgt = targets.to(dev, torch.int32).contiguous()
    if out is None:
        out = torch.empty(members, dtype=torch.float32, device=dev)
    rows_per_member = B * T
    if max_workspace is None:
        max_workspace = DEFAULT_WORKSPACE_BYTES
    per_chunk = units_that_fit(rows_per_member, members, max_workspace, pairs)
    need = workspace_bytes(rows_per_member * per_chunk)
    ws = workspace(dev, need)
    own_status = status is None
    if own_status:
        status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.call('noise_pop_forward_lowrank', w.flat.data_ptr(), w.packed.data_ptr(), w.rope(T).data_ptr(),
              tok.data_ptr(), tgt.data_ptr(), B, T, member_begin, members, pairs, float(sigma), seed & 0xFFFFFFFF,
              step & 0xFFFFFFFF, out.data_ptr(), ws.data_ptr(), need, status.data_ptr(),
              torch.cuda.current_stream(dev).cuda_stream)
    if own_status:
        code = int(status.item())
        if code:
            raise _lib.NoiseError(f'population forward: device status {_lib.STATUS_NAMES.get(code, code)}')
    return out


@torch.no_grad()
def evaluate(weights: Weights, val: torch.Tensor, batch: int = 16) -> float:
    """Mean next-token CE of the unperturbed model over validation rows [N, 2049] (utils/eval.py's
    number, computed with sigma = 0 through the population forward)."""
    total, count = 0.0, 0
    for i in range(0, len(val), batch):
        rows = val[i:i + batch].to(weights.device)
        loss = population_losses(weights, rows[:, :-1], rows[:, 1:], 0, 1, 1, 0.0, 0, 0)
        n = rows[:, 1:].numel()
        total += float(loss.item()) * n
        count += n
    return total / count

