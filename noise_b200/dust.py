"""DUST's direct-draw estimator on B200: the host-side mirror of `train/val/run.py`'s DUST pieces.

  capture                 -> noise_pop_capture (clean forward keeping block inputs, MLP hidden, logits)
  rerun(n, entry, jitter) -> noise_pop_forward_direct (orthogonal draws regenerated in-kernel)
  direct_errors           -> noise_dust_errors (centred / discounted rewards contracted with the draws)
  head_error              -> noise_coordinate_differences
  reassemble              -> one fp32 GEMM (torch.matmul, cuBLAS) per site, as the reference's einsum
"""
from __future__ import annotations

import math
import re
from dataclasses import dataclass

import torch

from . import _lib
from .model import LAYERS, TENSOR_ID, VOCAB, WIDTH, Weights
from .population import workspace, workspace_bytes

HIDDEN = 4 * WIDTH
SITE_KINDS = {'transformer.wte': 0, 'o': 1, 'attn': 2, 'fc': 3, 'mlp': 4}


@dataclass
class Site:
    name: str
    kind: int       # bit of NoiseDirect.mask
    width: int      # d
    sid: int        # stream id of the site's draws
    layer: int | None


def site(name: str) -> Site:
    """The jitter site behind one of the reference's site names (run.py:97-98, :182-183)."""
    if name == 'transformer.wte':
        return Site(name, 0, WIDTH, 2, None)
    m = re.fullmatch(r'o@(\d+)', name)
    if m:
        return Site(name, 1, WIDTH, 64 + int(m.group(1)), int(m.group(1)))
    m = re.fullmatch(r'transformer\.h\.(\d+)\.(attn\.c_proj|mlp\.c_fc|mlp\.c_proj)', name)
    if not m:
        raise ValueError(f'not a direct-draw site: {name}')
    layer, mod = int(m.group(1)), m.group(2)
    kind = {'attn.c_proj': 2, 'mlp.c_fc': 3, 'mlp.c_proj': 4}[mod]
    return Site(name, kind, HIDDEN if kind == 3 else WIDTH, TENSOR_ID[name + '.weight'], layer)


def chunk_size(draws: int, cap: int) -> int:
    """Largest divisor of draws up to cap (run.py:76-78)."""
    return next(n for n in range(min(cap, draws), 0, -1) if draws % n == 0)


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


class Capture:
    """The clean forward's intermediates for a [B, T] batch (run.py:244-254)."""

    def __init__(self, w: Weights, x: torch.Tensor, y: torch.Tensor):
        dev = w.device
        self.B, self.T = x.shape
        rows = self.B * self.T
        f32 = dict(dtype=torch.float32, device=dev)
        self.x = x.to(dev, torch.int32).contiguous()
        self.y = y.to(dev, torch.int32).contiguous()
        self.blocks = torch.empty(LAYERS, rows, WIDTH, **f32)
        self.x0 = torch.empty(rows, WIDTH, **f32)
        self.inv0 = torch.empty(rows, **f32)
        self.attn_out = torch.empty(LAYERS, rows, WIDTH, dtype=torch.bfloat16, device=dev)
        self.mid = torch.empty(LAYERS, rows, WIDTH, **f32)
        self.hidden = torch.empty(LAYERS, rows, HIDDEN, dtype=torch.bfloat16, device=dev)
        self.final = torch.empty(rows, WIDTH, **f32)
        self.logits = torch.empty(rows, VOCAB, **f32)
        self.clean_loss = torch.empty(rows, **f32)
        cap = _lib.NoiseCapture(*(t.data_ptr() for t in (self.blocks, self.x0, self.inv0, self.attn_out, self.mid,
                                                           self.hidden, self.final, self.logits, self.clean_loss)))
        ws = workspace(dev, workspace_bytes(rows))
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        _lib.call('noise_pop_capture', w.flat.data_ptr(), w.packed.data_ptr(), w.rope(self.T).data_ptr(),
                  self.x.data_ptr(), self.y.data_ptr(), self.B, self.T, _lib.ctypes.byref(cap), ws.data_ptr(),
                  ws.numel(), status.data_ptr(), _stream(dev))
        if int(status.item()):
            raise _lib.NoiseError('capture: device wait timed out')

    def module_input(self, s: Site) -> torch.Tensor:
        """The cached input of the module whose output is jittered (run.py:199, reassemble :467)."""
        if s.kind == 2:
            return self.attn_out[s.layer].float()
        if s.kind == 4:
            return self.hidden[s.layer].float()
        if s.kind == 3:
            m = self.mid[s.layer]
            return m * torch.rsqrt(m.pow(2).mean(-1, keepdim=True) + torch.finfo(torch.float32).eps)
        raise ValueError(s.name)


def rerun(w: Weights, cap: Capture, sites: list[Site], draws: int, draw_begin: int, sigma: float, entry,
          seed: int, step: int, max_workspace: int = 16 << 30) -> torch.Tensor:
    """Per-token losses [draws, B, T] of draws rerun from block `entry` (None: the embedding)."""
    dev = w.device
    rows = cap.B * cap.T
    spec = _lib.NoiseDirect()
    spec.entry = -1 if entry is None else entry
    spec.mask = 0
    for s in sites:
        spec.mask |= 1 << s.kind
        spec.site[s.kind] = s.sid
    spec.sigma = sigma
    if entry is not None:
        spec.x_entry = cap.blocks[entry].data_ptr()
        spec.inv0 = cap.inv0.data_ptr()
        spec.live = cap.hidden[entry].data_ptr()
    out = torch.empty(draws, cap.B, cap.T, dtype=torch.float32, device=dev)
    per = max(1, min(draws, max_workspace // max(1, workspace_bytes(rows))))
    ws = workspace(dev, workspace_bytes(rows * per))
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.call('noise_pop_forward_direct', w.flat.data_ptr(), w.packed.data_ptr(), w.rope(cap.T).data_ptr(),
              cap.x.data_ptr(), cap.y.data_ptr(), cap.B, cap.T, draw_begin, draws, _lib.ctypes.byref(spec),
              seed & 0xFFFFFFFF, step & 0xFFFFFFFF, out.data_ptr(), ws.data_ptr(), ws.numel(), status.data_ptr(),
              _stream(dev))
    if int(status.item()):
        raise _lib.NoiseError('direct rerun: device wait timed out')
    return out


def accumulate_errors(cap: Capture, perturbed: torch.Tensor, s: Site, draw_begin: int, chunk: int, sigma: float,
                      gamma: float, seed: int, step: int, errors: torch.Tensor | None = None) -> torch.Tensor:
    """errors [B*T, d] -= sum_i centred reward_i a_i / sigma over the draws of `perturbed` (run.py:353-368)."""
    dev = perturbed.device
    if errors is None:
        errors = torch.zeros(cap.B * cap.T, s.width, dtype=torch.float32, device=dev)
    live = cap.hidden[s.layer].data_ptr() if s.kind == 3 else None
    _lib.call('noise_dust_errors', cap.clean_loss.data_ptr(), perturbed.data_ptr(), perturbed.shape[0], chunk, cap.B,
              cap.T, draw_begin, s.sid, s.width, float(sigma), float(gamma), live, seed & 0xFFFFFFFF,
              step & 0xFFFFFFFF, errors.data_ptr(), _stream(dev))
    return errors


def direct_errors(w: Weights, cap: Capture, names: list[str], draws: int, sigma: float, entry=None, gamma=0.0,
                  seed: int = 0, step: int = 0, draw_offset: int = 0, nrep: int = 16) -> dict[str, torch.Tensor]:
    """run.py:332-378 without the memory prior: per-site output errors [B, T, d] from `draws` direct
    draws (global indices draw_offset ..), evaluated in blocks of whole chunks."""
    sites = [site(n) for n in names]
    n = chunk_size(draws, nrep)
    block = max(n, (2048 // n) * n)
    errors = {s.name: None for s in sites}
    for d0 in range(0, draws, block):
        cnt = min(block, draws - d0)
        perturbed = rerun(w, cap, sites, cnt, draw_offset + d0, sigma, entry, seed, step)
        for s in sites:
            errors[s.name] = accumulate_errors(cap, perturbed, s, draw_offset + d0, n, sigma, gamma, seed, step,
                                               errors[s.name])
    return {k: (v / draws).view(cap.B, cap.T, -1) for k, v in errors.items()}


def head_error(cap: Capture, sigma: float = 0.1) -> torch.Tensor:
    """The head's output error by coordinate differences (run.py:380-389), [B, T, 4096]."""
    out = torch.empty_like(cap.logits)
    _lib.call('noise_coordinate_differences', cap.logits.data_ptr(), cap.y.data_ptr(), cap.logits.shape[0],
              float(sigma), out.data_ptr(), _stream(cap.logits.device))
    return out.view(cap.B, cap.T, VOCAB)


def reassemble(cap: Capture, name: str, error: torch.Tensor) -> torch.Tensor:
    """Weight gradient from output error and the cached module input (run.py:465-471)."""
    err = error.reshape(-1, error.shape[-1]).float()
    if name == 'transformer.wte':
        g = torch.zeros(VOCAB, err.shape[1], dtype=torch.float32, device=err.device)
        return g.index_add_(0, cap.x.reshape(-1).long(), err)
    if name == 'lm_head':
        fin = cap.final
        inp = fin * torch.rsqrt(fin.pow(2).mean(-1, keepdim=True) + torch.finfo(torch.float32).eps)
    else:
        inp = cap.module_input(site(name))
    return err.t() @ inp
