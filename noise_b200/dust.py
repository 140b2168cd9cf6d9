"""DUST's direct-draw estimator on B200: the host-side mirror of `train/val/run.py`'s DUST pieces.

  capture                 -> noise_pop_capture (clean forward keeping block inputs, MLP hidden, logits)
  rerun(n, entry, jitter) -> noise_pop_forward_direct (orthogonal draws regenerated in-kernel)
  direct_errors           -> noise_dust_errors (centred / discounted rewards contracted with the draws)
  head_error              -> noise_coordinate_differences
  reassemble              -> noise_reassemble (errT . x on tf32 tensor cores, as the reference's einsum
                             under set_float32_matmul_precision('high'))
  CreditMemory            -> torch fp32 algebra (cuBLAS products, cuSOLVER Cholesky) at the same precision
"""
from __future__ import annotations

import contextlib
import math
import re
from dataclasses import dataclass

import torch

from . import _lib
from .model import LAYERS, TENSOR_ID, VOCAB, WIDTH, Weights
from .population import units_that_fit, workspace, workspace_bytes

HIDDEN = 4 * WIDTH
SITE_KINDS = {'transformer.wte': 0, 'o': 1, 'attn': 2, 'fc': 3, 'mlp': 4}


@contextlib.contextmanager
def reference_matmul_precision():
    """torch's fp32 products on TF32 tensor cores while the block runs, as the reference sets for its whole
    run (train/val/run.py:676: torch.set_float32_matmul_precision('high')); the caller's setting is
    restored afterwards."""
    prev = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision('high')
    try:
        yield
    finally:
        torch.set_float32_matmul_precision(prev)


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
        spec.y_entry = cap.attn_out[entry].data_ptr()  # the entry block starts from its clean attention output
    out = torch.empty(draws, cap.B, cap.T, dtype=torch.float32, device=dev)
    per = units_that_fit(rows, draws, max_workspace)
    need = workspace_bytes(rows * per)
    ws = workspace(dev, need)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.call('noise_pop_forward_direct', w.flat.data_ptr(), w.packed.data_ptr(), w.rope(cap.T).data_ptr(),
              cap.x.data_ptr(), cap.y.data_ptr(), cap.B, cap.T, draw_begin, draws, _lib.ctypes.byref(spec),
              seed & 0xFFFFFFFF, step & 0xFFFFFFFF, out.data_ptr(), ws.data_ptr(), need, status.data_ptr(),
              _stream(dev))
    if int(status.item()):
        raise _lib.NoiseError('direct rerun: device wait timed out')
    return out


def prior_struct(sites: list[Site], priors: dict | None) -> _lib.NoisePrior | None:
    """The NoisePrior of a rerun's jittered sites that carry a prior mu [B*T, d] (masked like the draws)."""
    if not priors:
        return None
    p = _lib.NoisePrior()
    for s in sites:
        if s.name in priors:
            mu = priors[s.name]
            p.site[p.count], p.d[p.count], p.mu[p.count] = s.sid, s.width, mu.data_ptr()
            p.count += 1
    return p if p.count else None


def accumulate_errors(cap: Capture, perturbed: torch.Tensor, s: Site, draw_begin: int, chunk: int, sigma: float,
                      gamma: float, seed: int, step: int, errors: torch.Tensor | None = None,
                      prior: _lib.NoisePrior | None = None) -> torch.Tensor:
    """errors [B*T, d] -= sum_i centred reward_i a_i / sigma over the draws of `perturbed` (run.py:353-373)."""
    dev = perturbed.device
    if errors is None:
        errors = torch.zeros(cap.B * cap.T, s.width, dtype=torch.float32, device=dev)
    live = cap.hidden[s.layer].data_ptr() if s.kind == 3 else None
    _lib.call('noise_dust_errors', cap.clean_loss.data_ptr(), perturbed.data_ptr(), perturbed.shape[0], chunk, cap.B,
              cap.T, draw_begin, s.sid, s.width, float(sigma), float(gamma), live,
              _lib.ctypes.byref(prior) if prior is not None else None, seed & 0xFFFFFFFF, step & 0xFFFFFFFF,
              errors.data_ptr(), _stream(dev))
    return errors


def direct_errors(w: Weights, cap: Capture, names: list[str], draws: int, sigma: float, entry=None, gamma=0.0,
                  seed: int = 0, step: int = 0, draw_offset: int = 0, nrep: int = 16,
                  priors: dict | None = None) -> dict[str, torch.Tensor]:
    """run.py:332-378: per-site output errors [B, T, d] from `draws` direct draws (global indices
    draw_offset ..), evaluated in blocks of whole chunks. priors {site: mu [B*T, d]} (alpha M c,
    masked like the site's draws) make the draws estimate the residual around mu, which is added back
    with centring's (1 - 1/n) shrinkage."""
    sites = [site(n) for n in names]
    n = chunk_size(draws, nrep)
    block = max(n, (2048 // n) * n)
    priors = {k: v.reshape(cap.B * cap.T, -1).float().contiguous() for k, v in (priors or {}).items()}
    pstruct = prior_struct(sites, priors)
    errors = {s.name: None for s in sites}
    for d0 in range(0, draws, block):
        cnt = min(block, draws - d0)
        perturbed = rerun(w, cap, sites, cnt, draw_offset + d0, sigma, entry, seed, step)
        for s in sites:
            errors[s.name] = accumulate_errors(cap, perturbed, s, draw_offset + d0, n, sigma, gamma, seed, step,
                                               errors[s.name], pstruct)
    kept = 1 - 1 / n if n > 1 else 1.0
    out = {}
    for k, v in errors.items():
        e = v / draws
        if k in priors:
            e = e + kept * priors[k]
        out[k] = e.view(cap.B, cap.T, -1)
    return out


class CreditMemory:
    """The credit memory of train/val/run.py:281-330: per direct site a ridge regression M = S (P +
    ridge)^-1 from the head's output error c at a token to the site's own output error, with S and the
    key covariance P kept as EMAs of this run's estimates, and a per-site scale alpha fitted on the
    retrievals. Dense fp32 algebra in torch (cuBLAS GEMMs, one cuSOLVER Cholesky per step)."""

    def __init__(self, beta: float = 0.9, ridge: float = 0.1, alpha_beta: float = 0.8, world: int = 1):
        self.beta, self.ridge, self.alpha_beta, self.world = beta, ridge, alpha_beta, world
        self.P = None
        self.S, self.alpha, self.calibration, self.fits, self.estimates = {}, {}, {}, {}, {}
        self._chol = None
        self._chol_of = None
        self._M = {}

    def _average(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.SUM)
            t.div_(self.world)
        return t

    def matrix(self, name: str) -> torch.Tensor | None:
        """M = S (P + ridge mean(diag P) I)^-1; one factorisation serves every site (run.py:281-292).
        P and S change only in remember(), so the first call after it solves for every site with a
        memory at once: one triangular solve whose right-hand sides are all the sites' S^T columns (each
        column is solved on its own, as in a solve per site), instead of one narrow solve per site."""
        S = self.S.get(name)
        if S is None:
            return None
        if self._chol_of is not self.P:
            lam = self.ridge * self.P.diagonal().mean()
            eye = torch.eye(len(self.P), dtype=self.P.dtype, device=self.P.device)
            self._chol = torch.linalg.cholesky(self.P + lam * eye)
            self._chol_of = self.P
            self._M = {}
        if name not in self._M:
            names = [n for n in self.S if n not in self._M]
            sol = torch.cholesky_solve(torch.cat([self.S[n].T for n in names], dim=1), self._chol)
            off = 0
            for n in names:
                d = self.S[n].shape[0]
                self._M[n] = sol[:, off:off + d].T
                off += d
        return self._M[name]

    def retrieve(self, credit: torch.Tensor, names: list[str]) -> dict:
        """{site: M c [B*T, d]} for the sites with a memory (run.py:294-302); credit is [B*T, 4096]."""
        out = {}
        for n in names:
            M = self.matrix(n)
            if M is not None:
                out[n] = credit @ M.T
        return out

    def priors(self, retrieved: dict, live: dict | None = None) -> dict:
        """alpha M c for the retrieved sites with a fitted alpha, masked by the live units (run.py:336-341)."""
        out = {}
        for n, r in retrieved.items():
            if n in self.alpha:
                mu = self.alpha[n] * r
                if live and n in live:
                    mu = mu * live[n]
                out[n] = mu
        return out

    def fit(self, name: str, retrieved: torch.Tensor, estimate: torch.Tensor, kept: float):
        """<r, estimate / kept> and |r|^2 for the next steps' alpha (run.py:375-377)."""
        target = estimate.reshape(retrieved.shape) / kept
        self.fits[name] = torch.stack([(retrieved * target).sum(), (retrieved * retrieved).sum()])

    def calibrate(self):
        """run.py:316-330: alpha = EMA<r, estimate> / EMA|r|^2 per site, fits averaged over ranks."""
        names = list(self.fits)
        if not names:
            return
        fits = self._average(torch.stack([self.fits[n] for n in names])).tolist()
        for n, (dot, ret) in zip(names, fits):
            if ret > 0:
                od, orr = self.calibration.get(n, (dot, ret))
                b = self.alpha_beta
                self.calibration[n] = b * od + (1 - b) * dot, b * orr + (1 - b) * ret
                self.alpha[n] = self.calibration[n][0] / self.calibration[n][1]
        self.fits.clear()

    def remember(self, credit: torch.Tensor, valid):
        """run.py:304-314: P = EMA(c^T c / valid), S_site = EMA(sum_t estimate_t c_t^T / valid)."""
        C = self._average(credit.T @ credit) / valid
        self.P = C * (1 - self.beta) if self.P is None else self.beta * self.P + (1 - self.beta) * C
        for n, e in self.estimates.items():
            G = self._average(e.reshape(credit.shape[0], -1).T @ credit) / valid
            S = self.S.get(n)
            self.S[n] = G * (1 - self.beta) if S is None else self.beta * S + (1 - self.beta) * G
        self.estimates.clear()


def head_error(cap: Capture, sigma: float = 0.1) -> torch.Tensor:
    """The head's output error by coordinate differences (run.py:380-389), [B, T, 4096]."""
    out = torch.empty_like(cap.logits)
    _lib.call('noise_coordinate_differences', cap.logits.data_ptr(), cap.y.data_ptr(), cap.logits.shape[0],
              float(sigma), out.data_ptr(), _stream(cap.logits.device))
    return out.view(cap.B, cap.T, VOCAB)


_CONTRACT_WS: dict = {}


def contract(err: torch.Tensor, x: torch.Tensor, normalise: bool, width: int | None = None) -> torch.Tensor:
    """g[o, i] = sum_k err[k, o] x[k, i] (noise_reassemble: tf32 tensor cores), x's rows scaled by
    1/rms first when `normalise`; `width` keeps x's first columns only (after the row norm)."""
    err = err.float().contiguous()
    x = x.contiguous()
    K, out = err.shape
    cols = width or x.shape[1]
    dev = err.device
    need = int(_lib.load().noise_reassemble_workspace_bytes(K, out, cols))
    ws = _CONTRACT_WS.get(dev)
    if ws is None or ws.numel() < need:
        ws = _CONTRACT_WS[dev] = torch.empty(need, dtype=torch.uint8, device=dev)
    g = torch.empty(out, cols, dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.call('noise_reassemble', err.data_ptr(), out, K, out, x.data_ptr(), int(x.dtype == torch.bfloat16),
              x.shape[1], cols, int(normalise), g.data_ptr(), ws.data_ptr(), ws.numel(), status.data_ptr(),
              _stream(dev))
    return g


def reassemble(cap: Capture, name: str, error: torch.Tensor) -> torch.Tensor:
    """Weight gradient from output error and the cached module input (run.py:465-471)."""
    err = error.reshape(-1, error.shape[-1]).float()
    if name == 'transformer.wte':
        g = torch.zeros(VOCAB, err.shape[1], dtype=torch.float32, device=err.device)
        return g.index_add_(0, cap.x.reshape(-1).long(), err)
    if name == 'lm_head':
        return contract(err, cap.final, True)
    s = site(name)
    if s.kind == 2:  # attn.c_proj reads the attention output (bf16)
        return contract(err, cap.attn_out[s.layer], False)
    if s.kind == 4:  # mlp.c_proj reads the relu^2 hidden (bf16)
        return contract(err, cap.hidden[s.layer], False)
    if s.kind == 3:  # mlp.c_fc reads the normalised stream after the attention
        return contract(err, cap.mid[s.layer], True)
    raise ValueError(name)


# ------------------------------------------------------------------------------------------------
# attention-internal (local) errors
# ------------------------------------------------------------------------------------------------
LOCAL_KINDS = {'q': 0, 'k': 1, 'v': 2, 'gate': 3, 've': 4}
LOCAL_SITES = {'q': 'attn.c_q', 'k': 'attn.c_k', 'v': 'attn.c_v', 'gate': 'attn.ve_gate'}
PACK_LAYER = 3 * WIDTH * WIDTH + WIDTH * WIDTH + 2 * HIDDEN * WIDTH  # packed bf16 weights per block
VE_LAYERS = (1, 3, 5, 7)


def local_layers(kind: str) -> list[int]:
    """Blocks with an estimate of `kind` (run.py:398): gates and value embeddings on VE blocks only."""
    return [i for i in range(LAYERS) if kind not in ('ve', 'gate') or i in VE_LAYERS]


def local_site(kind: str, layer: int) -> str:
    return f'value_embeds.{layer}' if kind == 've' else f'transformer.h.{layer}.{LOCAL_SITES[kind]}'


class LocalInputs:
    """Block `layer`'s clean attention inputs from the captured block input (run.py:418-425): the raw
    c_q / c_k / c_v outputs (bf16, one GEMM on the packed weights), the gate logits and value-embedding
    rows on VE blocks, the processed queries and keys and the clean values."""

    def __init__(self, w: Weights, cap: Capture, layer: int):
        dev, rows = w.device, cap.B * cap.T
        self.layer = layer
        x = cap.blocks[layer]
        self.h = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + torch.finfo(torch.float32).eps)
        hb = self.h.bfloat16().contiguous()
        qkv = torch.empty(rows, 3 * WIDTH, dtype=torch.bfloat16, device=dev)
        wq = w.packed[layer * PACK_LAYER: layer * PACK_LAYER + 3 * WIDTH * WIDTH]
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        _lib.call('noise_gemm_bf16', hb.data_ptr(), wq.data_ptr(), qkv.data_ptr(), rows, 3 * WIDTH, WIDTH, 1.0, 1,
                  status.data_ptr(), _stream(dev))
        self.raw = {n: qkv[:, i * WIDTH:(i + 1) * WIDTH].contiguous() for i, n in enumerate('qkv')}
        self.z = self.ve = None
        values = self.raw['v']
        if layer in VE_LAYERS:
            gw = w.views[f'transformer.h.{layer}.attn.ve_gate.weight']
            self.z = (hb[:, :32] @ gw.bfloat16().t()).float().contiguous()
            self.ve = w.views[f'value_embeds.{layer}.weight'][cap.x.reshape(-1).long()].contiguous()
            values = (values.float() + (2 * torch.sigmoid(self.z)).repeat_interleave(64, 1) * self.ve).bfloat16()
        self.values = values.contiguous()
        rope = w.rope(cap.T)
        self.processed = {}
        for n in 'qk':
            out = torch.empty(rows, WIDTH, dtype=torch.bfloat16, device=dev)
            _lib.call('noise_local_process', self.raw[n].data_ptr(), rope.data_ptr(), cap.B, cap.T, out.data_ptr(),
                      _stream(dev))
            self.processed[n] = out
        self.bases = {}

    def spec(self, kind: str, target: torch.Tensor, sigma: float, gamma: float) -> _lib.NoiseLocal:
        s = _lib.NoiseLocal()
        s.kind, s.layer = LOCAL_KINDS[kind], self.layer
        s.site = TENSOR_ID[local_site(kind, self.layer) + '.weight']
        s.sigma, s.gamma = sigma, gamma
        s.raw = self.raw[kind].data_ptr() if kind in ('q', 'k') else None
        s.q, s.k, s.values = self.processed['q'].data_ptr(), self.processed['k'].data_ptr(), self.values.data_ptr()
        if self.z is not None:
            s.gate_logits, s.ve = self.z.data_ptr(), self.ve.data_ptr()
        s.target = target.data_ptr()
        return s

    def input_of(self, kind: str) -> torch.Tensor:
        """The site module's cached input: the normed block input (first 32 channels for the gate)."""
        return self.h[:, :32] if kind == 'gate' else self.h


def local_errors(w: Weights, cap: Capture, kind: str, draws: int, targets: dict, seed: int, step: int,
                 draw_offset: int = 0, sigma: float = 0.1, gamma: float = 0.98, inputs: dict | None = None,
                 max_workspace: int = 4 << 30) -> dict[str, torch.Tensor]:
    """DUST.local_errors (run.py:391-463): {site: [B, T, width]} for every block with `kind`, from
    `draws` draws (global indices draw_offset ..) scored against targets[layer] ([B, T, 512])."""
    dev, B, T = w.device, cap.B, cap.T
    rows = B * T
    rope = w.rope(T)
    per = max(1, min(draws, 1024, 65535 // B,
                     max_workspace // max(1, int(_lib.load().noise_local_workspace_bytes(B, T, 1)))))
    ws = workspace(dev, int(_lib.load().noise_local_workspace_bytes(B, T, per)))
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = {}
    for layer in local_layers(kind):
        li = inputs[layer] if inputs is not None and layer in inputs else LocalInputs(w, cap, layer)
        target = targets[layer].reshape(rows, WIDTH).bfloat16().contiguous()
        spec = li.spec(kind, target, sigma, gamma)
        if kind in ('q', 'k'):
            base = torch.empty(rows, 8, dtype=torch.float32, device=dev)
            _lib.call('noise_local_baseline', _lib.ctypes.byref(spec), B, T, base.data_ptr(), status.data_ptr(),
                      _stream(dev))
            spec.base = base.data_ptr()
        width = 8 if kind == 'gate' else WIDTH
        err = torch.zeros(rows, width, dtype=torch.float32, device=dev)
        for d0 in range(0, draws, per):
            cnt = min(per, draws - d0)
            _lib.call('noise_local_errors', _lib.ctypes.byref(spec), rope.data_ptr(), B, T, draw_offset + d0, cnt,
                      seed & 0xFFFFFFFF, step & 0xFFFFFFFF, err.data_ptr(), ws.data_ptr(), ws.numel(),
                      status.data_ptr(), _stream(dev))
        if int(status.item()):
            raise _lib.NoiseError('local errors: device wait timed out')
        out[local_site(kind, layer)] = (err / draws).view(B, T, width)
        del target
    return out


def reassemble_local(w: Weights, cap: Capture, kind: str, layer: int, error: torch.Tensor,
                     inputs: LocalInputs | None = None) -> torch.Tensor:
    """Weight gradient of a local site (run.py:465-471): value embeddings by token id, else err^T x."""
    err = error.reshape(-1, error.shape[-1]).float()
    if kind == 've':
        g = torch.zeros(VOCAB, WIDTH, dtype=torch.float32, device=err.device)
        return g.index_add_(0, cap.x.reshape(-1).long(), err)
    # the site's input is the normalised block input (its first 32 channels for the gate)
    return contract(err, cap.blocks[layer], True, 32 if kind == 'gate' else None)


# ------------------------------------------------------------------------------------------------
# the estimator
# ------------------------------------------------------------------------------------------------
@dataclass
class Recipe:
    """Draws per update summed over GPUs, lists per block (run.py:41-59)."""
    writers: list
    hidden: list
    hubs: list
    embedding: int
    local: dict
    nrep: int
    lr: float
    betas: tuple = (0.7, 0.95)
    warmdown: float = 0.0
    gamma: float = 0.98
    first_gamma: float = 0.3
    anvil_lr: float = 0.023
    anvil_wd: float = 2.25
    memory_beta: float = 0.9
    mesa_ridge: float = 0.1
    alpha_beta: float = 0.8


def recipe(scale: float) -> Recipe:
    """The tuned 16k Adam cell with every draw count scaled, rounded to multiples of 64 (run.py:62-70)."""
    count = lambda k: max(64, round(k * scale / 64) * 64)  # noqa: E731
    return Recipe(writers=[count(256)] * LAYERS, hidden=[count(512)] * LAYERS, hubs=[count(512)] * LAYERS,
                  embedding=count(2048),
                  local=dict(q=count(384), v=count(384), gate=count(128), k=count(1664), ve=count(4608)),
                  nrep=16, lr=0.003, warmdown=0.3)


def token_losses(w: Weights, cap: Capture) -> torch.Tensor:
    """Per-token losses [B, T] of the current (unperturbed) weights: a plain forward from the embedding."""
    spec = _lib.NoiseDirect()
    spec.entry, spec.mask, spec.sigma = -1, 0, 0.0
    dev = w.device
    out = torch.empty(cap.B, cap.T, dtype=torch.float32, device=dev)
    ws = workspace(dev, workspace_bytes(cap.B * cap.T))
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.call('noise_pop_forward_direct', w.flat.data_ptr(), w.packed.data_ptr(), w.rope(cap.T).data_ptr(),
              cap.x.data_ptr(), cap.y.data_ptr(), cap.B, cap.T, 0, 1, _lib.ctypes.byref(spec), 0, 0,
              out.data_ptr(), ws.data_ptr(), ws.numel(), status.data_ptr(), _stream(dev))
    return out


class DUST:
    """Forward-only gradient estimator of train/val/run.py:162-542 on noise_b200's kernels.

    Every phase of the reference's step: capture, the coordinate head (head_error, the memory's
    key), direct errors of the writers, the MLP hidden layer, the embedding and the attention-output
    hubs (the first block with reward-to-go) with the credit memory's priors, the attention-internal
    local errors scored against the rank-averaged hubs, reassembly, two-sided ES on the mixing
    scalars, calibration, the rank average with its finite check, the memory write, and the
    ANVIL II + AdamW step."""

    def __init__(self, w: Weights, rec: Recipe, seed: int = 0, rank: int = 0, world: int = 1):
        counts = rec.writers + rec.hidden + rec.hubs + [rec.embedding] + list(rec.local.values())
        if any(k % world for k in counts) or 8 % world:
            raise ValueError('Every draw count must split evenly across the GPUs.')
        self.w, self.recipe, self.seed, self.rank, self.world = w, rec, seed, rank, world
        self.t = 0
        self.cap = None
        self.memory = CreditMemory(rec.memory_beta, rec.mesa_ridge, rec.alpha_beta, world)

    def _errors(self, names, count, sigma, entry=None, gamma=0.0):
        """direct_errors with the memory's retrievals (run.py:332-378); records fits and estimates."""
        per = count // self.world
        retrieved = self.memory.retrieve(self.credit, names)
        live = {n: (self.cap.hidden[entry] > 0).float() for n in names if n.endswith('mlp.c_fc')}
        errs = direct_errors(self.w, self.cap, names, per, sigma, entry, gamma, self.seed, self.t,
                             draw_offset=self.rank * per, nrep=self.recipe.nrep,
                             priors=self.memory.priors(retrieved, live))
        n = chunk_size(per, self.recipe.nrep)
        kept = 1 - 1 / n if n > 1 else 1.0
        for name, r in retrieved.items():
            self.memory.fit(name, r, errs[name], kept)
        self.memory.estimates.update(errs)
        return errs

    def scalar_gradients(self, draws: int, sigma: float = 0.03) -> dict:
        """Two-sided ES for the 16 mixing scalars (run.py:473-491). The Gaussian directions come from
        a CPU generator seeded by (seed, step, rank), so every rank draws its own."""
        dev = self.w.device
        lam = self.w.flat[:2 * LAYERS]  # resid_lambdas | x0_lambdas, contiguous at the front
        clean = lam.clone()
        estimate = torch.zeros(2 * LAYERS, dtype=torch.float32, device=dev)
        valid = (self.cap.y >= 0).float()
        g = torch.Generator().manual_seed((self.seed * 1_000_003 + self.t) * 8 + self.rank)
        try:
            for _ in range(draws):
                a = torch.randn(2 * LAYERS, generator=g).to(dev)
                losses = []
                for sign in (1.0, -1.0):
                    lam.copy_(clean + sign * sigma * a)
                    losses.append(token_losses(self.w, self.cap))
                diff = ((losses[0] - losses[1]) * valid).sum() / (2 * sigma)
                estimate += diff * a / draws
        finally:
            lam.copy_(clean)
        return {'resid_lambdas': estimate[:LAYERS], 'x0_lambdas': estimate[LAYERS:]}

    def _average(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.SUM)
            t.div_(self.world)
        return t

    @torch.no_grad()
    def step(self, x, y, optimizer) -> float:
        """One update (run.py:493-542) under the reference's matmul precision: the credit memory's fp32
        products run as TF32, as in the reference's run."""
        with reference_matmul_precision():
            return self._step(x, y, optimizer)

    def _step(self, x, y, optimizer) -> float:
        from .optim import DenseGrad
        self.t += 1
        r, layers = self.recipe, LAYERS
        self.cap = cap = Capture(self.w, x, y)
        grads = DenseGrad(self.w)
        head = head_error(cap)  # the memory's key at each token
        self.credit = head.view(-1, VOCAB)
        grads.views['lm_head.weight'].copy_(reassemble(cap, 'lm_head', head))
        for layer in range(layers):
            pre = f'transformer.h.{layer}.'
            gamma = r.first_gamma if layer == 0 else 0.0
            for names, count in (([pre + 'attn.c_proj', pre + 'mlp.c_proj'], r.writers[layer]),
                                 ([pre + 'mlp.c_fc'], r.hidden[layer])):
                for name, err in self._errors(names, count, 0.4, layer, gamma).items():
                    grads.views[name + '.weight'].copy_(reassemble(cap, name, err))
        err = self._errors(['transformer.wte'], r.embedding, 0.8)['transformer.wte']
        grads.views['transformer.wte.weight'].copy_(reassemble(cap, 'transformer.wte', err))
        self.targets = {}
        for layer in range(layers):
            sigma = 0.4 if layer < layers // 2 else 0.8
            gamma = r.first_gamma if layer == 0 else 0.0
            self.targets[layer] = self._average(self._errors([f'o@{layer}'], r.hubs[layer], sigma, layer, gamma)[f'o@{layer}'])
        inputs = {layer: LocalInputs(self.w, cap, layer) for layer in range(layers)}
        for kind, count in r.local.items():
            per = count // self.world
            errs = local_errors(self.w, cap, kind, per, self.targets, self.seed, self.t, draw_offset=self.rank * per,
                                inputs=inputs)
            for (name, err), layer in zip(errs.items(), local_layers(kind)):
                grads.views[name + '.weight'].copy_(reassemble_local(self.w, cap, kind, layer, err, inputs[layer]))
        del inputs
        for name, est in self.scalar_gradients(8 // self.world).items():
            grads.views[name].copy_(est)
        self.memory.calibrate()  # the next step's alpha
        valid = (cap.y >= 0).sum().float()
        grads.flat.div_(valid)
        if hasattr(optimizer, 'step_dense'):
            # sharded update: the ranks' shares are reduce-scattered, not all-reduced
            if not optimizer.step_dense(grads.flat, 1.0 / self.world):
                raise FloatingPointError('Non-finite estimate')
            self.memory.remember(self.credit, valid)
            return cap.clean_loss.view(cap.B, cap.T)[cap.y >= 0].mean().item()
        self._average(grads.flat)
        if not torch.isfinite(grads.flat).all():
            raise FloatingPointError('Non-finite estimate')
        self.memory.remember(self.credit, valid)  # after this step's estimates
        optimizer.step(grads)
        return cap.clean_loss.view(cap.B, cap.T)[cap.y >= 0].mean().item()
