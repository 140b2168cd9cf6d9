"""The fixed 37.7M-parameter transformer and its perturbed population forward, restated on CPU
(test infrastructure; see oracle/__init__.py).

Follows `utils/model.py` (GPT, norm, apply_rotary_emb, window attention, soft-capped CE) and
`train/val/eggroll.py` (make_model, lowrank, lowrank_embed, population_loss). Everything runs in the
dtype of the parameters handed in (float32 or float64) with no bf16 rounding: it is the function the
CUDA path approximates with bf16 operands and fp32 accumulation.
"""
from __future__ import annotations

import math

import torch
from torch.nn import functional as F

SEQ, VOCAB, LAYERS, HEADS, WIDTH, HEAD_DIM = 2048, 4096, 8, 8, 512, 64
GATE_CHANNELS = 32
VE_LAYERS = (1, 3, 5, 7)                       # utils/model.py:50-52 (has_ve)
WINDOWS = (1024, 1024, 1024, 2048, 1024, 1024, 1024, 2048)  # utils/model.py:185-191, pattern SSSL
SOFTCAP = 15.0                                 # utils/model.py:204
ROPE_BASE = 10000.0                            # utils/model.py:177


def param_specs():
    """(name, shape) in `GPT.named_parameters()` order; the index is the draw stream's tensor id."""
    specs = [('resid_lambdas', (LAYERS,)), ('x0_lambdas', (LAYERS,)),
             ('transformer.wte.weight', (VOCAB, WIDTH))]
    for i in range(LAYERS):
        pre = f'transformer.h.{i}.'
        specs += [(pre + 'attn.c_q.weight', (WIDTH, WIDTH)), (pre + 'attn.c_k.weight', (WIDTH, WIDTH)),
                  (pre + 'attn.c_v.weight', (WIDTH, WIDTH)), (pre + 'attn.c_proj.weight', (WIDTH, WIDTH))]
        if i in VE_LAYERS:
            specs.append((pre + 'attn.ve_gate.weight', (HEADS, GATE_CHANNELS)))
        specs += [(pre + 'mlp.c_fc.weight', (4 * WIDTH, WIDTH)), (pre + 'mlp.c_proj.weight', (WIDTH, 4 * WIDTH))]
    specs.append(('lm_head.weight', (VOCAB, WIDTH)))
    specs += [(f'value_embeds.{i}.weight', (VOCAB, WIDTH)) for i in VE_LAYERS]
    return specs


PARAM_SPECS = param_specs()
TENSOR_ID = {name: i for i, (name, _) in enumerate(PARAM_SPECS)}
N_PARAMS = sum(math.prod(s) for _, s in PARAM_SPECS)  # 37,749,776


def make_params(seed: int = 0, dust: bool = False) -> dict[str, torch.Tensor]:
    """The seed-0 initialisation on CPU, float32.

    Restates the RNG call sequence of `utils/model.py:149-175` (init_weights) followed by the c_proj
    re-initialisation of `train/val/eggroll.py:38-53` (identical in `train/val/run.py:545-557`), so
    the torch CPU generator yields the reference's exact values.
    """
    g = torch.manual_seed(seed)
    del g
    p = {name: torch.empty(shape) for name, shape in PARAM_SPECS}
    s = 3 ** 0.5 * WIDTH ** -0.5
    torch.nn.init.normal_(p['transformer.wte.weight'], mean=0.0, std=1.0)
    torch.nn.init.normal_(p['lm_head.weight'], mean=0.0, std=0.001)
    for i in range(LAYERS):
        pre = f'transformer.h.{i}.'
        torch.nn.init.uniform_(p[pre + 'attn.c_q.weight'], -s, s)
        torch.nn.init.uniform_(p[pre + 'attn.c_k.weight'], -s, s)
        torch.nn.init.uniform_(p[pre + 'attn.c_v.weight'], -s, s)
        torch.nn.init.zeros_(p[pre + 'attn.c_proj.weight'])
        torch.nn.init.uniform_(p[pre + 'mlp.c_fc.weight'], -s, s)
        torch.nn.init.zeros_(p[pre + 'mlp.c_proj.weight'])
    p['resid_lambdas'].fill_(1.0)
    p['x0_lambdas'].fill_(0.1)
    for i in VE_LAYERS:
        torch.nn.init.uniform_(p[f'value_embeds.{i}.weight'], -s, s)
    for i in VE_LAYERS:
        torch.nn.init.zeros_(p[f'transformer.h.{i}.attn.ve_gate.weight'])
    # named_modules order: per block attn.c_proj then mlp.c_proj
    for i in range(LAYERS):
        for name in (f'transformer.h.{i}.attn.c_proj.weight', f'transformer.h.{i}.mlp.c_proj.weight'):
            scale = 1.5 * (3 / p[name].shape[1]) ** 0.5
            torch.nn.init.uniform_(p[name], -scale, scale)
    return p


def rotary_tables(length: int) -> tuple[torch.Tensor, torch.Tensor]:
    """cos, sin [length, 32] rounded to bf16 then widened (utils/model.py:177-183)."""
    inv_freq = 1.0 / ROPE_BASE ** (torch.arange(0, HEAD_DIM, 2, dtype=torch.float32) / HEAD_DIM)
    t = torch.arange(length, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return freqs.cos().bfloat16().float(), freqs.sin().bfloat16().float()


def rms_norm(x: torch.Tensor) -> torch.Tensor:
    """Parameter-free RMSNorm with the float32 epsilon (utils/model.py:46-47, F.rms_norm default)."""
    eps = torch.finfo(torch.float32).eps
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [..., T, H, 64]; rotates (x1, x2) halves (utils/model.py:55-58)."""
    d = x.shape[-1] // 2
    x1, x2 = x[..., :d], x[..., d:]
    c, s = cos[:, None, :].to(x.dtype), sin[:, None, :].to(x.dtype)
    return torch.cat([x1 * c + x2 * s, x1 * -s + x2 * c], -1)


def window_attention(q, k, v, window: int, block: int = 256) -> torch.Tensor:
    """Causal attention where query s sees keys s-window..s (utils/model.py:17-31), scale 1/sqrt(64).
    q, k, v [N, T, H, 64]; computed in query blocks so no [T, T] score matrix is held."""
    n, t, h, d = q.shape
    out = torch.empty_like(q)
    scale = d ** -0.5
    for q0 in range(0, t, block):
        q1 = min(t, q0 + block)
        k0 = max(0, q0 - window)
        qs = q[:, q0:q1].transpose(1, 2)            # [N, H, bq, d]
        ks = k[:, k0:q1].transpose(1, 2)
        vs = v[:, k0:q1].transpose(1, 2)
        s = (qs @ ks.transpose(-1, -2)) * scale     # [N, H, bq, bk]
        qi = torch.arange(q0, q1)[:, None]
        ki = torch.arange(k0, q1)[None, :]
        mask = (qi >= ki) & (qi - ki <= window)
        s = s.masked_fill(~mask, float('-inf'))
        out[:, q0:q1] = (torch.softmax(s, -1) @ vs).transpose(1, 2)
    return out


def soft_cap(logits: torch.Tensor) -> torch.Tensor:
    return SOFTCAP * torch.tanh(logits / SOFTCAP)


def forward(p: dict, idx: torch.Tensor, targets: torch.Tensor | None = None, reduction: str = 'mean'):
    """GPT.forward (utils/model.py:193-209) for idx [B, T]: mean / per-token CE, or logits."""
    b, t = idx.shape
    cos, sin = rotary_tables(t)
    x = x0 = rms_norm(p['transformer.wte.weight'][idx])
    for i in range(LAYERS):
        pre = f'transformer.h.{i}.'
        x = p['resid_lambdas'][i] * x + p['x0_lambdas'][i] * x0
        h = rms_norm(x)
        q = (h @ p[pre + 'attn.c_q.weight'].t()).view(b, t, HEADS, HEAD_DIM)
        k = (h @ p[pre + 'attn.c_k.weight'].t()).view(b, t, HEADS, HEAD_DIM)
        v = (h @ p[pre + 'attn.c_v.weight'].t()).view(b, t, HEADS, HEAD_DIM)
        if i in VE_LAYERS:
            ve = p[f'value_embeds.{i}.weight'][idx].view(b, t, HEADS, HEAD_DIM)
            gate = 2 * torch.sigmoid(h[..., :GATE_CHANNELS] @ p[pre + 'attn.ve_gate.weight'].t())
            v = v + gate.unsqueeze(-1) * ve
        q, k = rms_norm(rope(q, cos, sin)), rms_norm(rope(k, cos, sin))
        y = window_attention(q, k, v, WINDOWS[i]).reshape(b, t, WIDTH)
        x = x + y @ p[pre + 'attn.c_proj.weight'].t()
        x = x + F.relu(rms_norm(x) @ p[pre + 'mlp.c_fc.weight'].t()).square() @ p[pre + 'mlp.c_proj.weight'].t()
    logits = soft_cap(rms_norm(x) @ p['lm_head.weight'].t())
    if targets is None:
        return logits
    return F.cross_entropy(logits.reshape(-1, VOCAB), targets.reshape(-1), ignore_index=-1, reduction=reduction)


def _lowrank(x, w, a, b, sign):
    """x [m, ..., in] through W + sign * a b^T per member (train/val/eggroll.py:56-58)."""
    shape = (-1,) + (1,) * (x.dim() - 2)
    xb = (x * b.view(b.shape[0], *([1] * (x.dim() - 2)), b.shape[1])).sum(-1, keepdim=True)
    return x @ w.t() + sign.view(shape + (1,)) * xb * a.view(a.shape[0], *([1] * (x.dim() - 2)), a.shape[1])


def _lowrank_embed(w, a, b, idx, sign):
    """Rows idx [B, T] of W [V, d] + sign * a b^T per member (train/val/eggroll.py:61-63) -> [m, B, T, d]."""
    return w[idx][None] + sign.view(-1, 1, 1, 1) * a[:, idx].unsqueeze(-1) * b[:, None, None, :]


def population_token_losses(p: dict, draws: dict, sign: torch.Tensor, idx: torch.Tensor,
                            targets: torch.Tensor) -> torch.Tensor:
    """Per-token CE [m, B, T] of m perturbed models, each on every row of idx/targets [B, T].

    Restates `population_loss` (train/val/eggroll.py:66-103): every 2-D parameter W is replaced by
    W + sign_m a_m b_m^T (draws[name] = (a [m, rows], b [m, cols])) and each mixing scalar vector by
    lambda + sign_m eps_m (draws[name] = eps [m, 8]). With B = 1 and one sequence this is exactly the
    reference function before its per-member mean."""
    m = sign.shape[0]
    bsz, t = idx.shape
    cos, sin = rotary_tables(t)
    s = sign.view(m, 1, 1, 1)
    emb = _lowrank_embed(p['transformer.wte.weight'], *draws['transformer.wte.weight'], idx, sign)
    x = x0 = rms_norm(emb)                                            # [m, B, T, d]
    for i in range(LAYERS):
        pre = f'transformer.h.{i}.'
        resid = p['resid_lambdas'][i] + s * draws['resid_lambdas'][:, i].view(m, 1, 1, 1)
        mix = p['x0_lambdas'][i] + s * draws['x0_lambdas'][:, i].view(m, 1, 1, 1)
        x = resid * x + mix * x0

        def lin(name, inp):
            return _lowrank(inp, p[pre + name], *draws[pre + name], sign)

        h = rms_norm(x)
        q = lin('attn.c_q.weight', h).view(m * bsz, t, HEADS, HEAD_DIM)
        k = lin('attn.c_k.weight', h).view(m * bsz, t, HEADS, HEAD_DIM)
        v = lin('attn.c_v.weight', h).view(m * bsz, t, HEADS, HEAD_DIM)
        if i in VE_LAYERS:
            name = f'value_embeds.{i}.weight'
            ve = _lowrank_embed(p[name], *draws[name], idx, sign).view(m * bsz, t, HEADS, HEAD_DIM)
            gate = 2 * torch.sigmoid(lin('attn.ve_gate.weight', h[..., :GATE_CHANNELS]))
            v = v + gate.view(m * bsz, t, HEADS, 1) * ve
        q, k = rms_norm(rope(q, cos, sin)), rms_norm(rope(k, cos, sin))
        y = window_attention(q, k, v, WINDOWS[i]).reshape(m, bsz, t, WIDTH)
        x = x + lin('attn.c_proj.weight', y)
        x = x + lin('mlp.c_proj.weight', F.relu(lin('mlp.c_fc.weight', rms_norm(x))).square())
    h = rms_norm(x)
    a, b = draws['lm_head.weight']
    out = torch.empty(m, bsz, t, dtype=h.dtype)
    for c in range(m):  # one member's logits at a time
        logits = soft_cap(_lowrank(h[c:c + 1], p['lm_head.weight'], a[c:c + 1], b[c:c + 1], sign[c:c + 1]))[0]
        out[c] = F.cross_entropy(logits.reshape(-1, VOCAB), targets.reshape(-1), reduction='none').view(bsz, t)
    return out


def population_losses(p, draws, sign, idx, targets) -> torch.Tensor:
    """Per-member mean CE [m] over all B x T tokens."""
    return population_token_losses(p, draws, sign, idx, targets).mean(dim=(1, 2))
