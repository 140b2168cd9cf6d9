"""Device-resident parameters of the fixed model in the reference's state-dict layout.

`Weights` holds one flat fp32 master buffer in `GPT.named_parameters()` order (utils/model.py:123-147)
with named views (the `final.pt` layout: 37,749,776 parameters), the packed bf16 copy the GEMMs
read, and the rotary table. Initialisation restates the reference's seed-0 RNG call sequence
(`utils/model.py:149-175`, then the c_proj re-initialisation of `train/val/eggroll.py:38-53` /
`train/val/run.py:545-557`) on the CPU generator, so weights equal the reference's CPU init exactly.
"""
from __future__ import annotations

import math

import torch

from . import _lib

SEQ, VOCAB, LAYERS, HEADS, WIDTH, HEAD_DIM, GATE = 2048, 4096, 8, 8, 512, 64, 32
VE_LAYERS = (1, 3, 5, 7)


def _specs():
    specs = [('resid_lambdas', (LAYERS,)), ('x0_lambdas', (LAYERS,)), ('transformer.wte.weight', (VOCAB, WIDTH))]
    for i in range(LAYERS):
        pre = f'transformer.h.{i}.'
        specs += [(pre + f'attn.c_{n}.weight', (WIDTH, WIDTH)) for n in ('q', 'k', 'v', 'proj')]
        if i in VE_LAYERS:
            specs.append((pre + 'attn.ve_gate.weight', (HEADS, GATE)))
        specs += [(pre + 'mlp.c_fc.weight', (4 * WIDTH, WIDTH)), (pre + 'mlp.c_proj.weight', (WIDTH, 4 * WIDTH))]
    specs.append(('lm_head.weight', (VOCAB, WIDTH)))
    specs += [(f'value_embeds.{i}.weight', (VOCAB, WIDTH)) for i in VE_LAYERS]
    return specs


PARAM_SPECS = _specs()
TENSOR_ID = {n: i for i, (n, _) in enumerate(PARAM_SPECS)}
N_PARAMS = sum(math.prod(s) for _, s in PARAM_SPECS)


def init_state(seed: int = 0) -> dict[str, torch.Tensor]:
    """The reference's seed-0 initialisation as CPU fp32 tensors."""
    torch.manual_seed(seed)
    p = {n: torch.empty(s) for n, s in PARAM_SPECS}
    s = 3 ** 0.5 * WIDTH ** -0.5
    torch.nn.init.normal_(p['transformer.wte.weight'], mean=0.0, std=1.0)
    torch.nn.init.normal_(p['lm_head.weight'], mean=0.0, std=0.001)
    for i in range(LAYERS):
        pre = f'transformer.h.{i}.'
        for n in ('attn.c_q', 'attn.c_k', 'attn.c_v'):
            torch.nn.init.uniform_(p[pre + n + '.weight'], -s, s)
        torch.nn.init.zeros_(p[pre + 'attn.c_proj.weight'])
        torch.nn.init.uniform_(p[pre + 'mlp.c_fc.weight'], -s, s)
        torch.nn.init.zeros_(p[pre + 'mlp.c_proj.weight'])
    p['resid_lambdas'].fill_(1.0)
    p['x0_lambdas'].fill_(0.1)
    for i in VE_LAYERS:
        torch.nn.init.uniform_(p[f'value_embeds.{i}.weight'], -s, s)
    for i in VE_LAYERS:
        torch.nn.init.zeros_(p[f'transformer.h.{i}.attn.ve_gate.weight'])
    for i in range(LAYERS):
        for n in (f'transformer.h.{i}.attn.c_proj.weight', f'transformer.h.{i}.mlp.c_proj.weight'):
            scale = 1.5 * (3 / p[n].shape[1]) ** 0.5
            torch.nn.init.uniform_(p[n], -scale, scale)
    return p


def rope_table(length: int) -> torch.Tensor:
    """[length, 64] fp32: cos | sin of the reference's bf16 rotary tables (utils/model.py:177-183)."""
    inv_freq = 1.0 / 10000.0 ** (torch.arange(0, HEAD_DIM, 2, dtype=torch.float32) / HEAD_DIM)
    freqs = torch.outer(torch.arange(length, dtype=torch.float32), inv_freq)
    return torch.cat([freqs.cos().bfloat16().float(), freqs.sin().bfloat16().float()], 1).contiguous()


class Weights:
    """Master fp32 parameters, packed bf16 GEMM weights and rotary tables on one CUDA device."""

    def __init__(self, device, state: dict[str, torch.Tensor] | None = None, seed: int = 0):
        lib = _lib.load()
        self.device = torch.device(device)
        assert lib.noise_param_count() == N_PARAMS
        self.flat = torch.empty(N_PARAMS, dtype=torch.float32, device=self.device)
        self.views, off = {}, 0
        for n, s in PARAM_SPECS:
            k = math.prod(s)
            self.views[n] = self.flat[off:off + k].view(s)
            off += k
        state = state if state is not None else init_state(seed)
        for n, _ in PARAM_SPECS:
            self.views[n].copy_(state[n].to(torch.float32))
        self.packed = torch.empty(lib.noise_packed_count(), dtype=torch.bfloat16, device=self.device)
        self._rope = {}
        self.pack()

    def pack(self):
        _lib.call('noise_pack_weights', self.flat.data_ptr(), self.packed.data_ptr(),
                  torch.cuda.current_stream(self.device).cuda_stream)

    def rope(self, length: int) -> torch.Tensor:
        if length not in self._rope:
            self._rope[length] = rope_table(length).to(self.device)
        return self._rope[length]

    def named_parameters(self):
        return list(self.views.items())

    def state_dict(self) -> dict[str, torch.Tensor]:
        """The `final.pt` layout: the reference's keys and shapes, fp32, on CPU."""
        return {n: v.detach().cpu().clone() for n, v in self.views.items()}
