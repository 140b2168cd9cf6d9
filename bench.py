#!/usr/bin/env python
"""Benchmark of the B200 EGGROLL ES update (the 1xB200 rank-1 configuration, weak-scaled over N GPUs).

One step = one full ES update: population forward of 1024 rank-1 antithetic members per GPU
(512 directions per GPU, sigma 1e-3), every member on the same 8 Zipf(1.1) sequences x 2048 tokens,
per-member CE losses, NCCL all-gather of losses (N > 1), centred-rank fitness, each rank's partial
Sigma f eps reduce-scattered, AdamW (lr 1e-3) on the owned tensors, parameter all-gather and
packed-weight refresh.

Extra keys of the same line, measured in the same process after the headline (skip: --no-extras):
  fixed_population        BASELINE config 4: 16,384 members split over the N GPUs, ANVIL II on the
                          block matrices + AdamW elsewhere, seconds per update (strong scaling)
  dust                    seconds per DUST update at the speedrun recipe (5,440 draws, config 3) and at
                          24,576 direct draws (config 5), draws split over the GPUs
  eggroll_131072_pairs    (N >= 8) config 5's EGGROLL population: 262,144 members, one update
  rank_agreement          (N = 1, with the CPU baseline) Spearman rho of 64 members' GPU losses against
                          the float32 CPU oracle on the same draws, and antithetic-pair sign flips

    python bench.py [--gpus N --steps K --warmup W]          # this repository's CUDA path
    python bench.py --impl reference [...]                   # the reference's own ES update on the host cores
    python bench.py --workload dust [--dust-scale S]          # seconds per DUST update (a separate line)
Multi-GPU: python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = 'member-tokens/sec/GPU (pop 16k) and seconds per ES update at 1/2/4/8 B200'
UNIT = 'member-tokens/s'
# The reference's published EGGROLL record (README.md:67: 131,072 antithetic pairs, 5.33 h for 610 updates on
# 8xH100) is 262,144 members x 2,048 tokens per 31.5 s update: 2.13 M member-tokens/s per GPU.
PUBLISHED_PER_GPU = 2.13e6
SEQ, BATCH = 2048, 8
# Algorithmic FLOPs per member-token of each kernel kind over one forward:
# per block q,k,v,proj,fc,mlp GEMMs; attention QK+PV over visible keys only (avg keys per query
# 768.75 for the 1024-token windows, 1024.5 for the full ones); head 512 x 4096.
FLOPS_PER_TOKEN = {
    'qkv': 8 * 2 * 512 * 1536, 'attention': 6 * 2048 * 768.75 + 2 * 2048 * 1024.5, 'proj': 8 * 2 * 512 * 512,
    'fc': 8 * 2 * 512 * 2048, 'mlp': 8 * 2 * 2048 * 512, 'head': 2 * 512 * 4096,
}
FORWARD_FLOPS_PER_TOKEN = sum(FLOPS_PER_TOKEN.values())  # 68,168,704
KINDS = ['embed', 'qkv', 'attention', 'proj', 'fc', 'mlp', 'head', 'loss', 'fitness', 'update', 'pack', 'other']


def load_peaks():
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return d['bf16_tflops'], d.get('bf16_tflops_sustained', d['bf16_tflops']), d['hbm_gbs'], 'measured'
    return 1590.0, 1400.0, 6650.0, 'fallback'


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while the timed region runs."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            uuid = str(torch.cuda.get_device_properties(self.dev).uuid)
            target = uuid if uuid.startswith('GPU-') else f'GPU-{uuid}'
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                                          '-i', target, '-lms', '200'], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except (OSError, RuntimeError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.reader.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.lines:
            parts = [x.strip() for x in line.split(',')]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith('active'):
                    reasons.add(name)
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': mx, 'reasons': sorted(reasons),
                'samples': len(sm)}


def dist_setup():
    rank, world = int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1))
    local = int(os.environ.get('LOCAL_RANK', 0))
    return rank, world, local


def sdpa_window(q, k, v, window):
    """The reference's window attention (utils/model.py:14-31: key k visible to query q iff 0 <= q - k <=
    window, scale 1/sqrt(64)) as masked SDPA on [B, T, H, D]: flex_attention does not lower on CPU."""
    t = q.shape[1]
    i = torch.arange(t)
    mask = (i[:, None] >= i[None, :]) & (i[:, None] - i[None, :] <= window)
    return torch.nn.functional.scaled_dot_product_attention(
        q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), attn_mask=mask).transpose(1, 2)


REF_DIR = ROOT / 'baseline' / '_ref'


def reference_sample(steps: int = 1, length: int = SEQ):
    """Time the reference's own ES update on the host cores: train/val/eggroll.py Eggroll.step (its
    population_loss, offsets into the fixed N(0, 1) buffer, z-score fitness, reconstruction and
    torch.optim.AdamW) from the installed baseline/_ref, on one sequence with two antithetic pairs
    (4 members x `length` tokens per step, CHUNK = 1; one pair would z-score a single difference). Only the attention primitive is swapped, for
    the identical masked SDPA, and population_loss runs eagerly (Inductor's CPU lowering of
    flex_attention fails). Falls back to the CPU restatement in oracle/ when baseline/_ref is absent.
    Returns (member-tokens per step, seconds per step, cores, kind, sample)."""
    from noise_b200.data import zipf_tokens
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    rows = zipf_tokens(1, length + 1, seed=1)
    x, y = rows[:, :-1].contiguous(), rows[:, 1:].contiguous()
    times = []
    if (REF_DIR / 'train' / 'val' / 'eggroll.py').exists():
        sys.path.insert(0, str(REF_DIR))
        import train.val.eggroll as eg
        import utils.model as um
        um.attention = eg.attention = sdpa_window
        eg.CHUNK = 1
        model = eg.make_model(torch.device('cpu'), eg.SEED)
        opt = torch.optim.AdamW(model.parameters(), lr=eg.LR, betas=eg.BETAS, eps=1e-8, weight_decay=0.0)
        es = eg.Eggroll(model, 2)
        es.loss = eg.population_loss
        for step in range(1, steps + 1):
            t0 = time.perf_counter()
            es.step(x, y, opt, step)
            times.append(time.perf_counter() - t0)
        sample = (f'reference Eggroll.step (baseline/_ref, fp32 CPU): 2 pairs = 4 members x 1 sequence x {length} '
                  'tokens, z-score fitness, reconstruction, AdamW over all 37.7M parameters')
        return 4 * length, times, cores, 'reference', sample
    from oracle import eggroll as oe
    from oracle import model as om
    params = om.make_params(0)
    draws, sign = oe.member_draws([0, 1], 1, 1e-3, 0, 1)
    with torch.no_grad():
        for _ in range(steps):
            t0 = time.perf_counter()
            om.population_losses(params, draws, sign, x, y)
            times.append(time.perf_counter() - t0)
    sample = f'2 members x 1 sequence x {length} tokens of the rank-1 population forward (fp32 CPU oracle port)'
    return 2 * length, times, cores, 'port', sample


def rank_agreement(dev, members: int = 64, length: int = 512):
    """How the GPU's bf16-operand member losses order members against the float32 CPU oracle on the same
    counter-based draws (oracle/ restates train/val/eggroll.py:66-103 and is pinned to the reference by
    tests/golden/population.npz): 64 members = 32 antithetic pairs at sigma 1e-3 on one sequence of 512
    tokens. Spearman rho of the losses, the pairs whose antithetic difference L[2i+1] - L[2i] changes
    sign, and the largest oracle |difference| among those (a flip is a near tie within bf16 rounding)."""
    import numpy as np
    from noise_b200.data import zipf_tokens
    from noise_b200.model import Weights
    from noise_b200.population import population_losses
    from oracle import eggroll as oe
    from oracle import model as om
    rows = zipf_tokens(1, length + 1, seed=17)
    x, y = rows[:, :-1], rows[:, 1:]
    pairs, sigma = members // 2, 1e-3
    got = population_losses(Weights(dev, seed=0), x, y, 0, members, pairs, sigma, 0, 1).cpu().double().numpy()
    draws, sign = oe.member_draws(np.arange(members), pairs, sigma, 0, 1)
    with torch.no_grad():
        want = om.population_losses(om.make_params(0), draws, sign, x, y).double().numpy()
    rg, rw = np.argsort(np.argsort(got)), np.argsort(np.argsort(want))
    rho = 1 - 6 * float(np.sum((rg - rw) ** 2)) / (members * (members ** 2 - 1))
    dg, dw = got[1::2] - got[0::2], want[1::2] - want[0::2]
    flips = np.sign(dg) != np.sign(dw)
    return {'members': members, 'tokens': length, 'sigma': sigma, 'spearman': rho, 'pairs': pairs,
            'pair_sign_flips': int(flips.sum()),
            'max_flipped_oracle_abs_diff': float(np.abs(dw[flips]).max()) if flips.any() else 0.0,
            'median_oracle_abs_diff': float(np.median(np.abs(dw))),
            'max_abs_loss_error': float(np.max(np.abs(got - want))),
            'checker': 'float32 CPU restatement of population_loss (oracle/)'}


def run_reference(args, rank, world):
    if rank != 0:
        return
    tok, times, cores, kind, sample = reference_sample(args.warmup + args.steps, SEQ)
    timed = times[args.warmup:] or times
    per_step = sum(timed) / len(timed)
    value = tok / per_step
    line = {
        'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': args.gpus, 'steps': len(timed),
        'warmup': args.warmup, 'ms_per_step': per_step * 1e3, 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic Zipf(1.1) tokens, seed-0 random init',
        'config': workload_config(world, args),
        'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': cores, 'kind': kind, 'sample': sample},
        'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(world, args):
    return {'workload': 'eggroll-rank1-antithetic', 'members_per_gpu': 2 * args.pairs_per_gpu,
            'pairs': args.pairs_per_gpu * world, 'sigma': args.sigma, 'sequences_per_member': BATCH,
            'seq_len': SEQ, 'fitness': 'centered_rank', 'optimizer': 'adamw lr 1e-3 betas (0.5, 0.95)',
            'update': 'sharded: per-rank partial sum f eps, reduce-scatter, region AdamW, parameter all-gather',
            'parallelism': f'members sharded dp{world}', 'operands': 'bf16 GEMM operands, fp32 accumulate/head/CE',
            'l2': 'inputs larger than L2 (activations streamed per chunk, GBs)'}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=5)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='noise', choices=['noise', 'reference'])
    ap.add_argument('--pairs-per-gpu', type=int, default=512)
    ap.add_argument('--sigma', type=float, default=1e-3)
    ap.add_argument('--workspace-gb', type=float, default=32.0)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--workload', default='eggroll', choices=['eggroll', 'dust'],
                    help='eggroll (the headline line) or dust: seconds per DUST update, a separate line')
    ap.add_argument('--dust-scale', type=float, default=0.3125, help='DUST recipe scale (1.0 = the 16k cell)')
    ap.add_argument('--no-extras', action='store_true',
                    help='skip the extra configurations (fixed population 16,384 with ANVIL, DUST updates)')
    args = ap.parse_args()
    rank, world, local = dist_setup()
    if args.impl == 'reference':
        run_reference(args, rank, world)
        return
    if args.workload == 'dust':
        run_dust(args, rank, world, local)
        return

    from noise_b200 import _lib, population
    from noise_b200.data import zipf_tokens
    from noise_b200.eggroll import BETAS, Eggroll
    from noise_b200.model import Weights
    from noise_b200.shard import ShardedOptimizer

    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        torch.distributed.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=dev)
    population.DEFAULT_WORKSPACE_BYTES = int(args.workspace_gb * (1 << 30))
    lib = _lib.load()

    pairs = args.pairs_per_gpu * world
    members_total = 2 * pairs
    w = Weights(dev, seed=0)
    opt = ShardedOptimizer(w, rank, world, kind='adamw', lr=1e-3, betas=BETAS)
    es = Eggroll(w, pairs, rank, world, sigma=args.sigma, seed=0, fitness='centered_rank', all_sequences=True)
    rows = zipf_tokens(BATCH, SEQ + 1, seed=1)
    rows_dev = rows.to(dev)
    x, y = rows_dev[:, :-1], rows_dev[:, 1:]
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    step = 0
    for _ in range(args.warmup):
        step += 1
        es.step(x, y, opt, step)
    torch.cuda.synchronize()

    # ---- device-resident timed region ----
    barrier()
    torch.cuda.synchronize()
    launches0 = lib.noise_launch_count()
    _lib.call('noise_profile_enable', 1)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            step += 1
            es.step(x, y, opt, step)
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    launches = lib.noise_launch_count() - launches0
    ms_kind = (ctypes_array('d', len(KINDS)), ctypes_array('q', len(KINDS)))
    _lib.call('noise_profile_read', ms_kind[0].buffer_info()[0], ms_kind[1].buffer_info()[0], len(KINDS))
    _lib.call('noise_profile_enable', 0)
    ms = ev0.elapsed_time(ev1) / args.steps
    t = torch.tensor([ms, float(launches)], dtype=torch.float64, device=dev)
    if world > 1:
        mx = t[:1].clone()
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
        sm = t[1:].clone()
        torch.distributed.all_reduce(sm, op=torch.distributed.ReduceOp.SUM)
        ms, launches = mx.item(), int(sm.item())
    tokens_per_step = members_total * BATCH * SEQ
    value = tokens_per_step / (ms / 1e3)

    # ---- end to end through the public API, host buffers ----
    host = rows.pin_memory()
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    ev2.record(stream)
    for _ in range(args.steps):
        step += 1
        rows_dev.copy_(host, non_blocking=True)
        es.step(rows_dev[:, :-1], rows_dev[:, 1:], opt, step)  # returns the mean loss on the host
    ev3.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = ev2.elapsed_time(ev3) / args.steps
    if world > 1:
        te = torch.tensor([ms_e2e], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
        ms_e2e = te.item()

    # ---- roofline of the dominant kernel, from the live per-kind events ----
    peak_burst, peak_sustained, hbm, peak_kind = load_peaks()
    kind_ms = {k: ms_kind[0][i] for i, k in enumerate(KINDS)}
    kind_n = {k: ms_kind[1][i] for i, k in enumerate(KINDS)}
    local_tokens = (members_total // world) * BATCH * SEQ * args.steps
    dominant = max(FLOPS_PER_TOKEN, key=lambda k: kind_ms[k])
    achieved = FLOPS_PER_TOKEN[dominant] * local_tokens / (kind_ms[dominant] / 1e3) / 1e12
    fwd_ms = sum(kind_ms[k] for k in ('embed', 'qkv', 'attention', 'proj', 'fc', 'mlp', 'head', 'loss'))
    fwd_tflops = FORWARD_FLOPS_PER_TOKEN * local_tokens / (fwd_ms / 1e3) / 1e12
    roofline = {
        'bound': 'tensor', 'kernel': dominant, 'achieved': achieved, 'peak': peak_sustained, 'unit': 'TFLOP/s',
        'frac': achieved / peak_sustained, 'peak_source': f'{peak_kind} bf16_tflops_sustained',
        'traffic': (TRAFFIC_BYTES_PER_ROW[dominant] * local_tokens * (1 if dominant == 'head' else 8)
                    / max(1, kind_n[dominant])) if dominant in TRAFFIC_BYTES_PER_ROW else None,
        'launches': kind_n[dominant], 'ms_per_launch': kind_ms[dominant] / max(1, kind_n[dominant]),
        'population_forward': {'achieved': fwd_tflops, 'frac': fwd_tflops / peak_sustained,
                               'frac_of_burst': fwd_tflops / peak_burst},
        'kernel_ms_per_step': {k: round(kind_ms[k] / args.steps, 3) for k in KINDS if kind_n[k]},
    }

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tok, times, cores, kind, sample = reference_sample(3, SEQ)
        cpu = {'value': tok / min(times[1:]), 'unit': UNIT, 'cores': cores, 'kind': kind, 'sample': sample}
        # the oracle's second use here: checking the GPU's member ranking on a small case
        extras_rank = rank_agreement(dev)

    extras = {}
    if cpu is not None:
        extras['rank_agreement'] = extras_rank
    if not args.no_extras:
        # one timed update where an update takes tens of seconds (up to 2 GPUs), two above
        extras['fixed_population'] = fixed_population(rank, world, dev, FIXED_MEMBERS, args.sigma, barrier,
                                                      steps=1 if world <= 2 else 2)
        extras['dust'] = {f'{scale}': dust_update(rank, world, dev, scale, steps, barrier)
                          for scale, steps in DUST_SCALES}
        if world >= 8:
            extras['eggroll_131072_pairs'] = fixed_population(rank, world, dev, 2 * 131072, args.sigma, barrier,
                                                              steps=1, warmup=0, kind='adamw')

    if rank == 0:
        clk = clocks.summary()
        line = {
            'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': ms, 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': (value / world) / PUBLISHED_PER_GPU, 'dtype': 'bf16',
            'data': 'synthetic Zipf(1.1) tokens, seed-0 random init (FineWeb unavailable offline)',
            'config': workload_config(world, args),
            'per_gpu': value / world, 's_per_update': ms / 1e3,
            'e2e': {'value': tokens_per_step / (ms_e2e / 1e3), 'unit': UNIT,
                    'h2d_bytes_per_step': host.numel() * host.element_size(), 'd2h_bytes_per_step': 4},
            'gpu_launches': launches, 'roofline': roofline, 'cpu_baseline': cpu,
            'clocks': {'sm_mhz': clk['sm_mhz'], 'sm_max_mhz': clk['sm_max_mhz'], 'reasons': clk['reasons']},
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# population 16,384 split over the GPUs (strong scaling), ANVIL II on the block
# matrices and AdamW elsewhere, the sharded update. Config 5's direct-draw population: the DUST recipe
# scale with 24,576 draws per update; the speedrun recipe (0.3125, 5,440 draws) is config 3's.
FIXED_MEMBERS = 16384
DUST_SCALES = ((0.3125, 2), (1.2657, 1))


def timed_steps(fn, steps, warmup, barrier, dev):
    """Device time per call of fn() (CUDA events on the current stream after `warmup` untimed calls),
    max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        fn()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1) / steps
    if torch.distributed.is_initialized():
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
    return ms


def fixed_population(rank, world, dev, members, sigma, barrier, steps=2, warmup=1, kind='anvil'):
    """Seconds per full ES update (draw generation through the optimizer step) at a fixed population
    split over the ranks: rank-1 antithetic members on the same 8 x 2048-token batch, centred-rank
    fitness, the sharded update (partial Sigma f eps, reduce-scatter, region optimizer, all-gather)."""
    from noise_b200 import _lib
    from noise_b200.data import zipf_tokens
    from noise_b200.dust import recipe
    from noise_b200.eggroll import BETAS, Eggroll
    from noise_b200.model import Weights
    from noise_b200.shard import ShardedOptimizer
    rec = recipe(1.0)
    w = Weights(dev, seed=0)
    opt = ShardedOptimizer(w, rank, world, kind=kind, lr=1e-3, betas=BETAS, anvil_lr=rec.anvil_lr,
                           anvil_wd=rec.anvil_wd, steps=610)
    es = Eggroll(w, members // 2, rank, world, sigma=sigma, seed=0, fitness='centered_rank', all_sequences=True)
    rows = zipf_tokens(BATCH, SEQ + 1, seed=1).to(dev)
    x, y = rows[:, :-1], rows[:, 1:]
    state = {'step': 0}

    def one():
        state['step'] += 1
        es.step(x, y, opt, state['step'])

    _lib.call('noise_profile_enable', 1)
    ms = timed_steps(one, steps, warmup, barrier, dev)
    kinds = (ctypes_array('d', len(KINDS)), ctypes_array('q', len(KINDS)))
    _lib.call('noise_profile_read', kinds[0].buffer_info()[0], kinds[1].buffer_info()[0], len(KINDS))
    _lib.call('noise_profile_enable', 0)
    calls = warmup + steps
    tokens = members * BATCH * SEQ
    return {'members': members, 'pairs': members // 2, 'members_per_gpu': members // world, 's_per_update': ms / 1e3,
            'value': tokens / (ms / 1e3), 'unit': UNIT, 'steps': steps, 'warmup': warmup,
            'optimizer': 'ANVIL II on block matrices, AdamW x300/x30/x1 elsewhere' if kind == 'anvil' else 'AdamW',
            'update': 'sharded: per-rank partial sum f eps, reduce-scatter, region optimizer, parameter all-gather',
            'update_ms_per_step': kinds[0][KINDS.index('update')] / calls,
            'fitness_ms_per_step': kinds[0][KINDS.index('fitness')] / calls,
            'scaling': 'strong'}


def dust_update(rank, world, dev, scale, steps, barrier, warmup=1):
    """Seconds per DUST update (train/val/run.py DUST.step with ANVIL II + AdamW) on 8 x 2048 tokens
    copied from pinned host memory each step, the recipe's draws split over the ranks."""
    from noise_b200.data import zipf_tokens
    from noise_b200.dust import DUST, recipe
    from noise_b200.model import Weights
    from noise_b200.optim import make_sharded_optimizer
    rec = recipe(scale)
    w = Weights(dev, seed=0)
    est = DUST(w, rec, 0, rank, world)
    opt = make_sharded_optimizer(w, rec.lr, rec.betas, rec.anvil_lr, rec.anvil_wd, 610, rank, world)
    rows = zipf_tokens(BATCH, SEQ + 1, seed=1).pin_memory()
    x, y = rows[:, :-1], rows[:, 1:]
    ms = timed_steps(lambda: est.step(x, y, opt), steps, warmup, barrier, dev)
    draws = sum(rec.writers) + sum(rec.hidden) + sum(rec.hubs) + rec.embedding + sum(rec.local.values())
    published = DUST_PUBLISHED_8XH100.get(scale)
    return {'recipe_scale': scale, 'draws_per_update': draws, 's_per_update': ms / 1e3, 'steps': steps,
            'warmup': warmup, 'reference_8xh100_s_per_update': published, 'scaling': 'strong',
            'update': 'estimate reduce-scattered, ANVIL II / AdamW on owned tensors, parameter all-gather'}


# The reference's own logs on 8xH100 (train/val/log, train/speedrun/log): seconds per DUST update.
DUST_PUBLISHED_8XH100 = {1.0: 4303.45 / 610, 0.3125: 1309.72 / 610}


def run_dust(args, rank, world, local):
    """Seconds per DUST update (train/val/run.py DUST.step + ANVIL II / AdamW) on B = 8 sequences of
    2048 tokens, inputs copied from pinned host memory every step; the recipe's draws split over the
    GPUs (strong scaling, as the reference)."""
    from noise_b200 import _lib
    from noise_b200.data import zipf_tokens
    from noise_b200.dust import DUST, recipe
    from noise_b200.model import Weights
    from noise_b200.optim import make_sharded_optimizer

    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        torch.distributed.init_process_group('nccl', timeout=datetime.timedelta(seconds=600), device_id=dev)
    lib = _lib.load()
    rec = recipe(args.dust_scale)
    w = Weights(dev, seed=0)
    est = DUST(w, rec, 0, rank, world)
    opt = make_sharded_optimizer(w, rec.lr, rec.betas, rec.anvil_lr, rec.anvil_wd, 610, rank, world)
    rows = zipf_tokens(BATCH, SEQ + 1, seed=1).pin_memory()
    x, y = rows[:, :-1], rows[:, 1:]
    for _ in range(args.warmup):
        est.step(x, y, opt)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    stream = torch.cuda.current_stream(dev)
    launches0 = lib.noise_launch_count()
    _lib.call('noise_profile_enable', 1)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            loss = est.step(x, y, opt)  # reads the clean loss back to the host
        ev1.record(stream)
        torch.cuda.synchronize()
    launches = lib.noise_launch_count() - launches0
    ms_kind = (ctypes_array('d', len(KINDS)), ctypes_array('q', len(KINDS)))
    _lib.call('noise_profile_read', ms_kind[0].buffer_info()[0], ms_kind[1].buffer_info()[0], len(KINDS))
    _lib.call('noise_profile_enable', 0)
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    published = DUST_PUBLISHED_8XH100.get(args.dust_scale)
    clk = clocks.summary()
    draws = sum(rec.writers) + sum(rec.hidden) + sum(rec.hubs) + rec.embedding + sum(rec.local.values())
    line = {
        'metric': 'seconds per DUST update (B = 8 x 2048 tokens)', 'value': ms / 1e3, 'unit': 's',
        'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms, 'higher_is_better': False,
        'scaling': 'strong', 'vs_baseline': (ms / 1e3) / published if (published and world == 8) else None,
        'dtype': 'bf16', 'data': 'synthetic Zipf(1.1) tokens, seed-0 random init (FineWeb unavailable offline)',
        'config': {'workload': f'dust-recipe-{args.dust_scale}', 'draws_per_update': draws,
                   'optimizer': 'ANVIL II on block matrices, AdamW elsewhere',
                   'reference_8xh100_s_per_update': published, 'last_clean_loss': loss},
        'e2e': {'value': ms / 1e3, 'unit': 's', 'h2d_bytes_per_step': rows.numel() * rows.element_size(),
                'd2h_bytes_per_step': 4},
        'gpu_launches': launches,
        'kernel_ms_per_step': {k: round(ms_kind[0][i] / args.steps, 3) for i, k in enumerate(KINDS) if ms_kind[1][i]},
        'clocks': {'sm_mhz': clk['sm_mhz'], 'sm_max_mhz': clk['sm_max_mhz'], 'reasons': clk['reasons']},
    }
    print(json.dumps(line), flush=True)


# DRAM bytes (read + write) per population row of one launch of each kind, from one ncu capture of the
# small case (262,144 rows per launch); traffic grows in proportion to the rows, so a bench launch's
# traffic is this times its rows.
TRAFFIC_BYTES_PER_ROW = {'attention': 4063, 'qkv': 4523, 'proj': 6203, 'fc': 5071, 'mlp': 9548}


def ctypes_array(code, n):
    import array
    return array.array(code, [0] * n)


if __name__ == '__main__':
    main()
