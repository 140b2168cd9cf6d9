"""The sharded update's host logic on CPU: the ownership plan, and the reduce-scatter / optimizer /
all-gather choreography on two gloo ranks against one process.

The CUDA kernels are replaced by CPU stand-ins with the same contracts: the partial reconstruction
writes sum over the rank's directions of w_d f(d) for every tensor at its out_offsets entry (f a
deterministic function of the direction and the flat index), and the region optimizer is SGD on
the region's tensors. Tolerance: parameters after two updates equal one process's to rtol 1e-6
(only the order of the fp32 sums differs), and equal across ranks bit for bit.
"""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from noise_b200.model import N_PARAMS, PARAM_SPECS

LR = 0.1


class CpuWeights:
    device = torch.device('cpu')

    def __init__(self):
        self.flat = torch.linspace(-1.0, 1.0, N_PARAMS, dtype=torch.float32)

    def pack(self):
        pass


def contribution(fw, d0, dn):
    """sum_{d in [d0, d0 + dn)} w_d f(d) over the flat layout, f(d)[i] = cos(0.37 d + 1e-5 i)."""
    i = torch.arange(N_PARAMS, dtype=torch.float64)
    g = torch.zeros(N_PARAMS, dtype=torch.float64)
    for d in range(d0, d0 + dn):
        g += float(fw[d]) * torch.cos(0.37 * d + 1e-5 * i)
    return g.float()


class CpuKernels:
    def partial(self, fw, pairs, d0, dn, scale, seed, step, offsets, out):
        g = -scale * contribution(fw, d0, dn)
        off = 0
        for t, (_, s) in enumerate(PARAM_SPECS):
            n = math.prod(s)
            out[offsets[t]:offsets[t] + n] = g[off:off + n]
            off += n


class RegionSgd:
    def __init__(self, w, region):
        self.w, self.region = w, region

    def step(self, grad):
        lo = sum(math.prod(s) for _, s in PARAM_SPECS[:self.region.tensor_begin])
        hi = sum(math.prod(s) for _, s in PARAM_SPECS[:self.region.tensor_end])
        self.w.flat[lo:hi] -= LR * grad[lo - self.region.base:hi - self.region.base]


def _run(rank, world, steps=2, pairs=6):
    from noise_b200.shard import ShardedOptimizer, ShardPlan
    w = CpuWeights()
    opt = ShardedOptimizer(w, rank, world, kernels=CpuKernels(),
                           optimizers=[RegionSgd(w, ShardPlan(world).region(rank))])
    for step in range(1, steps + 1):
        fw = torch.linspace(-1.0, 1.0, pairs) * step
        opt.zero_grad()
        opt.set_sum_fe(fw, 1.0 / pairs, 0, step)
        opt.step()
    return w.flat


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        torch.save(_run(rank, world), f'{out}.{rank}')
    finally:
        dist.destroy_process_group()


def test_plan_owns_every_tensor_once():
    from noise_b200.shard import ShardPlan
    total = sum(math.prod(s) for _, s in PARAM_SPECS)
    for world in (1, 2, 3, 4, 8):
        p = ShardPlan(world)
        assert p.bounds[0] == 0 and p.bounds[-1] == len(PARAM_SPECS) and p.bounds == sorted(p.bounds)
        assert sum(p.count) == total and p.size % 64 == 0 and p.size >= max(p.count)
        # every tensor lands inside its owner's padded region, regions start on 256-byte boundaries
        for t, (_, s) in enumerate(PARAM_SPECS):
            r = p.owner[t]
            assert r * p.size <= p.out_offsets[t] and p.out_offsets[t] + math.prod(s) <= r * p.size + p.count[r]
        assert max(p.count) <= 1.25 * total / world or world == 1 or max(p.count) == max(p.sizes)
        # the directions split into disjoint ranges that cover [0, P)
        for pairs in (1, 7, 512, 131072):
            spans = [p.directions(r, pairs) for r in range(world)]
            assert spans[0][0] == 0 and sum(n for _, n in spans) == pairs
            assert all(spans[r][0] + spans[r][1] == spans[r + 1][0] for r in range(world - 1))


def test_two_ranks_match_one(tmp_path):
    single = _run(0, 1)
    out = str(tmp_path / 'params')
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, start_method='spawn')
    got = [torch.load(f'{out}.{r}') for r in range(2)]
    assert torch.equal(got[0], got[1])
    torch.testing.assert_close(got[0], single, rtol=1e-6, atol=1e-7)
    assert not torch.equal(single, CpuWeights().flat)


def _run_dense(rank, world, steps=2):
    """Each rank holds its own share of a dense gradient (rank-dependent); the update must equal one
    process stepping with the average of the shares."""
    from noise_b200.shard import ShardedOptimizer, ShardPlan
    w = CpuWeights()
    opt = ShardedOptimizer(w, rank, world, kernels=CpuKernels(),
                           optimizers=[RegionSgd(w, ShardPlan(world).region(rank))])
    i = torch.arange(N_PARAMS, dtype=torch.float64)
    for step in range(1, steps + 1):
        if world == 1:  # one process: the average of both ranks' shares
            share = sum(torch.sin(0.3 * step + 0.7 * r + 1e-5 * i) for r in range(2)).float() / 2
        else:
            share = torch.sin(0.3 * step + 0.7 * rank + 1e-5 * i).float()
        assert opt.step_dense(share, 1.0 / world)
    return w.flat


def _worker_dense(rank, world, port, out):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        torch.save(_run_dense(rank, world), f'{out}.{rank}')
    finally:
        dist.destroy_process_group()


def test_dense_shares_two_ranks_match_one(tmp_path):
    """DUST's path: the ranks' dense gradient shares reduce-scattered and averaged, regions stepped,
    parameters all-gathered (rtol 1e-6 against one process with the averaged gradient)."""
    single = _run_dense(0, 1)
    out = str(tmp_path / 'dense')
    mp.start_processes(_worker_dense, args=(2, _free_port(), out), nprocs=2, start_method='spawn')
    got = [torch.load(f'{out}.{r}') for r in range(2)]
    assert torch.equal(got[0], got[1])
    torch.testing.assert_close(got[0], single, rtol=1e-6, atol=1e-7)


def test_dense_step_refuses_non_finite():
    from noise_b200.shard import ShardedOptimizer, ShardPlan
    w = CpuWeights()
    before = w.flat.clone()
    opt = ShardedOptimizer(w, 0, 1, kernels=CpuKernels(), optimizers=[RegionSgd(w, ShardPlan(1).region(0))])
    g = torch.zeros(N_PARAMS)
    g[12345] = float('nan')
    assert opt.step_dense(g) is False
    assert torch.equal(w.flat, before)
