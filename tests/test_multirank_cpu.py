"""Multi-rank host logic on CPU with gloo (world size 2), against a single-process run: member ranges,
the reference's member -> sequence layout and the loss all-gather order (the population forward is
replaced by a deterministic function of (member, sequence), so no GPU is needed), and the credit
memory's rank averages."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class _Model:
    device = torch.device('cpu')


def fake_loss(model, p, noise, sign, idx, targets):
    """loss(member j, rows) = j + 0.001 * first token of the row block (identifies the sequence)."""
    first = float(idx.reshape(-1)[0])
    return torch.arange(noise.begin, noise.begin + noise.count, dtype=torch.float32) + 1e-3 * first


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _losses(rank, world, pairs, all_sequences, x):
    from noise_b200.eggroll import Eggroll
    es = Eggroll(_Model(), pairs, rank, world, all_sequences=all_sequences, chunk=2)
    es.loss = fake_loss
    return es.gather(es.evaluate(x, x, step=1))


def _worker(rank, world, port, pairs, all_sequences, out):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        x = torch.arange(4 * 8).view(4, 8) * 10
        got = _losses(rank, world, pairs, all_sequences, x)
        torch.save(got, f'{out}.{rank}')
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('pairs,all_sequences', [(8, False), (2, False), (8, True)])
def test_two_ranks_match_one(tmp_path, pairs, all_sequences):
    x = torch.arange(4 * 8).view(4, 8) * 10
    single = _losses(0, 1, pairs, all_sequences, x)
    out = str(tmp_path / 'losses')
    mp.start_processes(_worker, args=(2, _free_port(), pairs, all_sequences, out), nprocs=2, start_method='spawn')
    for rank in range(2):
        assert torch.equal(torch.load(f'{out}.{rank}'), single)
    # reference layout: members = max(2P, 2B), member j on sequence j // (members / B)
    members = 2 * pairs if all_sequences else max(2 * pairs, 2 * 4)
    assert single.numel() == members
    if not all_sequences:
        per_seq = members // 4
        seq = torch.arange(members) // per_seq
        torch.testing.assert_close(single - torch.arange(members, dtype=torch.float32), 1e-3 * (seq * 80).float())


def test_uneven_split_rejected():
    from noise_b200.eggroll import Eggroll
    es = Eggroll(_Model(), 3, 0, 4, all_sequences=True)
    with pytest.raises(ValueError):
        es.member_range(8)


def _memory_inputs(rank, steps=2, tokens=48, keys=32, width=8):
    """Rank r's credit [tokens, keys] and one site's estimate [tokens, width] per step, and its fit."""
    g = torch.Generator().manual_seed(100 + rank)
    return [(torch.randn(tokens, keys, generator=g, dtype=torch.float64),
             torch.randn(tokens, width, generator=g, dtype=torch.float64),
             torch.randn(2, generator=g, dtype=torch.float64).abs()) for _ in range(steps)]


def _memory_run(world, inputs):
    """calibrate + remember over the steps, as DUST.step does once a step."""
    from noise_b200.dust import CreditMemory
    mem = CreditMemory(world=world)
    for credit, est, fit in inputs:
        mem.estimates['site'] = est
        mem.fits['site'] = fit
        mem.calibrate()
        mem.remember(credit, valid=2.0)
    return mem


def _memory_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        mem = _memory_run(world, _memory_inputs(rank))
        torch.save({'P': mem.P, 'S': mem.S['site'], 'alpha': mem.alpha['site']}, f'{out}.{rank}')
    finally:
        dist.destroy_process_group()


def test_credit_memory_rank_average(tmp_path):
    """train/val/run.py:304-330 with world 2: the key covariance, the site's regression statistic and
    the fitted alpha are the averages over ranks, identical on both ranks and equal to one process
    that sees the rank-averaged statistics (c^T c, e^T c and the fits are averaged before the EMAs)."""
    out = str(tmp_path / 'memory')
    mp.start_processes(_memory_worker, args=(2, _free_port(), out), nprocs=2, start_method='spawn')
    got = [torch.load(f'{out}.{r}') for r in range(2)]
    for k in ('P', 'S'):
        assert torch.equal(got[0][k], got[1][k])
    assert got[0]['alpha'] == got[1]['alpha']
    # one process: P = EMA of mean_r(c_r^T c_r) / valid, S = EMA of mean_r(e_r^T c_r) / valid,
    # alpha = EMA<r, e> / EMA|r|^2 of the mean fits
    beta, ab = 0.9, 0.8
    a, b = _memory_inputs(0), _memory_inputs(1)
    P = S = cal = None
    for (c0, e0, f0), (c1, e1, f1) in zip(a, b):
        fit = (f0 + f1) / 2
        cal = fit if cal is None else ab * cal + (1 - ab) * fit
        C = (c0.T @ c0 + c1.T @ c1) / 2 / 2.0
        G = (e0.T @ c0 + e1.T @ c1) / 2 / 2.0
        P = C * (1 - beta) if P is None else beta * P + (1 - beta) * C
        S = G * (1 - beta) if S is None else beta * S + (1 - beta) * G
    torch.testing.assert_close(got[0]['P'], P, rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(got[0]['S'], S, rtol=1e-12, atol=1e-12)
    assert abs(got[0]['alpha'] - float(cal[0] / cal[1])) < 1e-12
