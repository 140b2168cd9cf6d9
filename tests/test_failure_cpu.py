"""Failure detection on the host, with gloo ranks on CPU (no GPU is made to fault).

1. A rank that raises inside its population forward: the other rank is waiting in Eggroll's loss
   all-gather (train/val/eggroll.py:147-150) and must leave it with an error once the peer is gone,
   within the process group's timeout, rather than hang.
2. A rank that never joins: init_process_group on the rank that did start must fail after its
   timeout instead of waiting for good.
3. Mismatched member counts across ranks are refused before any collective runs
   (tests/test_multirank_cpu.py::test_uneven_split_rejected covers the split itself).
"""
import datetime
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class _Model:
    device = torch.device('cpu')


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    from noise_b200.eggroll import Eggroll
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    t0 = time.time()
    try:
        def loss(model, p, noise, sign, idx, targets):
            if rank == 1:
                raise RuntimeError('injected failure in the population forward')
            return torch.zeros(noise.count)

        es = Eggroll(_Model(), 4, rank, world, all_sequences=True)
        es.loss = loss
        x = torch.zeros(2, 8, dtype=torch.long)
        es.gather(es.evaluate(x, x, step=1))
        result = 'completed'
    except Exception as e:  # noqa: BLE001 - the outcome is what the test reads
        result = f'{type(e).__name__}: {str(e)[:200]}'
    with open(f'{out}.{rank}', 'w') as f:
        f.write(f'{time.time() - t0:.1f}\n{result}')
    if rank == 1:
        os._exit(0)  # leave without tearing the group down, as a crashed rank would
    try:
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        pass


def test_rank_that_raises_ends_the_others_collective(tmp_path):
    out = str(tmp_path / 'outcome')
    ctx = mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, start_method='spawn', join=False)
    deadline = time.time() + 120
    while not ctx.join(timeout=5):
        assert time.time() < deadline, 'a rank is still waiting'
    seconds0, result0 = open(f'{out}.0').read().split('\n', 1)
    _, result1 = open(f'{out}.1').read().split('\n', 1)
    assert 'injected failure' in result1
    assert result0 != 'completed', result0  # the survivor's all-gather ended with an error
    assert float(seconds0) < 60


def _lonely(port, out):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    t0 = time.time()
    try:
        dist.init_process_group('gloo', rank=0, world_size=2, timeout=datetime.timedelta(seconds=5))
        result = 'joined'
    except Exception as e:  # noqa: BLE001
        result = f'{type(e).__name__}'
    with open(out, 'w') as f:
        f.write(f'{time.time() - t0:.1f}\n{result}')


def test_rank_that_never_joins_times_out(tmp_path):
    out = str(tmp_path / 'lonely')
    p = mp.get_context('spawn').Process(target=_lonely, args=(_free_port(), out))
    p.start()
    p.join(timeout=120)
    assert not p.is_alive(), 'init_process_group is still waiting'
    seconds, result = open(out).read().split('\n', 1)
    assert result != 'joined'
    assert float(seconds) < 60
