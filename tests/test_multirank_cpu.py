"""Multi-rank host logic on CPU with gloo (world size 2): member ranges, the reference's member ->
sequence layout, and the loss all-gather order, against a single-process run. The population
forward is replaced by a deterministic function of (member, sequence) so no GPU is needed."""
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
