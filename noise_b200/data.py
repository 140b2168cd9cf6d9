"""Synthetic token stream standing in for FineWeb `train.pt` rows (not available offline).

Token ids are iid Zipf(s) over ranks 1..vocab, P(rank k) proportional to k^-s, mapped to ids by a
seeded permutation; rows have the reference's 2049-token shape (`utils/prepare_data.py:19-21`),
x = row[:-1], y = row[1:].
"""
from __future__ import annotations

import torch


def zipf_tokens(rows: int, length: int = 2049, s: float = 1.1, vocab: int = 4096, seed: int = 1) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    ranks = torch.arange(1, vocab + 1, dtype=torch.float64)
    probs = ranks ** -s
    probs /= probs.sum()
    perm = torch.randperm(vocab, generator=g)
    samples = torch.multinomial(probs, rows * length, replacement=True, generator=g)
    return perm[samples].view(rows, length)


TRAIN_ROWS, VAL_ROWS, ROW = 4880, 544, 2049  # utils/prepare_data.py:19-21 (rows of 2049 tokens)


def load_rows(path, rows: int, synthetic: bool, seed: int) -> torch.Tensor:
    """The FineWeb token rows of utils/prepare_data.py:load_rows (shape-checked), or seeded Zipf(1.1)
    rows of the same shape when the file is absent and `synthetic` is set."""
    from pathlib import Path
    path = Path(path)
    if path.exists():
        data = torch.load(path)
        if tuple(data.shape) != (rows, ROW):
            raise ValueError(f'{path}: expected [{rows}, {ROW}], got {list(data.shape)}')
        return data
    if not synthetic:
        raise FileNotFoundError(f'{path} is missing (prepare the data, or pass --synthetic)')
    return zipf_tokens(rows, ROW, seed=seed)

