"""Counter-based draws, restated in numpy (test infrastructure; see oracle/__init__.py).

Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11) and Box-Muller, with the stream layout used by
noise_b200/csrc/philox.cuh:
    key     = (seed, step)
    counter = (element // 4, (tensor << 1) | vector, direction, domain)
    lane    = element % 4; lanes (0, 1) and (2, 3) are Box-Muller pairs.
The reference draws from a fixed 2^28-float Gaussian buffer at random offsets
(`train/val/eggroll.py:114-128`); noise_b200 replaces that buffer by this stream, and parity with
the reference is established by injecting the same draws into the reference's `population_loss`.
"""
from __future__ import annotations

import numpy as np

MUL0, MUL1 = 0xD2511F53, 0xCD9E8D57
WEYL0, WEYL1 = 0x9E3779B9, 0xBB67AE85
MASK = 0xFFFFFFFF
DOMAIN_LOWRANK = 0x4C52
DOMAIN_DIRECT = 0x4452


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Vectorised Philox4x32-10 over broadcastable uint32 counters; returns four uint32 arrays."""
    c0, c1, c2, c3 = (np.asarray(c, dtype=np.uint64) & MASK for c in (c0, c1, c2, c3))
    c0, c1, c2, c3 = np.broadcast_arrays(c0, c1, c2, c3)
    k0 = np.uint64(k0 & MASK)
    k1 = np.uint64(k1 & MASK)
    m0, m1 = np.uint64(MUL0), np.uint64(MUL1)
    for _ in range(10):
        p0 = m0 * c0
        p1 = m1 * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & np.uint64(MASK)
        hi1, lo1 = p1 >> np.uint64(32), p1 & np.uint64(MASK)
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        k0 = np.uint64((int(k0) + WEYL0) & MASK)
        k1 = np.uint64((int(k1) + WEYL1) & MASK)
    return tuple(x.astype(np.uint32) for x in (c0, c1, c2, c3))


def open_unit(x):
    """((x >> 8) + 0.5) * 2^-24: exact in float32, strictly inside (0, 1)."""
    return ((np.asarray(x, dtype=np.uint32) >> np.uint32(8)).astype(np.float64) + 0.5) * 2.0 ** -24


def box_muller(x0, x1):
    r = np.sqrt(-2.0 * np.log(open_unit(x0)))
    ang = 2.0 * np.pi * open_unit(x1)
    return r * np.cos(ang), r * np.sin(ang)


def raw_block(seed, step, blocks, tensor, vector, direction, domain=DOMAIN_LOWRANK):
    """uint32 outputs [len(blocks), 4] of the stream (tensor, vector, direction)."""
    blocks = np.asarray(blocks, dtype=np.uint64)
    out = philox4x32_10(blocks, (tensor << 1) | vector, direction, domain, seed, step)
    return np.stack(out, axis=-1)


def gaussians(seed, step, tensor, vector, directions, length, domain=DOMAIN_LOWRANK):
    """float64 draws [len(directions), length] of element 0..length-1 of each direction's stream."""
    directions = np.atleast_1d(np.asarray(directions, dtype=np.uint64))
    nblk = (length + 3) // 4
    blocks = np.arange(nblk, dtype=np.uint64)
    x = philox4x32_10(blocks[None, :], (tensor << 1) | vector, directions[:, None], domain, seed, step)
    z0, z1 = box_muller(x[0], x[1])
    z2, z3 = box_muller(x[2], x[3])
    z = np.stack([z0, z1, z2, z3], axis=-1).reshape(len(directions), nblk * 4)
    return z[:, :length]
