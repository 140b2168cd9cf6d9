"""noise_fitness_static — fitness shaping without any device allocation by the caller.

Some callers cannot allocate device memory (an FFI host with no device allocator of its own, or a
process whose device memory another allocator has fully reserved), so they cannot pass
noise_fitness a scratch buffer. noise_fitness_static keeps that scratch in a static array inside the
library. This file is collected last on purpose; it checks, through the C ABI, that two calls in a
row give exactly what the allocating entry point gives (ranks and weights bit-equal, the tolerance
the fitness tests use), and that a population beyond the array's limit is refused.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _allocating(losses, pairs, mode):
    from noise_b200 import _lib
    n = losses.numel()
    lib = _lib.load()
    ws = torch.empty(lib.noise_fitness_workspace_bytes(n), dtype=torch.uint8, device='cuda')
    w = torch.empty(pairs, device='cuda')
    r = torch.empty(n, dtype=torch.int32, device='cuda')
    _lib.call('noise_fitness', losses.data_ptr(), n, pairs, mode, w.data_ptr(), r.data_ptr(), ws.data_ptr(),
              ws.numel(), torch.cuda.current_stream().cuda_stream)
    return w, r


def _static(losses, pairs, mode):
    from noise_b200 import _lib
    n = losses.numel()
    w = torch.empty(pairs, device='cuda')
    r = torch.empty(n, dtype=torch.int32, device='cuda')
    _lib.call('noise_fitness_static', losses.data_ptr(), n, pairs, mode, w.data_ptr(), r.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    return w, r


@pytest.mark.parametrize('mode', [0, 1])
def test_static_scratch_matches_allocating_entry_point(mode):
    rng = np.random.default_rng(mode)
    for call, (n, pairs) in enumerate([(262144, 131072), (1024, 512)]):  # two calls in a row, largest first
        x = (8.3 + 1e-3 * rng.standard_normal(n)).astype(np.float32)
        x[3] = x[9]
        losses = torch.from_numpy(x).cuda()
        w_ref, r_ref = _allocating(losses, pairs, mode)
        w, r = _static(losses, pairs, mode)
        torch.cuda.synchronize()
        assert torch.equal(r, r_ref), f'call {call}: ranks differ'
        assert torch.equal(w, w_ref), f'call {call}: weights differ'


def test_static_scratch_without_ranks_buffer():
    """Mode 0 (the z-score fitness Eggroll uses by default) with no ranks buffer: the rank kernel is
    skipped and the pair differences read only the losses; two calls in a row, bit-equal weights."""
    from noise_b200 import _lib
    rng = np.random.default_rng(7)
    for call, (n, pairs) in enumerate([(4096, 2048), (1024, 256)]):
        losses = torch.from_numpy((8.3 + 1e-3 * rng.standard_normal(n)).astype(np.float32)).cuda()
        w_ref, _ = _allocating(losses, pairs, 0)
        w = torch.empty(pairs, device='cuda')
        _lib.call('noise_fitness_static', losses.data_ptr(), n, pairs, 0, w.data_ptr(), None,
                  torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert torch.equal(w, w_ref), f'call {call}: weights differ'


def test_static_scratch_limit():
    from noise_b200 import _lib
    lib = _lib.load()
    limit = lib.noise_fitness_static_max_members()
    assert limit == 262144
    losses = torch.zeros(limit + 2, device='cuda')
    w = torch.empty(1, device='cuda')
    rc = lib.noise_fitness_static(losses.data_ptr(), limit + 2, 1, 1, w.data_ptr(), None,
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 6  # NOISE_SCRATCH_LIMIT
