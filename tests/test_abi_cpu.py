"""The C-ABI library on a machine without a GPU: it loads, it exports every function that
include/noise_b200.h declares, the Python binding (noise_b200/_lib.py) gives each of them a signature,
and the host-only size queries return the sizes the header documents. No call here touches a device.
"""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / 'include' / 'noise_b200.h'

# per population row, in the workspace's carve order: x fp32, xb bf16, qkv bf16, y bf16, hidden bf16,
# stats_a [4][16] fp32, stats_b [2][2] fp32, y.b_proj per head, hidden.b_mlp partials, 1/rms, head pieces
ROW_BYTES = [2048, 1024, 3072, 1024, 4096, 256, 16, 32, 8, 4, 16]
ROPE_BYTES = 20480 * 64 * 2      # the bf16 rotary table, sized for the longest sequence
DRAW_FLOATS_PER_DIRECTION = 101_560
DRAW_MAX_DIRECTIONS = 512


def declared() -> list[str]:
    text = re.sub(r'/\*.*?\*/', '', HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r'\b(noise_[a-z0-9_]+)\s*\(', text)))


def round_up(n: int, k: int = 256) -> int:
    return (n + k - 1) // k * k


def test_header_declares_the_entry_points():
    names = declared()
    for name in ('noise_pop_forward_lowrank', 'noise_pop_forward_direct', 'noise_fitness', 'noise_fitness_static',
                 'noise_update_sum_fe_adamw', 'noise_dust_errors', 'noise_local_errors'):
        assert name in names, name


def test_library_exports_and_binds_every_declared_function():
    from noise_b200 import _lib
    lib = _lib.load()
    names = declared()
    assert [n for n in names if not hasattr(lib, n)] == []
    assert [n for n in names if n not in _lib.SIGNATURES] == []


def test_parameter_and_packed_counts():
    from noise_b200 import _lib
    lib = _lib.load()
    assert lib.noise_param_count() == 37_749_776  # the final.pt layout
    # per block [c_q; c_k; c_v] | c_proj | c_fc | mlp.c_proj, then lm_head, in bf16
    assert lib.noise_packed_count() == 8 * (1536 * 512 + 512 * 512 + 2048 * 512 + 512 * 2048) + 4096 * 512


def test_population_workspace_bytes():
    """Per-row activations, the rotary table and the chunk's draw table (at most min(512, rows/256 + 2)
    directions of 406 KB)."""
    from noise_b200 import _lib
    lib = _lib.load()
    for rows in (128, 3 * 128, 2 * 2048, 16 * 16384, 147 * 16384):
        cap = min(DRAW_MAX_DIRECTIONS, rows // 256 + 2)
        want = ROPE_BYTES + round_up(cap * DRAW_FLOATS_PER_DIRECTION * 4) + sum(round_up(b * rows) for b in ROW_BYTES)
        assert lib.noise_pop_workspace_bytes(rows) == want, rows


def test_other_size_queries():
    from noise_b200 import _lib
    lib = _lib.load()
    assert lib.noise_fitness_workspace_bytes(1024) == round_up(1024 * 4) + (1024 // 2 + 1) * 8
    assert lib.noise_local_workspace_bytes(8, 2048, 16) == 16 * 8 * 2048 * (512 * 2 + 2 * 8 * 4) + 1024
    assert lib.noise_local_workspace_bytes(0, 2048, 16) == -1
    assert lib.noise_fitness_static_max_members() == 262_144
