"""ctypes binding of the C ABI declared in include/noise_b200.h.

The product path has exactly one implementation: the CUDA kernels in libnoise_b200.so. If the
library is missing or cannot be loaded, every call raises; nothing falls back to a CPU path.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / 'libnoise_b200.so'

NOISE_OK = 0
STATUS_NAMES = {
    0: 'ok', 1: 'bad argument', 2: 'launch failed', 3: 'device wait timed out',
    4: 'workspace too small', 5: 'unsupported configuration',
    6: 'larger than the static scratch array holds',
}

c_void_p, c_int, c_float, c_int64, c_uint32, c_size_t, c_uint64 = (
    ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int64, ctypes.c_uint32, ctypes.c_size_t,
    ctypes.c_uint64)

# name -> (restype, argtypes); the single source of truth for what the Python side binds.
SIGNATURES: dict[str, tuple] = {
    'noise_gemm_bf16': (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_int,
                                c_void_p, c_void_p]),
    'noise_selftest_wait_timeout': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    'noise_param_count': (c_int64, []),
    'noise_packed_count': (c_int64, []),
    'noise_pack_weights': (c_int, [c_void_p, c_void_p, c_void_p]),
    'noise_pop_workspace_bytes': (c_size_t, [c_int64]),
    'noise_pop_chunk_members': (c_int, [c_int64, c_int, c_int, c_size_t]),
    'noise_pop_forward_lowrank': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int64,
                                          c_int, c_int, c_float, c_uint32, c_uint32, c_void_p, c_void_p, c_size_t,
                                          c_void_p, c_void_p]),
    'noise_pop_forward_direct': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int64,
                                         c_int, c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_size_t, c_void_p,
                                         c_void_p]),
    'noise_pop_capture': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p,
                                  c_void_p, c_size_t, c_void_p, c_void_p]),
    'noise_dust_errors': (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int64, c_uint32, c_int, c_float,
                                  c_float, c_void_p, c_void_p, c_uint32, c_uint32, c_void_p, c_void_p]),
    'noise_coordinate_differences': (c_int, [c_void_p, c_void_p, c_int64, c_float, c_void_p, c_void_p]),
    'noise_reassemble_workspace_bytes': (c_int64, [c_int, c_int, c_int]),
    'noise_reassemble': (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                 c_void_p, c_size_t, c_void_p, c_void_p]),
    'noise_local_process': (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    'noise_local_baseline': (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    'noise_local_workspace_bytes': (c_int64, [c_int, c_int, c_int]),
    'noise_local_errors': (c_int, [c_void_p, c_void_p, c_int, c_int, c_int64, c_int, c_uint32, c_uint32, c_void_p,
                                   c_void_p, c_size_t, c_void_p, c_void_p]),
    'noise_adamw_dense': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_float,
                                  c_float, c_float, c_int, c_void_p]),
    'noise_anvil_sizes': (c_int, [c_void_p, c_void_p, c_void_p]),
    'noise_anvil_prepare': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float,
                                    c_float, c_float, c_float, c_void_p]),
    'noise_anvil_finish': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float,
                                   c_float, c_float, c_void_p]),
    'noise_fitness_workspace_bytes': (c_size_t, [c_int]),
    'noise_fitness': (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    'noise_update_sum_fe_adamw': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_float, c_uint32,
                                          c_uint32, c_void_p, c_float, c_float, c_float, c_float, c_float, c_int,
                                          c_void_p, c_void_p]),
    'noise_adamw_region': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float,
                                   c_float, c_float, c_float, c_int, c_void_p]),
    'noise_anvil_region_sizes': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    'noise_anvil_region_prepare': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                           c_void_p, c_float, c_float, c_float, c_float, c_void_p]),
    'noise_anvil_region_finish': (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_float, c_float, c_float, c_void_p]),
    'noise_anvil_polar_workspace_bytes': (c_int64, [c_void_p]),
    'noise_anvil_region_polar': (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_void_p,
                                         c_void_p]),
    'noise_sum_fe_partial': (c_int, [c_void_p, c_int, c_int, c_int, c_float, c_uint32, c_uint32, c_void_p, c_void_p,
                                     c_void_p]),
    'noise_fitness_static_max_members': (c_int, []),
    'noise_fitness_static': (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    'noise_launch_count': (c_int64, []),
    'noise_profile_enable': (c_int, [c_int]),
    'noise_profile_read': (c_int, [c_void_p, c_void_p, c_int]),
}


class NoiseError(RuntimeError):
    pass


class NoiseDirect(ctypes.Structure):
    """struct NoiseDirect of include/noise_b200.h."""
    _fields_ = [('entry', ctypes.c_int), ('mask', ctypes.c_uint32), ('site', ctypes.c_uint32 * 5),
                ('sigma', ctypes.c_float), ('x_entry', c_void_p), ('inv0', c_void_p), ('live', c_void_p),
                ('y_entry', c_void_p)]


class NoisePrior(ctypes.Structure):
    """struct NoisePrior of include/noise_b200.h."""
    _fields_ = [('count', ctypes.c_int), ('site', ctypes.c_uint32 * 2), ('d', ctypes.c_int * 2), ('mu', c_void_p * 2)]


class NoiseLocal(ctypes.Structure):
    """struct NoiseLocal of include/noise_b200.h."""
    _fields_ = [('kind', ctypes.c_int), ('layer', ctypes.c_int), ('site', ctypes.c_uint32), ('sigma', ctypes.c_float),
                ('gamma', ctypes.c_float)] + [(n, c_void_p) for n in ('raw', 'q', 'k', 'values', 'gate_logits', 've',
                                                                       'target', 'base')]


class NoiseRegion(ctypes.Structure):
    """struct NoiseRegion of include/noise_b200.h."""
    _fields_ = [('tensor_begin', ctypes.c_int), ('tensor_end', ctypes.c_int), ('base', ctypes.c_int64)]


class NoiseCapture(ctypes.Structure):
    """struct NoiseCapture of include/noise_b200.h."""
    _fields_ = [(n, c_void_p) for n in ('blocks', 'x0', 'inv0', 'y', 'mid', 'hidden', 'final_x', 'logits',
                                         'token_loss')]


_lib = None


def load() -> ctypes.CDLL:
    """Load the library once and attach argument types; raises if it is absent."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise NoiseError(f'{LIB_PATH} is missing: run `python -m noise_b200.build` (or __graft_entry__.build())')
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, args
        _lib = lib
    return _lib


def check(code: int, what: str) -> None:
    if code != NOISE_OK:
        raise NoiseError(f'{what}: {STATUS_NAMES.get(code, code)}')


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
