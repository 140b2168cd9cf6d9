"""Build the in-tree CUDA library `noise_b200/libnoise_b200.so` for sm_100a with nvcc.

The library is a plain C-ABI shared object (no torch headers): every `.cu` under `csrc/` is compiled
for `sm_100a` and linked with the static CUDA runtime. The build is incremental on source mtimes.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / 'csrc'
INCLUDE = HERE.parent / 'include'
LIB = HERE / 'libnoise_b200.so'
OBJ = HERE.parent / '_build'

NVCC_FLAGS = [
    '-gencode', 'arch=compute_100a,code=sm_100a',
    '-O3', '-std=c++17', '-lineinfo', '--expt-relaxed-constexpr',
    '-Xcompiler', '-fPIC,-O2', f'-I{INCLUDE}', f'-I{CSRC}',
]


def nvcc() -> str:
    for cand in (os.environ.get('NVCC'), '/usr/local/cuda/bin/nvcc', 'nvcc'):
        if cand and (Path(cand).exists() or cand == 'nvcc'):
            return cand
    raise RuntimeError('nvcc not found')


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, jobs: int = 8) -> Path:
    sources = sorted(CSRC.glob('*.cu'))
    headers = sorted(CSRC.glob('*.cuh')) + sorted(INCLUDE.glob('*.h'))
    OBJ.mkdir(exist_ok=True)
    objects, procs = [], []
    for src in sources:
        obj = OBJ / (src.stem + '.o')
        objects.append(obj)
        if _stale(obj, [src] + headers):
            cmd = [nvcc(), *NVCC_FLAGS, '-c', str(src), '-o', str(obj)]
            if verbose:
                print(' '.join(cmd), flush=True)
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
            if len(procs) >= jobs:
                _drain(procs)
    _drain(procs)
    if _stale(LIB, objects):
        cmd = [nvcc(), '-gencode', 'arch=compute_100a,code=sm_100a', '-shared', '-cudart', 'static',
               '-o', str(LIB), *map(str, objects)]
        if verbose:
            print(' '.join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def _drain(procs):
    failed = []
    while procs:
        src, p = procs.pop(0)
        out, _ = p.communicate()
        if p.returncode != 0:
            failed.append((src, out.decode(errors='replace')))
    if failed:
        msg = '\n'.join(f'--- {s.name}\n{o}' for s, o in failed)
        raise RuntimeError(f'nvcc failed:\n{msg}')


if __name__ == '__main__':
    print(build(verbose='-v' in sys.argv))
