"""Build libpq8.so in-tree with nvcc for sm_100a (B200).

    python -m parakeet_cuda_b200.build [--force] [--verbose]

The shared library is written next to this file so that it travels with the
source tree. nvcc cross-compiles without a GPU. A rebuild happens when any
source under ``csrc/`` or ``include/pq8.h`` is newer than the library.
"""
from __future__ import annotations

import argparse
import os
from pathlib import Path
import shutil
import subprocess
import sys

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / 'csrc'
INCLUDE = ROOT / 'include'
LIB = PKG / 'libpq8.so'

ARCH_FLAGS = ['-gencode', 'arch=compute_100a,code=sm_100a']
COMMON_FLAGS = ['-O3', '-std=c++17', '-lineinfo', '--expt-relaxed-constexpr', '-Xcompiler', '-fPIC',
                '-Xcompiler', '-fvisibility=hidden']


def nvcc_path() -> str:
    for cand in (os.environ.get('PQ8_NVCC'), shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError('nvcc not found; set PQ8_NVCC')


def sources():
    return sorted(CSRC.glob('*.cu')) + sorted(CSRC.glob('*.cpp'))


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob('*.cuh')) + [INCLUDE / 'pq8.h']
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False, extra=()) -> Path:
    if not force and not stale():
        return LIB
    cmd = [nvcc_path(), *ARCH_FLAGS, *COMMON_FLAGS, '-I', str(INCLUDE), '-I', str(CSRC), '-shared',
           *extra, '-o', str(LIB) + '.tmp', *map(str, sources()), '-lcublas']
    if verbose:
        print(' '.join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f'nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}')
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, file=sys.stderr)
    os.replace(str(LIB) + '.tmp', LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--force', action='store_true')
    ap.add_argument('--verbose', action='store_true')
    ap.add_argument('--ptxas-info', action='store_true', help='print registers / spills / smem per kernel')
    a = ap.parse_args()
    extra = ['-Xptxas', '-v'] if a.ptxas_info else []
    print(build(force=a.force or a.ptxas_info, verbose=a.verbose or a.ptxas_info, extra=extra))


if __name__ == '__main__':
    main()
