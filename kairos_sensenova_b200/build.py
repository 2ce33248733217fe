"""Build ``libkb200.so`` (the C-ABI extension) in-tree with nvcc for sm_100a.

``python -m kairos_sensenova_b200.build`` compiles every ``csrc/*.cu`` whose
object is older than its sources and links them into
``kairos_sensenova_b200/libkb200.so``.  No torch headers are used: the
library is plain CUDA C++ behind ``include/kb200.h``.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / 'csrc'
OBJ = PKG / '_build'
LIB = PKG / 'libkb200.so'
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
FLAGS = ['-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '-std=c++17', '-lineinfo',
         '-Xcompiler', '-fPIC', '-I', str(ROOT / 'include'), '-I', str(CSRC)]


def _deps():
    return [p for p in CSRC.iterdir() if p.suffix in ('.cuh', '.h')] + [ROOT / 'include' / 'kb200.h']


def build(verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob('*.cu'))
    dep_mtime = max(p.stat().st_mtime for p in _deps())

    def compile_one(src: Path):
        obj = OBJ / (src.stem + '.o')
        if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, dep_mtime):
            return obj
        cmd = [NVCC, *FLAGS, '-c', str(src), '-o', str(obj)]
        if verbose:
            print(' '.join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f'nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}')
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, srcs))
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [NVCC, '-gencode', 'arch=compute_100a,code=sm_100a', '-shared', '-o', str(LIB),
               *map(str, objs), '-lcudart']
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f'link failed:\n{r.stdout}\n{r.stderr}')
    return LIB


if __name__ == '__main__':
    print(build(verbose='-v' in sys.argv))
