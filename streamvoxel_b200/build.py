"""Build libsvx.so (the sm_100a kernels behind include/svx.h) in-tree with nvcc.

    python -m streamvoxel_b200.build [--force]

Objects go to streamvoxel_b200/_build/, the library to streamvoxel_b200/libsvx.so. nvcc cross-compiles for
sm_100a without a GPU. Rebuilds only when a source or header is newer than the library.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

PACKAGE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PACKAGE)
CSRC = os.path.join(PACKAGE, 'csrc')
BUILD = os.path.join(PACKAGE, '_build')
LIBRARY = os.path.join(PACKAGE, 'libsvx.so')
SOURCES = ['capi.cu', 'ease.cu', 'gemm.cu', 'attention.cu', 'embed_norm.cu', 'engine.cu']
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-std=c++17', '-lineinfo', '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden',
         '-I' + os.path.join(ROOT, 'include')]


def nvcc():
    path = shutil.which('nvcc') or '/usr/local/cuda/bin/nvcc'
    if not os.path.exists(path):
        raise RuntimeError('nvcc not found: libsvx.so needs the CUDA 12.9 toolkit to build')
    return path


def _inputs():
    names = [os.path.join(CSRC, n) for n in os.listdir(CSRC) if n.endswith(('.cu', '.cuh', '.h'))]
    return names + [os.path.join(ROOT, 'include', 'svx.h'), os.path.abspath(__file__)]


def stale():
    if not os.path.exists(LIBRARY):
        return True
    built = os.path.getmtime(LIBRARY)
    return any(os.path.getmtime(p) > built for p in _inputs())


def _compile(source):
    obj = os.path.join(BUILD, source.replace('.cu', '.o'))
    cmd = [nvcc(), *ARCH, *FLAGS, '-c', os.path.join(CSRC, source), '-o', obj]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode:
        raise RuntimeError(f'nvcc failed on {source}:\n{result.stderr}')
    return obj


def build(force=False, verbose=False):
    """Compile every kernel for sm_100a and link libsvx.so. Returns the library path."""
    if not force and not stale():
        return LIBRARY
    os.makedirs(BUILD, exist_ok=True)
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 1)) as pool:
        objects = list(pool.map(_compile, SOURCES))
    tmp = LIBRARY + '.tmp'
    cmd = [nvcc(), *ARCH, '-shared', '-Xcompiler', '-fPIC', *objects, '-o', tmp, '-lcudart']
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode:
        raise RuntimeError(f'link failed:\n{result.stderr}')
    os.replace(tmp, LIBRARY)
    if verbose:
        print(f'built {LIBRARY}')
    return LIBRARY


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument('--force', action='store_true')
    args = parser.parse_args()
    build(force=args.force, verbose=True)


if __name__ == '__main__':
    sys.exit(main())
