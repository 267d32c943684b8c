"""Builds libveda_b200.so (the C ABI over the sm_100a kernels) in-tree.

    python -m veda_b200.build [--verbose]     (from veda-on-comfyui_b200/)

Each csrc/*.cu is compiled with nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) into _build/, in parallel, and
linked into veda_b200/libveda_b200.so with the CUDA runtime linked
statically, so the library needs no torch and no libcuda at link time.
Objects are rebuilt when their source or any header is newer.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)                  # veda-on-comfyui_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, 'csrc')
INCLUDE = os.path.join(REPO, 'include')
BUILD = os.path.join(ROOT, '_build')
LIBRARY = os.path.join(PKG, 'libveda_b200.so')

ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-lineinfo', '-std=c++17', '-Xcompiler', '-fPIC',
         '--expt-relaxed-constexpr', '-Xcompiler', '-Wall']


def nvcc() -> str:
    found = shutil.which('nvcc')
    if found:
        return found
    default = os.path.join(os.environ.get('CUDA_HOME', '/usr/local/cuda'),
                           'bin', 'nvcc')
    if os.path.exists(default):
        return default
    raise RuntimeError('nvcc not found: set CUDA_HOME or put nvcc on PATH')


def _headers() -> list[str]:
    return (glob.glob(os.path.join(CSRC, '*.cuh'))
            + glob.glob(os.path.join(INCLUDE, '*.h')))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    mtime = os.path.getmtime(target)
    return any(os.path.getmtime(d) > mtime for d in deps)


def _compile(src: str, verbose: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.basename(src) + '.o')
    if not _stale(obj, [src] + _headers()):
        return obj, ''
    cmd = [nvcc(), *ARCH, *FLAGS, '-I', INCLUDE, '-I', CSRC, '-c', src,
           '-o', obj]
    if verbose:
        cmd[1:1] = ['-Xptxas', '-v']
    run = subprocess.run(cmd, capture_output=True, text=True)
    if run.returncode != 0:
        raise RuntimeError(f'nvcc failed on {src}:\n{run.stdout}{run.stderr}')
    return obj, run.stdout + run.stderr


def build(verbose: bool = False) -> str:
    """Compiles and links the library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, '*.cu')))
    with concurrent.futures.ThreadPoolExecutor(len(sources)) as pool:
        results = list(pool.map(lambda s: _compile(s, verbose), sources))
    objects = [obj for obj, _ in results]
    if verbose:
        for _, log in results:
            if log:
                print(log, file=sys.stderr)
    if _stale(LIBRARY, objects):
        cmd = [nvcc(), *ARCH, '-shared', '-o', LIBRARY, *objects,
               '-cudart', 'static']
        run = subprocess.run(cmd, capture_output=True, text=True)
        if run.returncode != 0:
            raise RuntimeError(f'link failed:\n{run.stdout}{run.stderr}')
    return LIBRARY


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.split('\n')[0])
    parser.add_argument('--verbose', action='store_true',
                        help='print ptxas register / spill reports')
    args = parser.parse_args()
    print(build(args.verbose))


if __name__ == '__main__':
    main()
