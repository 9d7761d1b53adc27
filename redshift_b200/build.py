"""Build ``build/libqvelox.so`` (sm_100a) from ``redshift_b200/csrc``.

The library keeps the reference's file name and location relative to the
repository root (``build/libqvelox.so``, cristianku/redshift Makefile:10-13),
so ``qvelox/runtime.py``'s default loader path finds it when the reference's
Python package sits beside this checkout.

    python -m redshift_b200.build          # incremental
    python -m redshift_b200.build --force  # rebuild everything
"""
import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / 'redshift_b200' / 'csrc'
BUILD = ROOT / 'build'
LIBRARY = BUILD / 'libqvelox.so'
SOURCES = ['status.cu', 'attention.cu', 'delta.cu', 'gdn_chunk.cu', 'delta_prefill.cu', 'prefill.cu', 'projection.cu', 'copy.cu',
           'runtime.cu', 'noalloc.cu']
HEADERS = ['common.cuh', 'hotpath.h']

NVCC_FLAGS = [
    '-gencode', 'arch=compute_100a,code=sm_100a',
    '-O3', '-std=c++17', '-lineinfo', '-rdc=true',
    '-Xcompiler', '-fPIC,-Wall,-Wextra,-Wno-unused-parameter',
    '--expt-relaxed-constexpr',
]


def nvcc():
    cuda = os.environ.get('CUDA_HOME', '/usr/local/cuda')
    path = Path(cuda) / 'bin' / 'nvcc'
    return str(path) if path.exists() else (shutil.which('nvcc') or 'nvcc')


def _stale(target, deps):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force=False, verbose=False, extra_flags=()):
    """Compile every CUDA source for sm_100a and link the shared library."""
    BUILD.mkdir(exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [ROOT / 'include' / 'runtime.h']
    objects = []
    for src in SOURCES:
        obj = BUILD / (Path(src).stem + '.o')
        objects.append(obj)
        if force or _stale(obj, [CSRC / src] + headers):
            cmd = [nvcc(), *NVCC_FLAGS, *extra_flags, '-I', str(ROOT / 'include'), '-c', str(CSRC / src), '-o', str(obj)]
            if verbose:
                print(' '.join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIBRARY, objects):
        cmd = [nvcc(), '-gencode', 'arch=compute_100a,code=sm_100a', '-rdc=true', '-shared',
               *map(str, objects), '-o', str(LIBRARY)]
        if verbose:
            print(' '.join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIBRARY


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument('--force', action='store_true')
    ap.add_argument('--verbose', '-v', action='store_true')
    ap.add_argument('--ptxas-info', action='store_true', help='print register / smem usage')
    args = ap.parse_args(argv)
    extra = ['-Xptxas', '-v'] if args.ptxas_info else []
    path = build(force=args.force or args.ptxas_info, verbose=args.verbose, extra_flags=extra)
    print(path)


if __name__ == '__main__':
    sys.exit(main())
