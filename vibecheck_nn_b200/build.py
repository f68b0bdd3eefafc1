"""Build libvcb.so in-tree with nvcc for sm_100a.

    python -m vibecheck_nn_b200.build [--force] [-v]

Compiles every ``csrc/*.cu`` into one shared library next to this file
(``vibecheck_nn_b200/libvcb.so``), exporting the C ABI of ``include/vcb.h``.
The CUDA runtime is linked statically, so the library only needs the driver.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, 'csrc')
INCLUDE = os.path.join(ROOT, 'include')
LIB_PATH = os.path.join(HERE, 'libvcb.so')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-lineinfo', '-std=c++17', '-Xptxas', '-v', '-shared',
         '-Xcompiler', '-fPIC', '-Xcompiler', '-O2']


def nvcc_path():
    for cand in (shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError('nvcc not found')


def sources():
    return sorted(glob.glob(os.path.join(CSRC, '*.cu')))


def _stale():
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = sources() + glob.glob(os.path.join(CSRC, '*.cuh')) + \
        glob.glob(os.path.join(INCLUDE, '*.h'))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False):
    """Compile libvcb.so if any source is newer than it.  Returns its path."""
    if not force and not _stale():
        return LIB_PATH
    tmp = LIB_PATH + '.tmp'
    cmd = [nvcc_path()] + ARCH + FLAGS + ['-I', INCLUDE, '-I', CSRC, '-o', tmp] + sources()
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError('nvcc failed building libvcb.so')
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == '__main__':
    build(force='--force' in sys.argv, verbose='-v' in sys.argv)
    print(LIB_PATH)
