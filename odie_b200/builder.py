"""Build the sm_100a shared library libodie_b200.so in-tree with nvcc.

The library is the product's compute path: every CUDA kernel plus the C-ABI
declared in include/odie_b200.h.  It is built next to this file so that it
travels with the repository snapshot; nothing is installed elsewhere.
"""
import os
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
SOURCES = ['encode.cu', 'step.cu', 'mlp_tc.cu', 'router.cu', 'probe.cu', 'layout.cu', 'residual.cu', 'selection.cu',
           'synth.cu', 'hashgrid32.cu', 'runtime.cu']
LIBRARY = PACKAGE / 'libodie_b200.so'
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-std=c++17', '-lineinfo', '--expt-relaxed-constexpr', '-Xcompiler', '-fPIC',
         '-Xcompiler', '-fvisibility=hidden', '-diag-suppress', '177']


def nvcc():
    return str(Path(os.environ.get('CUDA_HOME', '/usr/local/cuda')) / 'bin' / 'nvcc')


def stale():
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    inputs = list((PACKAGE / 'csrc').glob('*')) + [ROOT / 'include' / 'odie_b200.h', Path(__file__)]
    return any(p.stat().st_mtime > built for p in inputs)


def build(force=False, verbose=False):
    if not force and not stale():
        return LIBRARY
    build_dir = PACKAGE / '_build'
    build_dir.mkdir(exist_ok=True)
    objects = []
    include = ['-I', str(PACKAGE / 'csrc'), '-I', str(ROOT / 'include')]
    for source in SOURCES:
        obj = build_dir / (Path(source).stem + '.o')
        command = [nvcc(), *FLAGS, *ARCH, *include, '-c', str(PACKAGE / 'csrc' / source), '-o', str(obj)]
        if verbose:
            print(' '.join(command), file=sys.stderr)
        subprocess.run(command, check=True)
        objects.append(str(obj))
    tmp = LIBRARY.with_suffix('.so.tmp')
    subprocess.run([nvcc(), '-shared', *ARCH, *objects, '-o', str(tmp), '-lcudart'], check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose=True))
