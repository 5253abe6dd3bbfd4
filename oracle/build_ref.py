"""Compile the reference's own CUDA kernels for sm_100a into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  The reference ODIE tree keeps the hot-path kernels
in a few self-contained source files that build without its CMake/TCNN
runtime, so they are compiled here, from the files where they lie, into a GPU
oracle that travels to the GPU box with the repository snapshot:

  odie/packed_kernels.cu + odie/packed_bindings.cpp -> oracle/_ref/odie_ref_query*.so
      (torch extension: forward/backward of the packed-plane query)
  odie/residual_cuda.cu                            -> oracle/_ref/libref_residual.so
  odie/native/selection_cuda.cu                    -> oracle/_ref/libref_selection.so

Build flags follow the reference's own recipes (odie/model.py:121-134,
odie/gpu_residual.py:38-40, odie/selection_cuda.py:14-16) with the arch set to
sm_100a.  odie/native/runtime.cu is NOT buildable here: it needs the absent
tiny-cuda-nn static libraries and headers.

Nothing is copied into the repository: the sources are read in place and only
build outputs land in oracle/_ref/ (git-ignored).  Does nothing when the
reference tree is absent (the GPU box uses the prebuilt files).
"""
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / '_ref'


def reference_root():
    """The reference ODIE tree: $ODIE_REFERENCE, else a `reference` directory beside this repository."""
    configured = os.environ.get('ODIE_REFERENCE')
    return Path(configured) if configured else HERE.parent.parent / 'reference'


REFERENCE = reference_root()
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']


def nvcc():
    cuda = os.environ.get('CUDA_HOME', '/usr/local/cuda')
    return str(Path(cuda) / 'bin' / 'nvcc')


def build_shared(source, target, extra):
    if target.exists() and target.stat().st_mtime >= source.stat().st_mtime:
        return
    command = [nvcc(), '-shared', '-O3', *extra, *ARCH, '-Xcompiler', '-fPIC', str(source), '-o', str(target)]
    subprocess.run(command, check=True)


def build_query():
    from torch.utils.cpp_extension import load
    sources = [REFERENCE / 'odie' / 'packed_bindings.cpp', REFERENCE / 'odie' / 'packed_kernels.cu']
    build = OUT / 'query'
    build.mkdir(parents=True, exist_ok=True)
    load(name='odie_ref_query', sources=[str(s) for s in sources], build_directory=str(build),
         extra_cflags=['-O3'], extra_cuda_cflags=['-O3', '--expt-relaxed-constexpr', '-lineinfo', *ARCH],
         verbose=False)


def main():
    if not (REFERENCE / 'odie').is_dir():
        print('reference tree absent; using prebuilt oracle/_ref', file=sys.stderr)
        return 0
    OUT.mkdir(parents=True, exist_ok=True)
    build_shared(REFERENCE / 'odie' / 'residual_cuda.cu', OUT / 'libref_residual.so', ['--fmad=false', '--ftz=false'])
    build_shared(REFERENCE / 'odie' / 'native' / 'selection_cuda.cu', OUT / 'libref_selection.so', ['--fmad=false'])
    os.environ.setdefault('TORCH_CUDA_ARCH_LIST', '10.0')
    build_query()
    return 0


if __name__ == '__main__':
    sys.exit(main())
