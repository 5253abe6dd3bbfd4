"""odie_b200: B200-native (sm_100a) hot path of ODIE.

Routed multiresolution 2-D grid encoding (packed planes, dense and hashed
grids), fused tensor-core MLP heads, sparse Adam, live residual scoring and
exact greedy / tile top-k selection, behind the reference's C-ABI and Python
module API.  The compute lives in libodie_b200.so (built by odie_b200.build).
"""
from . import _lib  # noqa: F401

__all__ = ['build', 'library']


def build(force=False):
    from .builder import build as _build
    return _build(force=force)


def library():
    return _lib.library()
