"""CPU: the C-ABI library loads and exports every symbol include/odie_b200.h declares.

No compute call is made here (there may be no GPU); the GPU tests exercise them.
"""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / 'include' / 'odie_b200.h').read_text()
    return re.findall(r'ODIE_API\s+[\w\s\*]+?\b(\w+)\s*\(', text)


@pytest.fixture(scope='module')
def lib():
    from odie_b200 import builder as build_module
    build_module.build()
    return ctypes.CDLL(str(build_module.LIBRARY))


def test_header_declares_the_reference_boundary():
    names = set(declared_symbols())
    # the reference's runtime (odie/native/runtime.cu:318-331), residual and selection C-ABIs
    for name in ('odie_error', 'odie_create', 'odie_step', 'odie_pointers', 'odie_state', 'odie_configure',
                 'odie_release_contexts', 'odie_sync_weights', 'odie_pin_contexts', 'odie_copy', 'odie_destroy',
                 'score_chunk', 'selection_init', 'selection_chunk'):
        assert name in names, name


def test_library_exports_every_declared_symbol(lib):
    missing = [name for name in declared_symbols() if not hasattr(lib, name)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    from odie_b200 import _lib
    assert set(declared_symbols()) == set(_lib.exported_symbols())


def test_library_is_sm100a_only():
    """The build targets sm_100a exactly (no PTX fallback, no other architecture)."""
    from odie_b200 import builder as build_module
    assert build_module.ARCH == ['-gencode', 'arch=compute_100a,code=sm_100a']


def test_error_string_is_thread_local_and_empty(lib):
    lib.odie_error.restype = ctypes.c_char_p
    assert lib.odie_error() == b''


def test_create_rejects_bad_json_without_gpu(lib):
    """Invalid configuration fails on the host before any device work."""
    lib.odie_create.restype = ctypes.c_void_p
    lib.odie_create.argtypes = [ctypes.c_char_p]
    lib.odie_error.restype = ctypes.c_char_p
    assert lib.odie_create(b'{not json') is None
    assert b'invalid JSON' in lib.odie_error()
