"""ctypes binding of libodie_b200.so (the C-ABI in include/odie_b200.h).

The product path has no fallback: if the shared library is missing or was not
built for this tree, every entry point raises instead of computing anything on
the CPU.
"""
import ctypes as C
from functools import lru_cache
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / 'libodie_b200.so'

P, I32, I64, U64, B = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_bool


class HashLevel(C.Structure):
    """odie_hash_level of include/odie_b200.h."""
    _fields_ = [('scale', C.c_float), ('resolution', C.c_int32), ('capacity', C.c_int32),
                ('offset', C.c_int32), ('features', C.c_int32), ('column', C.c_int32), ('hashed', C.c_int32),
                ('cells', C.c_int32)]


SIGNATURES = {
    'odie_error': (C.c_char_p, []),
    'odie_launch_count': (C.c_longlong, []),
    'odie_create': (P, [C.c_char_p]),
    'odie_step': (I32, [P, U64, I32, I32]),
    'odie_step_grads': (I32, [P, U64, I32, I32]),
    'odie_step_stratified': (I32, [P, U64, U64, I32, I32]),
    'odie_stratified_ids': (I32, [U64, U64, I32, I32, I64, P, U64]),
    'odie_wait_probe': (I32, [C.c_uint32, P, U64]),
    'odie_fma_probe': (I64, [I32, P, U64]),
    'odie_step_heads': (I32, [P]),
    'odie_grid_update': (I32, [P]),
    'odie_join': (I32, [P]),
    'odie_profile': (I32, [P, I32]),
    'odie_profile_report': (C.c_char_p, [P]),
    'odie_pointers': (C.c_char_p, [P]),
    'odie_state': (C.c_char_p, [P, I32, I32]),
    'odie_configure': (I32, [P, C.c_char_p]),
    'odie_release_contexts': (None, [P]),
    'odie_pin_contexts': (None, [P]),
    'odie_sync_weights': (I32, [P]),
    'odie_copy': (I32, [U64, U64, U64, U64]),
    'odie_destroy': (None, [P]),
    'odie_decode': (I32, [P, I64, I64, P, P]),
    'odie_query_forward': (I32, [P, I64, P, P, I32, P, P, P, I32, P, P, U64]),
    'odie_query_backward': (I32, [P, I64, P, I32, P, I32, P, P, P, P, I64, U64]),
    'odie_hash_forward': (I32, [P, I64, P, C.POINTER(HashLevel), I32, I32, P, U64]),
    'odie_hash_backward': (I32, [P, I64, P, I32, C.POINTER(HashLevel), I32, P, I64, U64]),
    'score_chunk': (I32, [P, P, I64, I64, I32, I32, I32, I32, P, P, P, B, U64]),
    'selection_init': (I32, [P, I32, I32, P, P, P, P, P, P, P, I32, U64]),
    'selection_chunk': (I32, [P, I32, I32, I32, I32, B, P, P, P, P, P, P, I32, I32, P, P, U64]),
    'odie_tile_topk': (I32, [P, P, I32, I32, I32, I32, P, P, P, P, U64]),
    'odie_router_forward': (I32, [P, I64, I32, P, I32, P, P, P, U64]),
    'odie_router_forward_banded': (I32, [P, P, I64, I32, P, I32, I32, I32, I32, I32, P, P, P, I32, U64]),
    'odie_l2_probe': (I32, [P, I64, I32, I64, P, U64]),
    'odie_plane_index_scratch': (I64, [I32]),
    'odie_allocation_bitmap': (I32, [P, I32, I32, I32, I32, I32, I32, P, U64]),
    'odie_plane_index': (I32, [P, I32, P, P, P, P, P, P, U64]),
    'odie_expert_hash_forward': (I32, [P, I64, P, I64, P, C.POINTER(HashLevel), I32, I32, P, P, U64]),
    'odie_expert_hash_backward': (I32, [P, I64, P, I32, I64, P, C.POINTER(HashLevel), I32, P, P, I64, U64]),
    'odie_tile_topk_noalloc': (I32, [P, P, I32, I32, I32, I32, P, P, P, U64]),
    'odie_topk': (I32, [P, I32, I32, P, P, U64]),
    'odie_procedural_image': (I32, [U64, I32, I32, I32, I32, P, U64]),
    'odie_hashgrid32_create': (P, [C.c_char_p]),
    'odie_hashgrid32_step': (I32, [P, U64, U64, I64, P, I32, U64]),
    'odie_hashgrid32_update': (I32, [P, U64]),
    'odie_hashgrid32_decode': (I32, [P, I64, I64, P, P, U64]),
    'odie_hashgrid32_pointers': (C.c_char_p, [P]),
    'odie_hashgrid32_profile': (I32, [P, I32]),
    'odie_hashgrid32_profile_report': (C.c_char_p, [P]),
    'odie_hashgrid32_destroy': (None, [P]),
}


class LibraryMissing(RuntimeError):
    pass


@lru_cache(maxsize=1)
def library():
    if not LIBRARY.exists():
        raise LibraryMissing(f'{LIBRARY} is missing: run python -m odie_b200.build (or __graft_entry__.build())')
    lib = C.CDLL(str(LIBRARY))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def exported_symbols():
    return list(SIGNATURES)


def error():
    return library().odie_error().decode()


def check(code, what='odie_b200'):
    """Raise on a nonzero status (runtime calls use odie_error, CUDA calls the code)."""
    if code:
        message = error() if code == -1 else f'CUDA error {code}'
        raise RuntimeError(f'{what} failed: {message}')


def ptr(tensor):
    return None if tensor is None else tensor.data_ptr()


def stream_handle(stream=None):
    import torch
    return (stream or torch.cuda.current_stream()).cuda_stream
