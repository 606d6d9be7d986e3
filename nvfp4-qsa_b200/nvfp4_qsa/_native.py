"""ctypes binding of the C ABI in ``include/nvfp4_qsa.h``.

This is the only place Python touches the native library.  There is no CPU
fallback: if the library is missing or fails to load, every entry point raises
``RuntimeError``.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int32, c_int64, c_size_t, c_void_p, POINTER

from ._build import library_path

OK = 0
_STATUS_EXC = {
    1: ValueError,          # NVQSA_ERR_NULL_POINTER
    2: ValueError,          # NVQSA_ERR_BAD_SHAPE
    3: NotImplementedError,  # NVQSA_ERR_HEAD_DIM
    4: ValueError,          # NVQSA_ERR_MISALIGNED
    5: ValueError,          # NVQSA_ERR_WORKSPACE
    6: NotImplementedError,  # NVQSA_ERR_UNSUPPORTED
    7: RuntimeError,        # NVQSA_ERR_LAUNCH
    8: RuntimeError,        # NVQSA_ERR_CUDA
    9: ValueError,          # NVQSA_ERR_SCRATCH_LIMIT
}

_P = c_void_p
_I64 = c_int64
_I32 = c_int32
_F = c_float

# name -> (restype, argtypes)
_SIGNATURES = {
    "nvqsa_status_string": (ctypes.c_char_p, [c_int]),
    "nvqsa_abi_version": (c_int, []),
    "nvqsa_read_error_flags": (c_int, [POINTER(ctypes.c_uint32), c_int]),
    "nvqsa_set_stamp_buffer": (c_int, [_P]),
    "nvqsa_topk_indices": (c_int, [_P, _I64, _P, _I64, _I64, _I32, _P, _I64, _P]),
    "nvqsa_write_cache": (c_int, [
        _P, _I64, _I64,
        _P, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I32, _I32,
        _I64, _I64,
        _F, _F, _P]),
    "nvqsa_norm_rope_write_cache": (c_int, [
        _P, _I64, _I64,
        _P, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I32, _I32,
        _I64, _I64,
        _F, _F,
        _P, _F, _F,
        _P, _P, _I64, _I64,
        _I32, _I32,
        _P, _I64, _I64, _P]),
    "nvqsa_kv_proj_write_cache": (c_int, [
        _P, _I64, _I64, _I32,
        _P, _P, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I32, _I32,
        _I64, _I64, _F, _F,
        _P, _F, _F,
        _P, _P, _I64, _I64,
        _I32, _I32,
        _P, _I64, _I64,
        _P, _I64, _I64, _P]),
    "nvqsa_sparse_attention_workspace_size": (c_int, [_I64, _I32, _I32, _I32, _I64, POINTER(c_size_t)]),
    "nvqsa_sparse_attention": (c_int, [
        _P, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _I64, _I64, _I32,
        _F, _F,
        _P, _I64,
        _P, _I64, _I64,
        _P,
        _P, _I64, _I64,
        _I64, _I32, _I32,
        _P, c_size_t, _P]),
    "nvqsa_sparse_attention_grouped": (c_int, [
        _P, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _I64, _I64, _I32,
        _F, _F,
        _P, _I64,
        _P, _I64, _I64,
        _P,
        _P, _I64, _I64,
        _I64, _I32, _I32, _I32,
        _P, c_size_t, _P]),
    "nvqsa_sparse_attention_fp8": (c_int, [
        _P, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _I64, _I64, _I32, _F, _F,
        _P, _I64,
        _P, _I64, _I64,
        _P,
        _P, _I64, _I64,
        _I64, _I32, _I32,
        _P, c_size_t, _P]),
    "nvqsa_sparse_attention_bf16": (c_int, [
        _P, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _I64, _I64, _I32,
        _P, _I64,
        _P, _I64, _I64,
        _P,
        _P, _I64, _I64,
        _I64, _I32, _I32,
        _P, c_size_t, _P]),
    "nvqsa_sparse_attention_bf16_workspace_size": (c_int, [_I64, _I32, _I32, _I32, _I64, POINTER(c_size_t)]),
    "nvqsa_sparse_attention_partial": (c_int, [
        _P, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _I64, _I64, _I32,
        _F, _F,
        _P, _I64,
        _P, _I64, _I64,
        _P,
        _P, _P,
        _I64, _I32, _I32,
        _P, c_size_t, _P]),
    "nvqsa_sparse_attention_noalloc": (c_int, [
        _P, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _I64, _I64, _I32,
        _F, _F,
        _P, _I64,
        _P, _I64, _I64,
        _P,
        _P, _I64, _I64,
        _I64, _I32, _I32,
        _P]),
    "nvqsa_split_kv_exchange_bytes": (c_int, [_I64, _I32, _I32, _I32, POINTER(c_size_t)]),
    "nvqsa_exchange_alloc": (c_int, [c_size_t, POINTER(_P)]),
    "nvqsa_exchange_free": (c_int, [_P]),
    "nvqsa_ipc_get_handle": (c_int, [_P, _P]),
    "nvqsa_ipc_open_handle": (c_int, [_P, POINTER(_P)]),
    "nvqsa_ipc_close_handle": (c_int, [_P]),
    "nvqsa_sparse_attention_split_kv": (c_int, [
        _P, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _P, _I64, _I64, _I64,
        _I64, _I64, _I32,
        _F, _F,
        _P, _I64,
        _P, _I64, _I64,
        _P,
        _P, _I64, _I64,
        _I64, _I32, _I32,
        _P, c_size_t,
        _P, _I32, _I32, _I32, _P]),
    "nvqsa_merge_partials": (c_int, [_P, _P, _I32, _P, _I64, _I64, _I64, _I32, _I32, _P]),
    "nvqsa_merge_partials_strided": (c_int, [_P, _I64, _P, _I64, _I32, _P, _I64, _I64, _I64, _I32, _I32, _P]),
    "nvqsa_encode_rows": (c_int, [_P, _I64, _I64, _I32, _P, _P, _P, _P, _P, _P]),
    "nvqsa_decode_rows": (c_int, [_P, _P, _I64, _I64, _I32, _P, _P, _P]),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES)

_lib = None


def load():
    """Load (once) and return the native library; raises RuntimeError if absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.exists():
        raise RuntimeError(
            f"NVFP4 QSA CUDA library not built ({path}); run `python -m nvfp4_qsa._build` "
            "or __graft_entry__.build(). There is no CPU fallback.")
    lib = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def status_text(status: int) -> str:
    return load().nvqsa_status_string(int(status)).decode()


def read_error_flags(clear: bool = True) -> int:
    """Device error flags of the current device (bit 0: a bounded barrier wait ran out; bit 1: a split-KV
    peer's slot did not arrive in time)."""
    flags = ctypes.c_uint32(0)
    check(load().nvqsa_read_error_flags(ctypes.byref(flags), 1 if clear else 0), "nvqsa_read_error_flags")
    return int(flags.value)


def check(status: int, what: str) -> None:
    """Raise the Python exception mapped to a non-zero ABI status."""
    if status != OK:
        exc = _STATUS_EXC.get(int(status), RuntimeError)
        raise exc(f"{what}: {status_text(status)} (status {int(status)})")
