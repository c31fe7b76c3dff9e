"""ctypes binding of ``libleanselect_b200.so`` (the C ABI in ``include/leanselect_b200.h``).

There is no fallback: if the library is missing or cannot be loaded, every
operation raises.  Build it with ``python -m leanselect_b200.build``.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libleanselect_b200.so"

LS_OK = 0
LS_ERR_INVALID_ARGUMENT = 1
LS_ERR_UNSUPPORTED = 2
LS_ERR_ALIGNMENT = 3
LS_ERR_CUDA = 4

LS_DEVERR_TIMEOUT = 0x1
LS_DEVERR_PAGE_INDEX = 0x2
LS_DEVERR_SEQLENS = 0x4

LS_MAX_TOPK = 128
LS_MAX_ATTN_SPLITS = 64

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F32 = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> argument types (all return int), in header order.
SIGNATURES = {
    "ls_fold_weights": [_P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P],
    "ls_compressed_seqlens": [_P, _I32, _I32, _I32, _P, _P, _P],
    "ls_compress_keys": [_P, _P, _I32, _I64, _I32, _I32, _I32, _I32, _P, _P, _I64, _P, _P],
    "ls_compress_keys_dual": [_P, _P, _I32, _I32, _I64, _I32, _I32, _P, _P, _I64, _P, _P, _I64, _P,
                              _P],
    "ls_project_atom_keys": [_P, _I64, _I32, _I32, _P, _I32, _P, _P],
    "ls_project_queries": [_P, _I64, _I32, _I32, _I32, _P, _I32, _P, _P, _P],
    "ls_score_pages": [_P, _P, _P, _P, _P, _I32, _I32, _I64, _I64, _I32, _I32, _I32, _I32, _I32,
                       _I32, _P, _P, _P],
    "ls_score_pages_single": [_P, _P, _P, _I64, _I64, _I32, _I32, _I32, _I32, _I32, _I32, _I32,
                              _P, _P, _P],
    "ls_atom_scores": [_P, _P, _P, _P, _P, _I32, _I32, _I64, _I64, _I32, _I32, _I32, _I32, _I32,
                       _P, _P, _P],
    "ls_select_pages": [_P, _P, _P, _P, _P, _I32, _I32, _I64, _I64, _I32, _I32, _I32, _I32, _I32,
                        _I32, _I32, _I32, _I32, _P, _P, _SZ, _P, _P],
    "ls_select_pages_noalloc": [_P, _P, _P, _P, _P, _I32, _I32, _I64, _I64, _I32, _I32, _I32,
                                _I32, _I32, _I32, _I32, _I32, _I32, _P, _P, _P],
    "ls_compress_keys_f32": [_P, _P, _I32, _I64, _I32, _I32, _I32, _I32, _P, _P, _I64, _P, _P],
    "ls_select_pages_f32": [_P, _P, _P, _P, _P, _P, _I32, _I32, _I64, _I64, _I32, _I32, _I32, _I32,
                            _I32, _I32, _I32, _I32, _I32, _P, _P, _SZ, _P, _P],
    "ls_uniform_select_pages": [_P, _P, _P, _P, _I32, _I32, _I64, _I64, _I32, _I32, _I32, _I32,
                                _I32, _I32, _I32, _I32, _F32, _P, _P, _SZ, _P, _P],
    "ls_select_pages_chunk": [_P, _P, _P, _I64, _I32, _I32, _I64, _I32, _I32, _I32, _I32, _I32,
                              _I32, _I32, _I32, _I32, _P, _P, _SZ, _P, _P],
    "ls_bb_rms_norm": [_P, _P, _I64, _I32, _F32, _P, _P],
    "ls_bb_rope_split": [_P, _P, _P, _F32, _I64, _I32, _I32, _I32, _P, _P, _P, _P],
    "ls_bb_silu_mul": [_P, _I64, _I32, _P, _P],
    "ls_sparse_attn": [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I32, _I32, _I32, _P,
                       _I32, _I32, _F32, _I32, _P, _P, _P, _P],
    "ls_sparse_attn_split": [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I32, _I32, _I32,
                             _P, _I32, _I32, _F32, _I32, _I32, _P, _SZ, _P, _P, _P, _P],
    "ls_sparse_attn_gather_only": [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I32, _I32,
                                   _I32, _P, _I32, _I32, _I32, _P, _P],
    "ls_wait_timeout_probe": [_P, _P, ctypes.c_uint64, _P],
}
STRING_FUNCS = ("ls_status_string", "ls_last_error", "ls_version")
SIZE_FUNCS = {"ls_select_pages_workspace_bytes": [_I64, _I32, _I32],
              "ls_select_pages_f32_workspace_bytes": [_I64, _I64, _I32, _I32],
              "ls_uniform_select_workspace_bytes": [_I64, _I64, _I32, _I32, _I32],
              "ls_sparse_attn_split_workspace_bytes": [_I64, _I32, _I32]}

_lock = threading.Lock()
_lib = None


class LeanSelectError(RuntimeError):
    """A C-ABI call returned an error code or a kernel raised a status bit."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def load(path: os.PathLike | str | None = None) -> ctypes.CDLL:
    """Load the library once (per process) and declare its prototypes."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        target = Path(path) if path is not None else LIB_PATH
        if not target.exists():
            raise RuntimeError(
                f"leanselect_b200 native library not found at {target}; build it with "
                "`python -m leanselect_b200.build` (there is no CPU fallback)")
        lib = ctypes.CDLL(str(target))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        lib.ls_status_string.argtypes = [ctypes.c_int]
        lib.ls_status_string.restype = ctypes.c_char_p
        lib.ls_last_error.argtypes = []
        lib.ls_last_error.restype = ctypes.c_char_p
        lib.ls_version.argtypes = []
        lib.ls_version.restype = ctypes.c_char_p
        for name, argtypes in SIZE_FUNCS.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_size_t
        if path is None:
            _lib = lib
        return lib


def call(name: str, *args) -> None:
    """Invoke a C-ABI entry point and raise :class:`LeanSelectError` on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != LS_OK:
        text = lib.ls_status_string(rc).decode()
        detail = lib.ls_last_error().decode()
        raise LeanSelectError(rc, f"{name} failed with {text}: {detail}")


def version() -> str:
    return load().ls_version().decode()
