"""Loads libmignoncuda.so (built in-tree by ``mignon_ai_b200.build``) and declares its C-ABI.

There is no fallback: if the library cannot be built or loaded, every call raises.
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

_lib = None

c_i8p = ctypes.POINTER(ctypes.c_int8)
c_i32p = ctypes.POINTER(ctypes.c_int32)
c_f32p = ctypes.POINTER(ctypes.c_float)
c_vp = ctypes.c_void_p


class MignonCudaError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"mignoncuda status {status}: {message}")
        self.status = status


def _declare(L):
    i = ctypes.c_int
    L.mc_last_error.restype = ctypes.c_char_p
    L.mc_version.restype = i
    L.mc_gemm_i8_dev.restype = i
    L.mc_gemm_i8_dev.argtypes = [c_vp, c_vp, i, i, i, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]
    L.mc_gemm_f32a_dev.restype = i
    L.mc_gemm_f32a_dev.argtypes = [c_vp, c_vp, i, i, i, ctypes.c_float, c_vp, c_vp, c_vp, c_vp, c_vp]
    L.mc_gemm_i8.restype = i
    L.mc_gemm_i8.argtypes = [i, c_vp, c_vp, i, i, i, c_vp, c_vp, c_vp, c_vp, c_vp]
    for name, argtypes in EXTRA_SIGNATURES.items():
        f = getattr(L, name)
        f.restype = i
        f.argtypes = argtypes


# Signatures of the engine entry points (filled in by the modules that use them).
EXTRA_SIGNATURES: dict = {}


def register(signatures: dict):
    """Adds C-ABI signatures; applies them at once if the library is already loaded."""
    EXTRA_SIGNATURES.update(signatures)
    if _lib is not None:
        for name, argtypes in signatures.items():
            f = getattr(_lib, name)
            f.restype = ctypes.c_int
            f.argtypes = argtypes


def lib(build_if_missing: bool = True):
    """The loaded library; builds it first when the sources are newer (needs nvcc)."""
    global _lib
    if _lib is None:
        if build_if_missing and _build.needs_build():
            _build.build()
        if not os.path.exists(_build.LIB):
            raise MignonCudaError(-1, f"{_build.LIB} is missing and could not be built")
        L = ctypes.CDLL(_build.LIB)
        _declare(L)
        _lib = L
    return _lib


def check(status: int):
    if status != 0:
        raise MignonCudaError(status, lib().mc_last_error().decode(errors="replace"))


def ptr(a):
    """Data pointer of a numpy array or torch tensor (None for None)."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return ctypes.c_void_p(a.data_ptr())
    return a.ctypes.data_as(ctypes.c_void_p)
