"""The C-ABI library on a machine without a GPU: it loads, exports every function that
include/mignon_cuda.h declares, and reports the missing device as an error status (no compute
call is made)."""
import ctypes
import os
import re

import pytest

from mignon_ai_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "mignon_cuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z_0-9]*\s*\*?\s*(mc_[a-z_0-9]+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for n in ("mc_last_error", "mc_version", "mc_gemm_i8_dev", "mc_gemm_f32a_dev", "mc_load_model", "mc_batch_open",
              "mc_prefill", "mc_append", "mc_generate", "mc_generate_dev"):
        assert n in names


def test_library_exports_every_declared_function():
    L = _lib.lib()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, f"declared in include/mignon_cuda.h but not exported: {missing}"


def test_version_and_error_string():
    L = _lib.lib()
    v = L.mc_version()
    assert v >= 100
    assert isinstance(L.mc_last_error(), bytes)


def test_null_arguments_are_rejected_before_any_device_call():
    L = _lib.lib()
    assert L.mc_open(None, None) == 1  # MC_INVALID_ARGUMENT: null output
    assert b"null" in L.mc_last_error()


def test_open_without_a_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = _lib.lib()
    h = ctypes.c_void_p()
    st = L.mc_open(None, ctypes.byref(h))
    assert st != 0
    assert L.mc_last_error()
