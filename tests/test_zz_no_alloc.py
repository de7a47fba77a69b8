"""The allocation-free GEMM entry point (mc_gemm_f32a_noalloc_dev) against the allocating one.

Some programs that drive this library cannot allocate GPU memory when they call it: a host
runtime that may only hand over buffers it registered in advance, or a service whose GPU memory is
budgeted once at start-up. The
allocation-free entry point serves them by keeping its one scratch buffer (the per-row maxima
the activation slicing needs) in a fixed device array inside the library. This test checks, on
two calls in a row with different inputs, that its results equal the allocating entry point's
(which takes the scratch buffer from the caller): both run the same kernels, so the outputs
must agree bit for bit. The file sorts last so that a run that stops at the first failure has
already run every other test; it also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from mignon_ai_b200 import _lib

pytestmark = pytest.mark.gpu


def _declare():
    L = _lib.lib()
    vp = ctypes.c_void_p
    L.mc_gemm_f32a_noalloc_dev.restype = ctypes.c_int
    L.mc_gemm_f32a_noalloc_dev.argtypes = [vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, vp, vp, vp]
    return L


def test_noalloc_gemm_matches_allocating_gemm_twice():
    import torch
    L = _declare()
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(11)
    m, n, k = 384, 256, 384
    w = torch.from_numpy(rng.integers(-127, 128, (n, k)).astype(np.int8)).to(dev)
    bias = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(dev)
    scale = 0.0123
    for call in range(2):
        # different activations on each call, so a stale scratch value would show
        x = torch.from_numpy((rng.standard_normal((m, k)) * (1 + 3 * call)).astype(np.float32)).to(dev)
        y_ref = torch.zeros((m, n), dtype=torch.float32, device=dev)
        scratch = torch.zeros(m, dtype=torch.float32, device=dev)
        _lib.check(L.mc_gemm_f32a_dev(_lib.ptr(x), _lib.ptr(w), m, n, k, scale, _lib.ptr(bias), _lib.ptr(y_ref), None,
                                      _lib.ptr(scratch), None))
        y = torch.full((m, n), float("nan"), dtype=torch.float32, device=dev)
        _lib.check(L.mc_gemm_f32a_noalloc_dev(_lib.ptr(x), _lib.ptr(w), m, n, k, scale, _lib.ptr(bias), _lib.ptr(y),
                                              None))
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref), f"call {call}: max |diff| {float((y - y_ref).abs().max())}"


def test_noalloc_gemm_rejects_rows_above_its_fixed_maximum():
    import torch
    L = _declare()
    dev = torch.device("cuda:0")
    m, n, k = 65537, 128, 128
    x = torch.zeros((m, k), dtype=torch.float32, device=dev)
    w = torch.zeros((n, k), dtype=torch.int8, device=dev)
    y = torch.zeros((m, n), dtype=torch.float32, device=dev)
    status = L.mc_gemm_f32a_noalloc_dev(_lib.ptr(x), _lib.ptr(w), m, n, k, 1.0, None, _lib.ptr(y), None)
    torch.cuda.synchronize()
    assert status == 1  # MC_INVALID_ARGUMENT
    assert b"65536" in L.mc_last_error()


def test_noalloc_gemm_on_two_devices():
    """The set-up of the first call (the array's address, the kernels' shared-memory attribute)
    is per device: a first call on device 0 must not leave device 1 without it."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    L = _declare()
    rng = np.random.default_rng(12)
    m, n, k = 256, 256, 512
    xs = (rng.standard_normal((m, k)) * 2).astype(np.float32)
    ws = rng.integers(-127, 128, (n, k)).astype(np.int8)
    for d in (0, 1):
        dev = torch.device("cuda", d)
        with torch.cuda.device(d):
            x, w = torch.from_numpy(xs).to(dev), torch.from_numpy(ws).to(dev)
            y_ref = torch.zeros((m, n), dtype=torch.float32, device=dev)
            scratch = torch.zeros(m, dtype=torch.float32, device=dev)
            _lib.check(L.mc_gemm_f32a_dev(_lib.ptr(x), _lib.ptr(w), m, n, k, 0.5, None, _lib.ptr(y_ref), None,
                                          _lib.ptr(scratch), None))
            y = torch.full((m, n), float("nan"), dtype=torch.float32, device=dev)
            _lib.check(L.mc_gemm_f32a_noalloc_dev(_lib.ptr(x), _lib.ptr(w), m, n, k, 0.5, None, _lib.ptr(y), None))
            torch.cuda.synchronize(dev)
            assert torch.equal(y, y_ref), f"device {d}"


def test_noalloc_gemm_rejects_bad_shapes_before_any_cuda_call():
    import torch
    L = _declare()
    dev = torch.device("cuda:0")
    x = torch.zeros((64, 128), dtype=torch.float32, device=dev)
    w = torch.zeros((100, 128), dtype=torch.int8, device=dev)
    y = torch.zeros((64, 100), dtype=torch.float32, device=dev)
    status = L.mc_gemm_f32a_noalloc_dev(_lib.ptr(x), _lib.ptr(w), 64, 100, 128, 1.0, None, _lib.ptr(y), None)
    assert status == 1  # MC_INVALID_ARGUMENT: N % 128 != 0
