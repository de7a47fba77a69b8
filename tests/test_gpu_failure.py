"""The failure path of the kernels' bounded waits, without a GPU fault: a kernel waits on a barrier
that nothing completes, its wait gives up after its 2 s limit, records the device error word and
returns; the call reports MC_DEVICE_TIMEOUT with the device's message, and the device keeps
working (a generation right after it matches one before it)."""
import ctypes

import numpy as np
import pytest

from mignon_ai_b200 import _lib, quant, synth

pytestmark = pytest.mark.gpu

MC_DEVICE_TIMEOUT = 5


def test_bounded_wait_reports_timeout_and_device_stays_usable():
    spec = synth.ModelSpec(**{**synth.CONFIGS[1].__dict__, "vocab": 256})
    gm = quant.Model.decode(synth.build_model_file(spec))
    prompts = synth.prompts_uniform_fast(4, 8, spec.vocab, seed=3)
    lens = np.full(4, 8, np.int32)
    b = gm.new_batch(4, 0, 8)
    before, _ = b.generate(prompts, lens, 5)
    L = _lib.lib()
    L.mc_selftest_wait_timeout.restype = ctypes.c_int
    L.mc_selftest_wait_timeout.argtypes = [ctypes.c_int]
    st = L.mc_selftest_wait_timeout(0)
    assert st == MC_DEVICE_TIMEOUT, (st, L.mc_last_error())
    assert b"gave up" in L.mc_last_error()
    after, _ = b.generate(prompts, lens, 5)
    np.testing.assert_array_equal(before, after)
    b.close()
    gm.close()
