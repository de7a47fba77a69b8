"""Pins the oracle's kernels to the reference's own kernel tests and known answers.

Restates internal/kernels/int8_test.go, accuracy_test.go, internal/ca/layout_test.go,
internal/quant/tensor_test.go and the selection tests of internal/generate.
"""
import math

import numpy as np
import pytest

from mignon_ai_b200 import synth


@pytest.fixture(params=[1, 0], ids=["avx2", "pure"])
def avx2_mode(request, oracle):
    prev = oracle.lib().or_get_avx2()
    oracle.lib().or_set_avx2(request.param)
    yield request.param
    oracle.lib().or_set_avx2(prev)


def test_dot_int8_matches_float64_reference(oracle, avx2_mode):
    """TestDotInt8F32MatchesReference (int8_test.go:15-38): n = 0..100, extreme weights."""
    rng = np.random.default_rng(1)
    for n in range(101):
        x = rng.standard_normal(n).astype(np.float32)
        w = rng.integers(-128, 128, n).astype(np.int8)
        if n > 0:
            w[0], w[n - 1] = -128, 127
        want = float(np.dot(x.astype(np.float64), w.astype(np.float64)))
        mag = float(np.sum(np.abs(x.astype(np.float64) * w)))
        got = oracle.dot_i8_f32(x, w)
        assert abs(got - want) <= 1e-5 * mag + 1e-6, (n, got, want)


def test_dot_int8_uses_shorter_slice(oracle, avx2_mode):
    """TestDotInt8F32UsesShorterSlice (int8_test.go:41-50): known answers 6 and 3."""
    x = np.arange(1, 10, dtype=np.float32)
    assert oracle.dot_i8_f32(x, np.ones(3, np.int8)) == 6.0
    assert oracle.dot_i8_f32(x[:2], np.ones(10, np.int8)) == 3.0


def test_matvec_int8(oracle, avx2_mode):
    """TestMatVecInt8 (int8_test.go:53-77): rows, stride, scale and bias, tolerance 1e-4."""
    rows, cols, stride = 5, 37, 40
    rng = np.random.default_rng(2)
    w = rng.integers(-128, 128, rows * stride).astype(np.int8)
    x = rng.standard_normal(cols).astype(np.float32)
    bias = np.array([0.5, -1, 2, 0, 3], np.float32)
    y = oracle.matvec_i8(w, rows, stride, 0.01, x, bias)
    for r in range(rows):
        want = bias[r] + 0.01 * np.dot(w[r * stride:r * stride + cols].astype(np.float64), x.astype(np.float64))
        assert abs(y[r] - want) <= 1e-4


def test_intrinsics_match_scalar_statement_of_assembly(oracle):
    """The AVX2-intrinsic kernels and the scalar statement of the same assembly order agree bit
    for bit, so the oracle's order does not depend on the compiler."""
    if not oracle.lib().or_get_avx2():
        pytest.skip("oracle built without AVX2")
    import ctypes
    L = oracle.lib()
    rng = np.random.default_rng(7)
    for n in list(range(0, 70)) + [127, 128, 129, 384, 1152]:
        x = rng.standard_normal(n).astype(np.float32)
        y = rng.standard_normal(n).astype(np.float32)
        w = rng.integers(-127, 128, n).astype(np.int8)
        fp = x.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        wp = w.ctypes.data_as(ctypes.POINTER(ctypes.c_int8))
        yp = y.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        a, b = L.or_dot_i8_f32(fp, wp, n), L.or_dot_i8_f32_scalar_order(fp, wp, n)
        assert np.float32(a).tobytes() == np.float32(b).tobytes(), n
        a, b = L.or_dot_f32(fp, yp, n), L.or_dot_f32_scalar_order(fp, yp, n)
        assert np.float32(a).tobytes() == np.float32(b).tobytes(), n


def test_simd_and_pure_dot_f32_agree(oracle):
    """TestSIMDPureGoVsASMEquivalence (accuracy_test.go:36-60): DotF32 within 1e-4."""
    rng = np.random.default_rng(1337)
    L = oracle.lib()
    for n in [0, 1, 2, 3, 5, 7, 8, 9, 15, 16, 17, 23, 31, 32, 33, 47, 64, 65]:
        x = rng.standard_normal(n).astype(np.float32)
        y = rng.standard_normal(n).astype(np.float32)
        L.or_set_avx2(1)
        a = oracle.dot_f32(x, y)
        L.or_set_avx2(0)
        b = oracle.dot_f32(x, y)
        L.or_set_avx2(1)
        assert abs(a - b) <= 1e-4


def test_fast_exp_accuracy(oracle, avx2_mode):
    """TestExpAndSigmoidAccuracy (accuracy_test.go:10-33): relative error <= 1e-4."""
    xs = np.array([-20, -15, -10, -5, -2.5, -1, -0.5, 0, 0.5, 1, 2.5, 5, 10, 15, 20], np.float32)
    out = np.zeros_like(xs)
    import ctypes
    oracle.lib().or_vec_exp_f32(out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                xs.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), xs.size)
    for x, got in zip(xs, out):
        want = np.float32(math.exp(float(x)))
        assert abs(float(got) - float(want)) / float(want) <= 1e-4, (x, got, want)
        scalar = oracle.lib().or_fast_exp_f32(float(x))
        assert abs(scalar - float(want)) / float(want) <= 1e-4


def test_sigmoid_clamped(oracle):
    """sigmoidClamped (stream.go:128-136) saturates beyond |x| > 15."""
    s = oracle.lib().or_sigmoid_clamped
    assert s(15.5) == 1.0 and s(-15.5) == 0.0
    assert abs(s(0.0) - 0.5) == 0.0
    assert abs(s(2.0) - 1 / (1 + math.exp(-2))) < 1e-7


def test_step_dilation_known_answers(oracle):
    """TestStepDilation (internal/ca/layout_test.go:41-50)."""
    cases = [(1, 2, 0, 1), (1, 2, 3, 8), (1, 2, 10, 32), (4, 2, 1, 8), (37, 2, 0, 32)]
    for ini, base, step, want in cases:
        assert oracle.lib().or_step_dilation(ini, base, step) == want
        assert synth.step_dilation(ini, base, step) == want


def test_block_configs():
    """BuildBlockConfigs (ca/model.go:33-59): configs 1-3 keep dilation 1 (one step per block);
    config 4 (6 blocks x 2 steps, base 2) gets [1,2],[2,4],[4,8],[8,16],[16,32],[32,32]."""
    for b in synth.build_block_configs(8, 1, 2):
        assert (b.steps, b.initial_dilation) == (1, 1)
    dil = [[synth.step_dilation(b.initial_dilation, b.dilation_base, s) for s in range(b.steps)]
           for b in synth.build_block_configs(6, 2, 2)]
    assert dil == [[1, 2], [2, 4], [4, 8], [8, 16], [16, 32], [32, 32]]
    two = synth.build_block_configs(2, 3, 2)
    assert [(b.steps, b.initial_dilation) for b in two] == [(3, 1), (3, 4)]


def test_quantizer_round_trip(oracle):
    """TestQuantizeFloat32 (internal/quant/tensor_test.go:7-22): error <= 0.05."""
    w = np.array([-1.5, -0.75, 0.0, 0.33, 1.25, 2.0], np.float32)
    for data, scale in (synth.quantize_tensor(w), oracle.quantize(w)):
        deq = synth.dequantize_tensor(data, scale)
        assert np.all(np.abs(w - deq) <= 0.05)


def test_quantizer_python_matches_c(oracle):
    """The package's quantizer and the oracle's agree bit for bit, ties included."""
    rng = np.random.default_rng(5)
    for w in (rng.standard_normal(10000).astype(np.float32) * 0.02,
              np.array([0.5, -0.5, 1.5, 127.0, -127.0, 63.5, 0.0], np.float32),
              np.zeros(7, np.float32)):
        a, sa = synth.quantize_tensor(w)
        b, sb = oracle.quantize(w)
        assert np.float32(sa) == np.float32(sb)
        assert np.array_equal(a, b)


def test_argmax_prob_known_answer(oracle):
    """TestGreedyContinuationStopsAndReportsProbabilities (greedy_test.go:9-22): one logit of 1
    among zeros has probability e/(e+V-1); ties go to the first index (greedy.go:92-95)."""
    V = 8
    logits = np.zeros(V, np.float32)
    logits[3] = 1
    best, p = oracle.argmax_prob(logits)
    assert best == 3 and abs(p - math.e / (math.e + V - 1)) <= 1e-12
    best, _ = oracle.argmax_prob(np.array([0.5, 2, 2, 1], np.float32))
    assert best == 1


def test_sampler_known_answers(oracle):
    """TestSampleRawLogitsAdvanced (sample_test.go:15-45) cases without repetition penalty."""
    logits = np.array([2.0, 0.5, 5.0, -1.0], np.float32)
    assert oracle.sample_topk(logits, 0.0, 0, 0.3) == 2
    for u in (0.0, 0.5, 0.999):
        assert oracle.sample_topk(logits, 0.8, 1, u) == 2
        assert oracle.sample_topk(np.array([-10, -10, 20, -10], np.float32), 1.0, 0, u) == 2


def test_log_prob_normalised(oracle):
    """logProb (eval/suite.go:201-209) is a log-softmax: probabilities sum to one."""
    rng = np.random.default_rng(3)
    l = rng.standard_normal(50).astype(np.float32)
    s = sum(math.exp(oracle.log_prob(l, i)) for i in range(50))
    assert abs(s - 1.0) < 1e-12


def test_philox_known_answers(oracle):
    """Philox4x32-10 known-answer vectors of Random123 (kat_vectors)."""
    kat = [((0, 0, 0, 0), (0, 0), (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
           ((0xffffffff,) * 4, (0xffffffff, 0xffffffff), (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
           ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
            (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1))]
    for ctr, key, want in kat:
        assert tuple(oracle.philox(ctr, key)) == want
        got = synth.philox4x32(np.array([ctr], np.uint64), key[0], key[1])[0]
        assert tuple(int(v) for v in got) == want
    for s, t in [(0, 0), (5, 7), (65535, 100)]:
        assert oracle.lib().or_sample_uniform(s, t) == synth.sample_uniform(s, t)
