"""The oracle's full decode-loop policy (or_sample_policy / or_generate_policy): the reference's
own known answers for SampleRawLogitsAdvanced (internal/generate/sample_test.go:15-45) and the
constraint test (:105-120), and a line-by-line Python statement of sample.go:33-247 on random
cases. CPU only."""
import numpy as np
import pytest

from mignon_ai_b200 import synth
from policy_ref import py_policy


def test_sample_raw_logits_advanced_known_answers(oracle):
    """TestSampleRawLogitsAdvanced (sample_test.go:15-45), all four cases, for many draws."""
    S = oracle.Sampling
    logits = [2.0, 0.5, 5.0, -1.0]
    for u in (0.0, 0.3, 0.77, 0.999999):
        assert oracle.sample_policy(logits, S(0.0, 1.0, 0, 1.0), u=u)[0] == 2
        assert oracle.sample_policy(logits, S(0.8, 1.0, 1, 1.0), u=u)[0] == 2
        assert oracle.sample_policy([-10.0, -10.0, 20.0, -10.0], S(1.0, 1.0, 0, 0.90), u=u)[0] == 2
        assert oracle.sample_policy(logits, S(0.0, 10.0, 0, 1.0), prefix=[2], u=u)[0] != 2


def test_constraint_mask_known_answer(oracle):
    """TestSampleContinuationAppliesConstraint (sample_test.go:105-120): the favourite token 3 is
    not allowed; index 0 wins the argmax among the remaining zeros."""
    logits = [0.0] * 8
    logits[3] = 1.0
    allowed = np.zeros(8, np.int32)
    allowed[3] = -1
    tok, _ = oracle.sample_policy(logits, oracle.Sampling(0.0, 1.0, 0, 1.0), allowed=allowed)
    assert tok == 0


def test_trigram_ban_known_answer(oracle):
    """sample.go:213-227: after 5 6 7 5 6 the pair (5, 6) was followed by 7, so 7 is banned even
    when it has the largest logit."""
    logits = [0.0] * 10
    logits[7] = 3.0
    logits[9] = 1.0
    sp = oracle.Sampling(0.0, 1.0, 0, 1.0, 0, 1)
    assert oracle.sample_policy(logits, sp, gen=[5, 6, 7, 5, 6])[0] == 9
    assert oracle.sample_policy(logits, sp, gen=[5, 6, 7, 5, 8])[0] == 7


@pytest.mark.parametrize("case", range(6))
def test_policy_matches_python_statement(oracle, case):
    rng = np.random.default_rng(100 + case)
    S = oracle.Sampling
    samplings = [
        S(0.0, 1.3, 0, 1.0, 6, 1),    # greedy with penalty and ban
        S(0.8, 1.0, 0, 1.0, 0, 0),    # pure temperature
        S(0.8, 1.0, 0, 0.0, 0, 0),    # truncated branch over the whole vocabulary (top-p 0 is off)
        S(0.7, 1.2, 40, 0.9, 6, 1),   # the reference's benchmark knobs (sample_test.go:47-59)
        S(1.3, 2.0, 0, 0.5, 4, 1),    # nucleus only
        S(0.5, 1.1, 3, 1.0, 0, 0),    # top-k only, whole prefix as window
    ]
    V = [16, 64, 257, 1024, 2048, 100][case]
    for sp in samplings:
        for trial in range(8):
            logits = (rng.standard_normal(V) * (0.02 if trial % 2 else 2.0)).astype(np.float32).astype(np.float64)
            if trial == 3:
                logits[:] = np.round(logits)  # many ties
            prefix = rng.integers(-2, V + 2, size=int(rng.integers(0, 9))).tolist()
            gen = rng.integers(0, min(V, 6), size=int(rng.integers(0, 14))).tolist()
            allowed = None
            if trial == 5:
                allowed = np.where(rng.random(V) < 0.3, -1, 0).astype(np.int32)
                allowed[int(rng.integers(0, V))] = 0
            u = synth.sample_uniform(case, trial)
            want = py_policy(logits, sp, prefix, gen, allowed, u)
            got = oracle.sample_policy(logits, sp, prefix, gen, allowed, u)
            assert got[0] == want[0], (sp.temperature, sp.top_k, sp.top_p, trial)
            assert got[1] == pytest.approx(want[1], rel=1e-12, abs=0.0)


def test_generate_policy_stops_and_lengths(oracle):
    """or_generate_policy ends a session before a stop token and pads with -1; greedy with no
    penalty, ban or constraint equals or_generate_greedy."""
    small = synth.ModelSpec(**{**synth.CONFIGS[1].__dict__, "vocab": 256})
    data = synth.build_model_file(small)
    om = oracle.Model(data)
    n, P, T = 6, 8, 10
    prompts = synth.prompts_uniform_fast(n, P, small.vocab, seed=9)
    lens = np.full(n, P, np.int32)
    lens[2] = 0
    want, wp, _ = om.generate_greedy(prompts, lens, T)
    got, gp, glen, _ = om.generate_policy(prompts, lens, T, oracle.Sampling(0.0, 1.0, 0, 1.0))
    np.testing.assert_array_equal(got, want)
    np.testing.assert_allclose(gp, wp, rtol=1e-6)
    assert glen[2] == 0 and (got[2] == -1).all()
    stop = int(want[0, 3])
    got, _, glen, _ = om.generate_policy(prompts, lens, T, oracle.Sampling(0.0, 1.0, 0, 1.0), stops=[stop])
    first = int(np.nonzero(want[0] == stop)[0][0])
    assert glen[0] == first and (got[0, first:] == -1).all()
    np.testing.assert_array_equal(got[0, :first], want[0, :first])
