"""The committed fixtures of tests/golden.

reference_kats.json holds the known answers of the reference's own tests (read from their
source); the oracle must reproduce every one. The *.npz fixtures hold the oracle's outputs on small
seeded cases (written by tests/golden/make_golden.py); the oracle must reproduce them exactly, and
the CUDA path must meet the parity gates against them: logits within 1e-3 of their largest
magnitude, greedy streams equal except from a step whose top-2 logit gap is below 1e-4,
log-probabilities within 2e-3 of the largest logit, sampled streams equal except from a step
within 5e-3 of a decision edge."""
import json
import math
import os

import numpy as np
import pytest

from mignon_ai_b200 import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _kats():
    with open(os.path.join(GOLDEN, "reference_kats.json")) as f:
        return json.load(f)


def _load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def _spec(fx):
    return synth.ModelSpec(**{**synth.CONFIGS[int(fx["config"])].__dict__, "vocab": int(fx["vocab"])})


# ---- the reference's known answers, on the oracle (CPU) ---------------------------------------

def test_reference_sampler_known_answers(oracle):
    for case in _kats()["sample_raw_logits_advanced"]["cases"]:
        sp = oracle.Sampling(case["temperature"], case["rep_penalty"], case["top_k"], case["top_p"])
        for u in (0.0, 0.25, 0.5, 0.999):
            tok, _ = oracle.sample_policy(case["logits"], sp, prefix=case["recent"], u=u)
            if "want" in case:
                assert tok == case["want"], case
            else:
                assert tok != case["not"], case


def test_reference_constraint_and_greedy_known_answers(oracle):
    k = _kats()
    c = k["constraint"]
    logits = [0.0] * c["vocab"]
    logits[c["favourite"]] = 1.0
    allowed = np.zeros(c["vocab"], np.int32)
    allowed[c["banned"]] = -1
    assert oracle.sample_policy(logits, oracle.Sampling(0.0, 1.0, 0, 1.0), allowed=allowed)[0] == c["want"]
    g = k["greedy_probability"]
    logits = np.zeros(g["vocab"], np.float32)
    logits[3] = 1.0
    tok, p = oracle.argmax_prob(logits)
    assert tok == 3 and abs(p - g["want"]) <= g["tol"]


def test_reference_kernel_and_layout_known_answers(oracle):
    k = _kats()
    for case in k["dot_int8_shorter_slice"]["cases"]:
        assert oracle.dot_i8_f32(case["x"], case["w"]) == case["want"]
    for init, base, step, want in k["step_dilation"]["cases"]:
        assert oracle.lib().or_step_dilation(init, base, step) == want
        assert synth.step_dilation(init, base, step) == want
    cfg = synth.build_block_configs(2, 3, 2)
    assert [[c.steps, c.dilation_base, c.initial_dilation] for c in cfg] == k["default_two_block_config"]["steps_base_initial"]
    q = k["quantizer_round_trip"]
    d, s = oracle.quantize(q["weights"])
    assert np.max(np.abs(np.float32(q["weights"]) - d.astype(np.float32) * s)) <= q["max_abs_error"]


# ---- the oracle reproduces its frozen outputs (CPU) -------------------------------------------

@pytest.mark.parametrize("name", ["config1", "config2"])
def test_oracle_reproduces_golden_generation(oracle, name):
    fx = _load(name)
    om = oracle.Model(synth.build_model_file(_spec(fx)))
    toks, probs, logits = om.generate_greedy(fx["prompts"], fx["lens"], fx["tokens"].shape[1], logits=True)
    np.testing.assert_array_equal(toks, fx["tokens"])
    np.testing.assert_array_equal(logits, fx["logits"])
    np.testing.assert_array_equal(probs, fx["probs"])


def test_oracle_reproduces_golden_scores_and_policy(oracle):
    fx = _load("config4")
    om = oracle.Model(synth.build_model_file(_spec(fx)))
    np.testing.assert_array_equal(om.score(fx["seqs"]), fx["logprobs"])
    fx = _load("policy")
    om = oracle.Model(synth.build_model_file(_spec(fx)))
    s = fx["sampling"]
    sp = oracle.Sampling(s[0], s[1], int(s[2]), s[3], int(s[4]), int(s[5]))
    toks, _, lens, _ = om.generate_policy(fx["prompts"], fx["lens"], fx["tokens"].shape[1], sp, penalize_prompt=True,
                                          session0=int(fx["session0"]), logits=True)
    np.testing.assert_array_equal(toks, fx["tokens"])
    np.testing.assert_array_equal(lens, fx["out_lens"])


# ---- the CUDA path against the fixtures (GPU) --------------------------------------------------

@pytest.mark.gpu
@pytest.mark.parametrize("name", ["config1", "config2"])
def test_cuda_generation_meets_golden(name):
    from mignon_ai_b200 import quant
    fx = _load(name)
    gm = quant.Model.decode(synth.build_model_file(_spec(fx)))
    n, steps = fx["tokens"].shape
    b = gm.new_batch(n, 0, fx["prompts"].shape[1])
    logits, nxt, _ = b.prefill(fx["prompts"], fx["lens"], want_logits=True)
    want0 = fx["logits"][:, 0]
    assert np.max(np.abs(logits - want0)) <= 1e-3 * np.max(np.abs(want0))
    toks, probs = b.generate(fx["prompts"], fx["lens"], steps)
    b.close()
    gm.close()
    for s in range(n):
        diff = np.nonzero(toks[s] != fx["tokens"][s])[0]
        if diff.size:
            t = int(diff[0])
            top2 = np.sort(fx["logits"][s, t].astype(np.float64))[-2:]
            assert top2[1] - top2[0] < 1e-4, f"session {s} step {t}"
        else:
            np.testing.assert_allclose(probs[s], fx["probs"][s], rtol=1e-3)


@pytest.mark.gpu
def test_cuda_scores_meet_golden():
    from mignon_ai_b200 import quant
    fx = _load("config4")
    gm = quant.Model.decode(synth.build_model_file(_spec(fx)))
    seqs = fx["seqs"]
    b = gm.new_batch(seqs.shape[0], 0, seqs.shape[1])
    got = b.score(seqs, np.full(seqs.shape[0], seqs.shape[1], np.int32))
    b.close()
    gm.close()
    want = fx["logprobs"]
    assert np.max(np.abs(got[:, :want.shape[1]] - want)) <= 2e-3 * max(1.0, np.max(np.abs(want)))


@pytest.mark.gpu
def test_cuda_policy_meets_golden():
    from mignon_ai_b200 import quant
    from policy_ref import policy_margin
    fx = _load("policy")
    gm = quant.Model.decode(synth.build_model_file(_spec(fx)))
    s = fx["sampling"]
    sp = quant.Sampling(s[0], s[1], int(s[2]), s[3], int(s[4]), bool(s[5]))
    n, steps = fx["tokens"].shape
    b = gm.new_batch(n, 0, fx["prompts"].shape[1])
    toks, _, lens = b.generate_policy(fx["prompts"], fx["lens"], steps, sp, penalize_prompt=True,
                                      session0=int(fx["session0"]))
    b.close()
    gm.close()
    for i in range(n):
        diff = np.nonzero(toks[i] != fx["tokens"][i])[0]
        if diff.size == 0:
            continue
        t = int(diff[0])
        m = policy_margin(fx["logits"][i, t], sp, fx["prompts"][i, :fx["lens"][i]].tolist(),
                          fx["tokens"][i, :t].tolist(), None, synth.sample_uniform(int(fx["session0"]) + i, t))
        assert m < 5e-3, f"session {i} step {t}: {m:.3g} from a decision edge"
