"""Continuous batching (mc_sched_*) on the GPU: requests of different prompt lengths and token
limits run through a small pool of slots, admitted as slots free up, and every request's tokens
follow the oracle's sampleContinuation for that request alone (or_generate_policy with the same
draw key), under the parity rule of the policy tests: a stream may leave the oracle's only at a
step within 5e-3 of a decision edge."""
import numpy as np
import pytest

from mignon_ai_b200 import quant, synth
from policy_ref import policy_margin

pytestmark = pytest.mark.gpu

S = quant.Sampling


def _oracle_sampling(oracle, sp):
    return oracle.Sampling(sp.temperature, sp.rep_penalty, sp.top_k, sp.top_p, sp.rep_window, sp.ban_trigrams)


def _requests(n, vocab, max_prompt, max_new, seed):
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, max_prompt + 1, size=n).astype(np.int32)
    lens[3] = 0  # an empty prompt generates nothing
    n_new = rng.integers(1, max_new + 1, size=n).astype(np.int32)
    prompts = synth.prompts_uniform_fast(n, max_prompt, vocab, seed=seed)
    return prompts, lens, n_new


def _check_against_oracle(oracle, om, sp, prompts, lens, n_new, key0, stops, got, penalize):
    n = len(lens)
    steps = int(n_new.max())
    wt, _, wl, wlog = om.generate_policy(prompts, lens, steps, _oracle_sampling(oracle, sp), penalize_prompt=penalize,
                                         session0=key0, stops=stops, logits=True)
    diverged = 0
    for i in range(n):
        want = wt[i, :min(int(wl[i]), int(n_new[i]))]
        toks = got[i]
        m = min(len(toks), len(want))
        diff = np.nonzero(np.asarray(toks[:m]) != want[:m])[0]
        if diff.size == 0:
            assert len(toks) == len(want), (i, len(toks), len(want))
            continue
        t = int(diff[0])
        diverged += 1
        margin = policy_margin(wlog[i, t], sp, prompts[i, :lens[i]].tolist() if penalize else (), want[:t].tolist(),
                               None, synth.sample_uniform(key0 + i, t))
        assert margin < 5e-3, f"request {i} token {t}: {toks[t]} != {want[t]}, {margin:.3g} from a decision edge"
    assert diverged <= n // 4, diverged


@pytest.mark.parametrize("sp", [S(0.0, 1.0, 0, 1.0, 0, False), S(0.8, 1.2, 40, 0.9, 6, True)])
def test_scheduler_matches_oracle(oracle, sp):
    """40 requests through 8 slots of a config-2-shaped model (4 attention blocks, vocabulary
    1024): prompt lengths 0..24, token limits 1..12, one stop token, the prompt as penalty prefix."""
    spec = synth.ModelSpec(**{**synth.CONFIGS[2].__dict__, "vocab": 1024})
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n, P, T, key0 = 40, 24, 12, 1000
    prompts, lens, n_new = _requests(n, spec.vocab, P, T, seed=31)
    stops = [int(prompts[0, 1])]
    penalize = sp.rep_penalty > 1.0
    sched = quant.Scheduler(gm, 8, sp, max_prompt=P, max_new=T, penalize_prompt=penalize, stops=stops)
    ids = [sched.submit(prompts[i, :lens[i]], int(n_new[i]), draw_key=key0 + i) for i in range(n)]
    sched.run(steps_per_poll=3)
    got = [sched.result(r)[0] for r in ids]
    st = sched.stats()
    sched.close()
    assert st["finished"] == n and st["in_flight"] == 0
    assert 2 <= st["prefill_passes"] < n  # slots were refilled, several requests per pass
    assert len(got[3]) == 0
    _check_against_oracle(oracle, om, sp, prompts, lens, n_new, key0, stops, got, penalize)


def test_scheduler_interleaved_submissions(oracle):
    """Requests submitted while others run, with an admission threshold of one free slot: each
    still gets the tokens it would get alone."""
    spec = synth.ModelSpec(**{**synth.CONFIGS[1].__dict__, "vocab": 512})
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n, P, T, key0 = 24, 16, 10, 7
    prompts, lens, n_new = _requests(n, spec.vocab, P, T, seed=37)
    sp = S(0.9, 1.3, 0, 0.95, 6, True)
    sched = quant.Scheduler(gm, 4, sp, max_prompt=P, max_new=T)
    sched.set_admit_min(1)
    ids = []
    for i in range(n):
        ids.append(sched.submit(prompts[i, :lens[i]], int(n_new[i]), draw_key=key0 + i))
        if i % 3 == 2:
            sched.step(2)
    sched.run(steps_per_poll=2)
    got = [sched.result(r)[0] for r in ids]
    st = sched.stats()
    sched.close()
    assert st["finished"] == n and st["tokens"] == sum(len(g) for g in got)
    _check_against_oracle(oracle, om, sp, prompts, lens, n_new, key0, [], got, False)


def test_scheduler_rejects_bad_requests():
    from mignon_ai_b200._lib import MignonCudaError
    spec = synth.ModelSpec(**{**synth.CONFIGS[1].__dict__, "vocab": 256})
    gm = quant.Model.decode(synth.build_model_file(spec))
    sched = quant.Scheduler(gm, 2, S(), max_prompt=8, max_new=4)
    with pytest.raises(MignonCudaError):
        sched.submit([5] * 3, 5)  # above max_new
    with pytest.raises(MignonCudaError):
        sched.submit([5] * 9, 2)  # above max_prompt
    rid = sched.submit([5, 6], 2)
    assert sched.result(rid) is None  # still queued
    sched.run()
    assert len(sched.result(rid)[0]) == 2
    sched.close()


@pytest.mark.parametrize("sp", [S(0.0, 1.0, 0, 1.0, 0, False), S(0.7, 1.0, 8, 1.0, 0, False)])
def test_scheduler_one_token_prompts(oracle, sp):
    """Admission passes of one-token prompts run through the decode kernels (the fused greedy head
    for plain argmax): the per-slot token counts and limits hold there too."""
    spec = synth.ModelSpec(**{**synth.CONFIGS[2].__dict__, "vocab": 512})
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n, T, key0 = 12, 9, 50
    rng = np.random.default_rng(41)
    prompts = rng.integers(5, spec.vocab, size=(n, 1)).astype(np.int32)
    lens = np.ones(n, np.int32)
    n_new = rng.integers(1, T + 1, size=n).astype(np.int32)
    sched = quant.Scheduler(gm, 4, sp, max_prompt=4, max_new=T)
    sched.set_admit_min(1)
    ids = [sched.submit(prompts[i], int(n_new[i]), draw_key=key0 + i) for i in range(n)]
    sched.run(steps_per_poll=2)
    got = [sched.result(r)[0] for r in ids]
    sched.close()
    assert [len(g) for g in got] == n_new.tolist()
    _check_against_oracle(oracle, om, sp, prompts, lens, n_new, key0, [], got, False)
