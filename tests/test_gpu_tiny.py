"""Whole-job greedy generation of small models without attention (tiny_generate_kernel: one CTA per
session runs the prompt and every decode step in one launch, the blocks' int8 weights in shared
memory, the digit-plane dot products on dp4a).

* config 1 exactly (its benchmark workload: 64 sessions, 32-token prompts, 64 tokens) and ragged
  prompts (one empty, one of a single token, two longer than the window) against the oracle: the
  streams equal except from a step where the oracle's top-2 gap is below 1e-4, the probabilities
  within 1e-4 relative on equal streams;
* the same job through the batched kernels (MC_TINY_OFF=1) gives the same tokens except at such
  near-ties;
* afterwards the sessions continue exactly as after the batched job: the logits of further
  appends agree with those of a batch that ran the job on the batched kernels.
"""
import numpy as np
import pytest

from mignon_ai_b200 import quant, synth

from test_gpu_engine import check_logits, compare_streams

pytestmark = pytest.mark.gpu


def _spec(**over):
    return synth.ModelSpec(**{**synth.CONFIGS[1].__dict__, **over})


def _check_probs(gp, wp, gt, wt):
    for s in range(gt.shape[0]):
        eq = np.nonzero(gt[s] != wt[s])[0]
        k = int(eq[0]) if eq.size else gt.shape[1]
        if k:
            np.testing.assert_allclose(gp[s, :k], wp[s, :k], rtol=1e-4)


@pytest.mark.parametrize("case", ["config1", "ragged", "three blocks"])
def test_tiny_generate_matches_oracle(oracle, monkeypatch, case):
    monkeypatch.delenv("MC_TINY_OFF", raising=False)
    spec = _spec() if case != "three blocks" else _spec(blocks=3, steps=2, state=32, hidden=96, vocab=700)
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n, plen, n_new = (64, 32, 64) if case == "config1" else (40, 40, 24)
    prompts = synth.prompts_uniform_fast(n, plen, spec.vocab, seed=11)
    lens = np.full(n, plen, np.int32)
    if case == "ragged":
        lens = synth.prompt_lengths(n, 1, plen, seed=11)
        lens[3] = 1
        lens[5] = 0
    wt, wp, wl = om.generate_greedy(prompts, lens, n_new, logits=True)
    b = gm.new_batch(n, 0, plen)
    gt, gp = b.generate(prompts, lens, n_new)
    b.close()
    gm.close()
    act = lens > 0
    compare_streams(gt[act], wt[act], wl[act])
    _check_probs(gp[act], wp[act], gt[act], wt[act])


def test_tiny_and_batched_jobs_agree_and_sessions_continue(monkeypatch):
    """The whole-job kernel and the batched kernels on one job (config 1, ragged prompts), then
    three appends of the same tokens on both batches: every logit within the engine's 1e-3 bar."""
    spec = _spec()
    gm = quant.Model.decode(synth.build_model_file(spec))
    n, plen, n_new = 48, 32, 20
    prompts = synth.prompts_uniform_fast(n, plen, spec.vocab, seed=12)
    lens = synth.prompt_lengths(n, 1, plen, seed=12)
    out = {}
    for label, off in (("tiny", False), ("batched", True)):
        if off:
            monkeypatch.setenv("MC_TINY_OFF", "1")
        else:
            monkeypatch.delenv("MC_TINY_OFF", raising=False)
        b = gm.new_batch(n, 0, plen)
        t, p = b.generate(prompts, lens, n_new)
        follow = []
        nxt = t[:, -1].copy()
        for _ in range(3):
            logits, nxt2, _ = b.append(nxt, want_logits=True)
            follow.append(logits.copy())
            nxt = nxt2
        b.close()
        out[label] = (t, p, follow)
    monkeypatch.delenv("MC_TINY_OFF", raising=False)
    tt, tp, tf = out["tiny"]
    bt, bp, bf = out["batched"]
    same = np.all(tt == bt, axis=1)
    assert same.mean() > 0.9, f"only {same.sum()} of {n} streams equal"
    np.testing.assert_allclose(tp[same], bp[same], rtol=1e-4)
    for k in range(3):
        for s in np.nonzero(same)[0]:
            check_logits(tf[k][s], bf[k][s], f"append {k} session {s}")
    gm.close()
