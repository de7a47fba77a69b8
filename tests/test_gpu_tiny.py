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
  appends agree with those of a batch that ran the job on the batched kernels;
* appends (mc_append, the Go provider's Session.Append on a batch of one) of such models run
  through the same kernel, one launch per token carrying the session state in from memory: a
  config-1 session against the oracle session, and several sessions against the batched kernels.
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


def test_tiny_session_appends_match_oracle(oracle, monkeypatch):
    """The reference's session shape on config 1: prefill 32 tokens, then 60 appends (past the
    64-token window), every logit row against the oracle session."""
    monkeypatch.delenv("MC_TINY_OFF", raising=False)
    spec = _spec()
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    tokens = synth.prompts_uniform_fast(1, 92, spec.vocab, seed=21)[0]
    os_, gs = om.new_session(64), gm.new_session(64)
    check_logits(gs.prefill(tokens[:32]), os_.prefill(tokens[:32]), "prefill")
    for i, t in enumerate(tokens[32:]):
        check_logits(gs.append(int(t)), os_.append(int(t)), f"append {i}")
    gs.close()
    gm.close()


@pytest.mark.parametrize("n", [1, 7])
def test_tiny_appends_match_batched(monkeypatch, n):
    """The same prefill, then 24 appends of the same tokens, on the whole-job kernel and on the
    batched kernels (MC_TINY_OFF=1): logits within the engine's 1e-3 bar, next tokens equal
    except at near-ties, probabilities within 1e-4 on equal tokens; one session has an empty
    prompt and appends nothing."""
    spec = _spec()
    gm = quant.Model.decode(synth.build_model_file(spec))
    prompts = synth.prompts_uniform_fast(n, 20, spec.vocab, seed=23)
    lens = synth.prompt_lengths(n, 1, 20, seed=23)
    if n > 1:
        lens[2] = 0
    feed = synth.prompts_uniform_fast(24, n, spec.vocab, seed=24)
    out = {}
    for label, off in (("tiny", False), ("batched", True)):
        if off:
            monkeypatch.setenv("MC_TINY_OFF", "1")
        else:
            monkeypatch.delenv("MC_TINY_OFF", raising=False)
        b = gm.new_batch(n, 0, 20)
        b.prefill(prompts, lens)
        rows = []
        for k in range(24):
            logits, nxt, prob = b.append(feed[k], want_logits=True)
            rows.append((logits.copy(), nxt.copy(), prob.copy()))
        b.close()
        out[label] = rows
    monkeypatch.delenv("MC_TINY_OFF", raising=False)
    for k in range(24):
        (tl, tn, tp), (bl, bn, bp) = out["tiny"][k], out["batched"][k]
        for s in range(n):
            if lens[s] == 0:
                continue
            check_logits(tl[s], bl[s], f"append {k} session {s}")
            top = np.sort(bl[s])[-2:]
            if tn[s] != bn[s]:
                assert top[1] - top[0] < 1e-4, f"append {k} session {s}: {tn[s]} != {bn[s]}"
            else:
                np.testing.assert_allclose(tp[s], bp[s], rtol=1e-4)
    gm.close()

