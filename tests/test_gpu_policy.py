"""The whole decode-loop policy on the GPU (policy_kernel through mc_sample_rows and
mc_generate_policy) against the oracle's or_sample_policy / or_generate_policy.

On given logits the tokens must equal the oracle's: the kernel's running sums differ from the
reference's left-to-right sums by rounding only, so a token may differ only where the draw lies
within 1e-9 of a bucket edge. Through the model the logits agree to 1e-3 of their maximum, so a
stream may leave the oracle's only at a step within 5e-3 of a decision edge (the rule of the
sampling test in test_gpu_engine.py)."""
import numpy as np
import pytest

from mignon_ai_b200 import quant, synth
from policy_ref import policy_margin, py_policy

pytestmark = pytest.mark.gpu

S = quant.Sampling


def _oracle_sampling(oracle, sp):
    return oracle.Sampling(sp.temperature, sp.rep_penalty, sp.top_k, sp.top_p, sp.rep_window, sp.ban_trigrams)


def test_sample_rows_known_answers():
    """TestSampleRawLogitsAdvanced (internal/generate/sample_test.go:15-45), all four cases, on the
    device, for several draws at once."""
    u = np.array([0.0, 0.3, 0.77, 0.999999])
    logits = np.tile(np.array([2.0, 0.5, 5.0, -1.0], np.float32), (4, 1))
    t, _ = quant.sample_rows(logits, S(0.0, 1.0, 0, 1.0, 0, False), u=u)
    assert (t == 2).all()
    t, p = quant.sample_rows(logits, S(0.8, 1.0, 1, 1.0, 0, False), u=u)
    assert (t == 2).all() and (p == 1.0).all()
    dom = np.tile(np.array([-10.0, -10.0, 20.0, -10.0], np.float32), (4, 1))
    t, _ = quant.sample_rows(dom, S(1.0, 1.0, 0, 0.90, 0, False), u=u)
    assert (t == 2).all()
    t, _ = quant.sample_rows(logits, S(0.0, 10.0, 0, 1.0, 0, False), recent=np.full((4, 1), 2), u=u)
    assert (t != 2).all()


def test_sample_rows_constraint_and_trigram_known_answers():
    """TestSampleContinuationAppliesConstraint (sample_test.go:105-120): the favourite token is
    not allowed and index 0 wins among the zeros; and the 3-gram block (sample.go:213-227)."""
    logits = np.zeros((2, 10), np.float32)
    logits[:, 3] = 1.0
    allowed = np.zeros((2, 10), np.int32)
    allowed[0, 3] = -1
    t, _ = quant.sample_rows(logits, S(0.0, 1.0, 0, 1.0, 0, False), allowed=allowed)
    assert t.tolist() == [0, 3]
    logits[:, 7] = 3.0
    logits[:, 9] = 2.0
    recent = np.array([[5, 6, 7, 5, 6], [5, 6, 7, 5, 8]], np.int32)
    t, _ = quant.sample_rows(logits, S(0.0, 1.0, 0, 1.0, 0, True), recent=recent)
    assert t.tolist() == [9, 7]


CASES = [
    S(0.0, 1.3, 0, 1.0, 6, True),     # argmax with penalty and 3-gram block
    S(0.8, 1.0, 0, 1.0, 0, False),    # pure temperature, draw in index order
    S(0.8, 1.0, 0, 0.0, 0, False),    # truncated branch over the whole vocabulary
    S(0.7, 1.2, 40, 0.9, 6, True),    # the reference's benchmark knobs (sample_test.go:47-59)
    S(1.3, 2.0, 0, 0.5, 4, True),     # nucleus only
    S(0.5, 1.1, 3, 1.0, 0, False),    # top-k only, whole recent list as the window
    S(0.9, 1.0, 1000, 0.95, 0, False),  # the largest top-k that selects its candidates
    S(0.9, 1.0, 1500, 1.0, 0, True),    # a top-k beyond that sorts the whole row
]


@pytest.mark.parametrize("kernel", ["warp", "block"])
@pytest.mark.parametrize("V", [16, 257, 2048, 4096, 16384])
def test_sample_rows_match_oracle(oracle, V, kernel, monkeypatch):
    """Both kernels on the same rows: the warp-per-row kernel takes argmax, the index-order draw
    and top-k up to 64; MC_POLICY_BLOCK=1 sends every launch to the CTA-per-row kernel. Row 3
    ties everywhere (one value: the warp kernel's candidate room overflows and its 64-bit select
    runs), row 5 holds values a few float ulps apart, and the masked rows of the odd cases put
    -1e300 entries below the group-maximum bound."""
    if kernel == "block":
        monkeypatch.setenv("MC_POLICY_BLOCK", "1")
    else:
        monkeypatch.delenv("MC_POLICY_BLOCK", raising=False)
    rng = np.random.default_rng(V)
    n = 48 if V <= 4096 else 12
    for ci, sp in enumerate(CASES):
        scale = np.where(np.arange(n) % 2 == 0, 2.0, 0.02)[:, None]
        logits = (rng.standard_normal((n, V)) * scale).astype(np.float32)
        logits[3] = np.round(logits[3])  # ties
        logits[5] = (1.0 + np.spacing(np.float32(1.0)) * rng.integers(0, 64, V)).astype(np.float32)
        m = 14
        recent = rng.integers(0, min(V, 6), size=(n, m)).astype(np.int32)
        rlen = rng.integers(0, m + 1, size=n).astype(np.int32)
        allowed = np.where(rng.random((n, V)) < 0.2, -1, 0).astype(np.int32)
        allowed[:, 0] = 0
        use_mask = ci % 2 == 1
        got_t, got_p = quant.sample_rows(logits, sp, recent=recent, recent_lens=rlen,
                                         allowed=allowed if use_mask else None, session0=7 * ci, step=V)
        osp = _oracle_sampling(oracle, sp)
        for r in range(n):
            u = synth.sample_uniform(7 * ci + r, V)
            gen = recent[r, :rlen[r]].tolist()
            al = allowed[r] if use_mask else None
            want_t, want_p = oracle.sample_policy(logits[r].astype(np.float64), osp, (), gen, al, u)
            if got_t[r] != want_t:
                m_edge = policy_margin(logits[r], sp, (), gen, al, u)
                assert m_edge < 1e-9, f"V={V} case {ci} row {r}: {got_t[r]} != {want_t} ({m_edge:.3g} from an edge)"
                continue
            assert got_p[r] == pytest.approx(want_p, rel=1e-5), (V, ci, r)


@pytest.mark.parametrize("kernel", ["warp", "block"])
def test_sample_rows_zero_probability_ties(oracle, kernel, monkeypatch):
    """Rows where fewer than k tokens have a non-zero probability: the automaton allows 10 tokens
    (the others get -1e300), or the logits spread so far that most exponentials underflow to 0.
    The k-th probability is then 0 and the top k is completed by the lowest indices among the
    zeros, which the warp kernel's group-maximum bound cannot see (its exact fallback runs)."""
    if kernel == "block":
        monkeypatch.setenv("MC_POLICY_BLOCK", "1")
    else:
        monkeypatch.delenv("MC_POLICY_BLOCK", raising=False)
    rng = np.random.default_rng(77)
    n, V = 16, 2048
    logits = rng.standard_normal((n, V)).astype(np.float32)
    logits[n // 2:] *= 3000.0
    allowed = np.full((n, V), -1, np.int32)
    for r in range(n // 2):
        allowed[r, rng.choice(V, 10, replace=False)] = 0
    allowed[n // 2:] = 0
    for ci, sp in enumerate([S(0.8, 1.0, 40, 1.0, 0, False), S(0.8, 1.2, 40, 0.95, 6, True),
                             S(0.0, 1.0, 0, 1.0, 0, False), S(0.8, 1.0, 0, 1.0, 0, False)]):
        got_t, got_p = quant.sample_rows(logits, sp, allowed=allowed, session0=3 * ci, step=5)
        osp = _oracle_sampling(oracle, sp)
        for r in range(n):
            u = synth.sample_uniform(3 * ci + r, 5)
            want_t, want_p = oracle.sample_policy(logits[r].astype(np.float64), osp, (), [], allowed[r], u)
            if got_t[r] != want_t:
                m_edge = policy_margin(logits[r], sp, (), [], allowed[r], u)
                assert m_edge < 1e-9, f"case {ci} row {r}: {got_t[r]} != {want_t} ({m_edge:.3g} from an edge)"
                continue
            assert got_p[r] == pytest.approx(want_p, rel=1e-5), (ci, r)


def _oracle_cum(logits, temperature, k):
    """The running sum after the k most probable entries as the reference computes it
    (sample.go:119-152): x = logit / T, exponentials of x - max summed in index order, each
    divided by the sum, sorted descending, summed in that order."""
    x = logits.astype(np.float64) * (1.0 / temperature)
    e = np.exp(x - x.max())
    s = float(np.cumsum(e)[-1])
    p = e * (1.0 / s)
    q = p[np.lexsort((np.arange(p.size), -p))]
    cum = 0.0
    for i in range(k):
        cum += float(q[i])
    return cum


@pytest.mark.parametrize("delta", [0.0, 5e-8, -5e-8, 2e-7, -2e-7, 1e-6, -4e-6, 2e-5, -2e-5])
def test_sample_rows_top_p_at_the_sum_bound(oracle, delta, monkeypatch):
    """The warp kernel sums the softmax denominator from exponentials good to 2e-6 (relative) and
    decides a top-p comparison that lies within 8e-6 of its threshold with the exact sum: top-p
    set within 2e-5 of each row's running sum after its third or fifth candidate (inside and
    outside that margin) must cut where the reference cuts, with the same token and probability
    (delta 0, the threshold on the sum itself, may go either way and is skipped)."""
    monkeypatch.delenv("MC_POLICY_BLOCK", raising=False)
    rng = np.random.default_rng(91)
    n, V = 6, 2048
    logits = (rng.standard_normal((n, V)) * 3.0).astype(np.float32)
    for r in range(n):
        kc = 3 if r % 2 == 0 else 5
        top_p = _oracle_cum(logits[r], 0.8, kc) * (1.0 + delta)
        sp = S(0.8, 1.0, 40, top_p, 0, False)
        osp = _oracle_sampling(oracle, sp)
        rows = np.repeat(logits[r:r + 1], 4, axis=0)
        got_t, got_p = quant.sample_rows(rows, sp, session0=11 * r, step=3)
        for j in range(4):
            u = synth.sample_uniform(11 * r + j, 3)
            want_t, want_p = oracle.sample_policy(rows[j].astype(np.float64), osp, (), [], None, u)
            if policy_margin(rows[j], sp, (), [], None, u) < 1e-9:
                continue  # on an edge (delta 0): either cut is the reference's up to rounding
            assert got_t[j] == want_t, (r, j)
            assert got_p[j] == pytest.approx(want_p, rel=1e-6), (r, j)


def test_sample_rows_python_statement_on_one_row():
    """The device's answer on one row equals the plain-Python statement for every case."""
    rng = np.random.default_rng(5)
    logits = (rng.standard_normal((1, 300)) * 1.5).astype(np.float32)
    for sp in CASES:
        u = 0.6180339887
        t, p = quant.sample_rows(logits, sp, recent=np.array([[4, 9, 4, 9, 11]], np.int32), u=[u])
        want = py_policy(logits[0].astype(np.float64), sp, (), [4, 9, 4, 9, 11], None, u)
        assert int(t[0]) == want[0]
        assert float(p[0]) == pytest.approx(want[1], rel=1e-5)


def _dfa(V, rng):
    """A three-state token automaton: state 0 forbids a third of the vocabulary, state 1 another
    third, state 2 nothing; every allowed token moves to the next state (2 stays)."""
    d = np.zeros((3, V), np.int32)
    d[0] = 1
    d[1] = 2
    d[2] = 2
    d[0, rng.random(V) < 0.33] = -1
    d[1, rng.random(V) < 0.33] = -1
    return d


@pytest.mark.parametrize("sp", [S(0.0, 1.3, 0, 1.0, 6, True), S(0.8, 1.2, 40, 0.9, 6, True),
                                S(1.0, 1.5, 0, 0.8, 6, True)])
def test_generate_policy_matches_oracle(oracle, sp):
    """mc_generate_policy on config-2 shapes (4 attention blocks, vocabulary 1024): ragged prompts
    (one empty), the prompt as penalty prefix, a constraint automaton on half of the sessions and
    a stop token; against or_generate_policy with the same draws."""
    base = synth.CONFIGS[2]
    spec = synth.ModelSpec(**{**base.__dict__, "vocab": 1024})
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n, P, steps = 16, 24, 14
    rng = np.random.default_rng(17)
    prompts = synth.prompts_uniform_fast(n, P, spec.vocab, seed=17)
    lens = rng.integers(1, P + 1, size=n).astype(np.int32)
    lens[5] = 0
    dfa = _dfa(spec.vocab, rng)
    start = np.where(np.arange(n) % 2 == 0, 0, -1).astype(np.int32)
    stop = [int(prompts[0, 0])]
    wt, wp, wl, wlog = om.generate_policy(prompts, lens, steps, _oracle_sampling(oracle, sp), penalize_prompt=True,
                                          dfa=dfa, dfa_start=start, session0=3, stops=stop, logits=True)
    b = gm.new_batch(n, 0, P)
    gt, gp, gl = b.generate_policy(prompts, lens, steps, sp, penalize_prompt=True, dfa=dfa, dfa_start=start,
                                   session0=3, stops=stop)
    b.close()
    assert gl[5] == 0 and (gt[5] == -1).all()
    diverged = 0
    for s in range(n):
        diff = np.nonzero(gt[s] != wt[s])[0]
        if diff.size == 0:
            assert gl[s] == wl[s]
            np.testing.assert_allclose(gp[s, :gl[s]], wp[s, :wl[s]], rtol=2e-2, atol=1e-6)
            continue
        t = int(diff[0])
        diverged += 1
        gen = wt[s, :t].tolist()
        state = start[s]
        for tok in gen:
            state = dfa[state, tok] if state >= 0 else -1
        al = dfa[state] if state >= 0 else None
        m = policy_margin(wlog[s, t], sp, prompts[s, :lens[s]].tolist(), gen, al, synth.sample_uniform(3 + s, t))
        assert m < 5e-3, f"session {s} step {t}: {gt[s, t]} != {wt[s, t]}, {m:.3g} from a decision edge"
    assert diverged <= n // 4, diverged
    # the constraint held: no forbidden token was emitted while a session was in states 0 or 1
    for s in range(n):
        state = start[s]
        for tok in gt[s, :gl[s]]:
            if state >= 0:
                assert dfa[state, tok] >= 0, (s, tok, state)
                state = dfa[state, tok]


def test_generate_policy_stops_and_lengths(oracle):
    """Greedy with nothing switched on follows the oracle's greedy stream (equal except from a
    step where the oracle's top-2 gap is below 1e-4); a stop token ends a session before it, and
    its tokens up to there are those of the run without stops."""
    spec = synth.ModelSpec(**{**synth.CONFIGS[1].__dict__, "vocab": 512})
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n, P, steps = 8, 8, 10
    prompts = synth.prompts_uniform_fast(n, P, spec.vocab, seed=23)
    lens = np.full(n, P, np.int32)
    want, _, wlog = om.generate_greedy(prompts, lens, steps, logits=True)
    b = gm.new_batch(n, 0, P)
    plain = S(0.0, 1.0, 0, 1.0, 0, False)
    got, gp, gl = b.generate_policy(prompts, lens, steps, plain)
    assert (gl == steps).all()
    for s in range(n):
        diff = np.nonzero(got[s] != want[s])[0]
        if diff.size:
            t = int(diff[0])
            top2 = np.sort(wlog[s, t].astype(np.float64))[-2:]
            assert top2[1] - top2[0] < 1e-4, f"session {s} step {t}: {got[s, t]} != {want[s, t]}"
    stop = int(got[0, 4])
    got2, _, gl2 = b.generate_policy(prompts, lens, steps, plain, stops=[stop])
    b.close()
    for s in range(n):
        hit = np.nonzero(got[s] == stop)[0]
        first = int(hit[0]) if hit.size else steps
        assert gl2[s] == first and (got2[s, first:] == -1).all()
        np.testing.assert_array_equal(got2[s, :first], got[s, :first])


def test_policy_rejects_bad_automaton():
    from mignon_ai_b200._lib import MignonCudaError
    spec = synth.ModelSpec(**{**synth.CONFIGS[1].__dict__, "vocab": 256})
    gm = quant.Model.decode(synth.build_model_file(spec))
    b = gm.new_batch(2, 0, 4)
    dfa = np.zeros((2, 256), np.int32)
    dfa[1, 7] = 2  # no state 2
    with pytest.raises(MignonCudaError):
        b.generate_policy(np.ones((2, 4), np.int32), np.full(2, 4, np.int32), 3, S(0.8), dfa=dfa,
                          dfa_start=np.zeros(2, np.int32))
    b.close()
