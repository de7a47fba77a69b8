"""The benchmark configurations at their own shapes, against the CPU oracle.

* config 4 at its real sequence length (128 tokens: the prefill attention's span passes the
  64-token window, dh = 48) through mc_score;
* config 3 at its real vocabulary (4096: 32 head chunks, top-k 40 merged over the splits) with
  per-session token limits (mc_generate_limits), ragged prompts and sampling at T = 0.8;
* sliding attention windows (window < span) through the fast prefill kernel and the staged decode
  kernel at head widths 32, 48 and 64;
* prefills that run in several passes over the sessions (a batch whose scratch is smaller than
  the prefill) give bit-identical results to a single pass.

Bars as in test_gpu_engine: logits within 1e-3 * max|logit|, log-probabilities within 2e-3 *
max|logit|, greedy streams equal except after a top-2 gap below 1e-4, sampled streams equal except
at a draw within 5e-3 of a CDF bucket edge.
"""
import numpy as np
import pytest

from mignon_ai_b200 import quant, synth

from test_gpu_engine import _cdf_margin, check_logits, compare_streams, run_steps

pytestmark = pytest.mark.gpu


def test_score_config4_full_length(oracle):
    """Config 4 exactly (D 192, H 512, 6 blocks x 2 rule steps, dilations to 32, 4 heads of 48,
    window 64, vocabulary 2048) on 128-token sequences: every next-token log-probability."""
    spec = synth.CONFIGS[4]
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n, L = 6, 128
    seqs = synth.prompts_uniform_fast(n, L, spec.vocab, seed=4)
    want = om.score(seqs)
    b = gm.new_batch(n, 0, L)
    got = b.score(seqs, np.full(n, L, np.int32))
    scale = max(float(np.max(np.abs(om.call(seqs[s])))) for s in range(2))
    err = float(np.max(np.abs(got - want)))
    assert err <= 2e-3 * scale, f"max |dlogprob| {err:.3g} > {2e-3 * scale:.3g}"
    b.close()
    gm.close()


def test_config3_sampled_limits_full_vocab(oracle):
    """Config 3 exactly (D 384, H 1024, 8 attention blocks of 6 x 64, vocabulary 4096), its
    workload's sampling (T 0.8, top-k 40, Philox keyed by the session index) with ragged prompts
    of 16..64 tokens and a token limit per session. Each session's tokens up to its limit are the
    oracle's sampled stream (cut at the limit), then -1."""
    spec = synth.CONFIGS[3]
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n, T, K = 12, 0.8, 40
    lens = synth.prompt_lengths(n, 16, 64, seed=3)
    prompts = synth.prompts_uniform_fast(n, 64, spec.vocab, seed=3)
    limits = (1 + np.arange(n) * 7 % 20).astype(np.int32)  # 1..20 tokens
    n_max = int(limits.max())
    wt, wl = om.generate_sample(prompts, lens, n_max, T, K, session0=0, logits=True)
    b = gm.new_batch(n, 0, 64, top_k=K)
    gt, _, glen = b.generate_limits(prompts, lens, limits, temperature=T)
    b.close()
    gm.close()
    assert np.array_equal(glen, limits)
    diverged = 0
    for s in range(n):
        k = int(limits[s])
        assert np.all(gt[s, k:] == -1)
        diff = np.nonzero(gt[s, :k] != wt[s, :k])[0]
        if diff.size == 0:
            continue
        t = int(diff[0])
        diverged += 1
        m = _cdf_margin(wl[s, t], T, K, synth.sample_uniform(s, t))
        assert m < 5e-3, f"session {s} step {t}: {gt[s, t]} != {wt[s, t]} with the draw {m:.3g} from a bucket edge"
    assert diverged <= n // 4, diverged


@pytest.mark.parametrize("levels", [5, 1], ids=["five levels", "one level"])
def test_sampling_ties_at_the_bound(oracle, levels):
    """Logits that tie in blocks of hundreds: a model whose tied embedding is zero, so every logit
    is its head bias, here (v mod levels). More than 128 entries then reach the select's bound, so
    it takes its exact radix select over the whole row. The top 40 are the lowest indices of the
    top level, and every sampled stream equals the oracle's (T 0.8, vocabulary 4096)."""
    spec = synth.ModelSpec(vocab=4096, state=128, hidden=256, blocks=1, steps=1, attn_heads=4, attn_window=64)
    qm = synth.build_model(spec)
    qm.embed = synth.QTensor(np.zeros_like(qm.embed.data), qm.embed.scale)
    qm.head_b = (np.arange(spec.vocab) % levels).astype(np.float32)
    data = synth.encode_model(qm)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n, n_new, T, K = 24, 6, 0.8, 40
    prompts = synth.prompts_uniform_fast(n, 16, spec.vocab, seed=8)
    lens = np.full(n, 16, np.int32)
    wt, wl = om.generate_sample(prompts, lens, n_new, T, K, session0=0, logits=True)
    b = gm.new_batch(n, 0, 16, top_k=K)
    gt, _ = b.generate(prompts, lens, n_new, temperature=T)
    b.close()
    gm.close()
    top = levels - 1
    assert np.all(gt % levels == top), "a token outside the top level"
    for s in range(n):
        diff = np.nonzero(gt[s] != wt[s])[0]
        if diff.size == 0:
            continue
        t = int(diff[0])
        m = _cdf_margin(wl[s, t], T, K, synth.sample_uniform(s, t))
        assert m < 5e-3, f"session {s} step {t}: {gt[s, t]} != {wt[s, t]} with the draw {m:.3g} from a bucket edge"


WINDOWED = [("dh32 window 16", 128, 4, 16), ("dh48 window 24", 192, 4, 24), ("dh64 window 20", 128, 2, 20)]


@pytest.mark.parametrize("case", WINDOWED, ids=[c[0] for c in WINDOWED])
def test_sliding_window_attention_matches_oracle(oracle, case):
    """Attention windows shorter than the span: 40-token prompts (the prefill kernel's window
    start inside the segment) and 30 greedy appends (the staged decode kernel reading a ring
    whose window has slid), logits at every step against the oracle."""
    name, D, heads, window = case
    spec = synth.ModelSpec(vocab=512, state=D, hidden=2 * D, blocks=2, steps=1, attn_heads=heads, attn_window=window)
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n, plen, n_new = 20, 40, 30
    prompts = synth.prompts_uniform_fast(n, plen, spec.vocab, seed=31)
    lens = np.full(n, plen, np.int32)
    lens[3] = 9  # shorter than the window
    wt, _, wl = om.generate_greedy(prompts, lens, n_new, logits=True)
    gt, _, gl = run_steps(gm, prompts, lens, n_new)
    for t in range(n_new):
        for s in range(n):
            if np.array_equal(gt[s, :t], wt[s, :t]):
                check_logits(gl[s, t], wl[s, t], f"{name} session {s} step {t}")
    compare_streams(gt, wt, wl)
    gm.close()


@pytest.mark.parametrize("vocab", [512, 2048])
def test_prefill_passes_match_one_pass(monkeypatch, vocab):
    """A batch whose prefill needs more scratch than MC_PREFILL_SCRATCH_MB allows runs each prefill
    in passes over contiguous sessions (layers, head and selection per pass). The kernels are the
    same, so greedy and sampled generation, prefill logits and scoring are bit-identical to a
    batch that holds the whole prefill at once. Ragged and idle sessions included. At vocabulary
    2048 the sampled selection takes its bound from the head's group maxima (64 groups of 32
    columns), offset per pass like the logits; at 512 it computes them itself."""
    spec = synth.ModelSpec(**{**synth.CONFIGS[2].__dict__, "vocab": vocab})
    gm = quant.Model.decode(synth.build_model_file(spec))
    n = 300
    prompts = synth.prompts_uniform_fast(n, 48, spec.vocab, seed=41)
    lens = synth.prompt_lengths(n, 1, 48, seed=41)
    lens[5] = 0
    limits = (1 + np.arange(n) % 16).astype(np.int32)
    act = lens > 0
    got = {}
    for label, mb in (("one pass", None), ("passes", "1")):
        if mb:
            monkeypatch.setenv("MC_PREFILL_SCRATCH_MB", mb)
        else:
            monkeypatch.delenv("MC_PREFILL_SCRATCH_MB", raising=False)
        b = gm.new_batch(n, 0, 48, top_k=16)
        r = {}
        r["greedy"] = b.generate(prompts, lens, 8)
        r["sampled"] = b.generate(prompts, lens, 8, temperature=0.9, session0=7)
        r["limits"] = b.generate_limits(prompts, lens, limits, temperature=0.9)
        r["prefill"] = b.prefill(prompts, lens, want_logits=True)
        r["score"] = b.score(prompts, lens)
        b.close()
        got[label] = r
    monkeypatch.delenv("MC_PREFILL_SCRATCH_MB", raising=False)
    for key in ("greedy", "sampled", "limits", "prefill"):
        for i, (a, c) in enumerate(zip(got["one pass"][key], got["passes"][key])):
            assert np.array_equal(a[act], c[act]), f"{key}[{i}]: {np.sum(a[act] != c[act])} entries differ"
    assert np.array_equal(got["one pass"]["score"], got["passes"]["score"])
    gm.close()


def test_generate_limits_greedy_matches_generate():
    """Greedy mc_generate_limits: each session's row is mc_generate's row cut at its limit (the
    fused greedy head with per-session counters), -1 after it; a limit of n_max everywhere gives
    mc_generate's rows exactly."""
    spec = synth.ModelSpec(**{**synth.CONFIGS[2].__dict__, "vocab": 512})
    gm = quant.Model.decode(synth.build_model_file(spec))
    n, n_max = 200, 20
    prompts = synth.prompts_uniform_fast(n, 48, spec.vocab, seed=43)
    lens = synth.prompt_lengths(n, 1, 48, seed=43)
    limits = (1 + np.arange(n) * 3 % n_max).astype(np.int32)
    limits[0] = n_max
    b = gm.new_batch(n, 0, 48)
    t0, p0 = b.generate(prompts, lens, n_max)
    t1, p1, l1 = b.generate_limits(prompts, lens, limits)
    assert np.array_equal(l1, limits)
    for s in range(n):
        k = int(limits[s])
        assert np.array_equal(t1[s, :k], t0[s, :k]) and np.all(t1[s, k:] == -1), s
        assert np.array_equal(p1[s, :k], p0[s, :k]), s
    t2, _, _ = b.generate_limits(prompts, lens, np.full(n, n_max, np.int32))
    assert np.array_equal(t2, t0)
    b.close()
    gm.close()
