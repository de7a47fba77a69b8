"""The B200 engine against the CPU oracle on the same model files and prompts.

Bars (from the north star): logits within max |dlogit| <= 1e-3 * max |logit| at every step;
greedy token streams identical except after a step where the oracle's top-2 logit gap is below
1e-4 (the stream is excused from that step on).
"""
import numpy as np
import pytest

from mignon_ai_b200 import quant, synth

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3
TIE_GAP = 1e-4


def small_spec(k, vocab=None):
    spec = synth.CONFIGS[k]
    return synth.ModelSpec(**{**spec.__dict__, **({"vocab": vocab} if vocab else {})})


def check_logits(got, want, label):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    tol = LOGIT_TOL * max(1e-30, np.max(np.abs(want)))
    err = np.max(np.abs(got - want))
    assert err <= tol, f"{label}: max |dlogit| {err:.3g} > {tol:.3g}"
    return err


def compare_streams(got, want, want_logits):
    """Greedy streams equal, except from the first step where the oracle's top-2 gap < 1e-4."""
    excused = 0
    for s in range(want.shape[0]):
        for t in range(want.shape[1]):
            if got[s, t] == want[s, t]:
                continue
            top2 = np.sort(want_logits[s, t])[-2:]
            assert top2[1] - top2[0] < TIE_GAP, f"session {s} step {t}: {got[s, t]} != {want[s, t]}"
            excused += 1
            break
    return excused


def run_steps(model, prompts, lens, n_new):
    """Prefill + appends through the C-ABI with logits at every step (greedy feedback)."""
    b = model.new_batch(len(prompts), 0, prompts.shape[1])
    logits, nxt, prob = b.prefill(prompts, lens, want_logits=True)
    L = [logits.copy()]
    T = [nxt.copy()]
    P = [prob.copy()]
    for _ in range(n_new - 1):
        logits, nxt, prob = b.append(nxt, want_logits=True)
        L.append(logits.copy())
        T.append(nxt.copy())
        P.append(prob.copy())
    b.close()
    return np.stack(T, 1), np.stack(P, 1), np.stack(L, 1)


@pytest.mark.parametrize("cfg,n_sess,plen,n_new", [(1, 64, 32, 12), (2, 96, 48, 10)])
def test_decode_matches_oracle(oracle, cfg, n_sess, plen, n_new):
    spec = small_spec(cfg)
    data = synth.build_model_file(spec)
    om = oracle.Model(data)
    gm = quant.Model.decode(data)
    prompts = synth.prompts_uniform_fast(n_sess, plen, spec.vocab, seed=cfg)
    lens = np.full(n_sess, plen, np.int32)
    wt, wp, wl = om.generate_greedy(prompts, lens, n_new, logits=True)
    gt, gp, gl = run_steps(gm, prompts, lens, n_new)
    for t in range(n_new):
        for s in range(n_sess):
            if np.array_equal(gt[s, :t], wt[s, :t]):
                check_logits(gl[s, t], wl[s, t], f"cfg{cfg} session {s} step {t}")
    compare_streams(gt, wt, wl)
    same = gt == wt
    assert np.allclose(gp[same], wp[same], rtol=1e-4, atol=0)


EQUIV = [("1blk", [synth.BlockConfig(3, 2, 1)], 64, 0, 0),
         ("2blk", [synth.BlockConfig(2, 2, 1), synth.BlockConfig(2, 2, 2)], 64, 0, 0),
         ("2blk ctx=256", [synth.BlockConfig(2, 2, 1), synth.BlockConfig(2, 2, 2)], 256, 0, 0),
         ("1blk attn", [synth.BlockConfig(3, 2, 1)], 64, 2, 0),
         ("2blk attn", [synth.BlockConfig(2, 2, 1), synth.BlockConfig(2, 2, 2)], 64, 2, 0),
         ("2blk attn window", [synth.BlockConfig(2, 2, 1), synth.BlockConfig(2, 2, 2)], 64, 4, 3)]


@pytest.mark.parametrize("case", EQUIV, ids=[c[0] for c in EQUIV])
def test_session_stream_matches_oracle(oracle, case):
    """The reference's session test shape (session_test.go:18-52) on the GPU: prefill 5, stream 35
    tokens through a 12-token window, then a long prefill; logits against the oracle session."""
    name, blocks, ctx, heads, window = case
    qm = synth.build_model_uniform(16, 8, 12, blocks, heads, window, ctx, seed=3)
    data = synth.encode_model(qm)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    tokens = synth.uniform_ints(40, 0, 15, 9, 77, 0).astype(np.int32)
    os_, gs = om.new_session(12), gm.new_session(12)
    check_logits(gs.prefill(tokens[:5]), os_.prefill(tokens[:5]), f"{name} prefill")
    for i, t in enumerate(tokens[5:]):
        check_logits(gs.append(int(t)), os_.append(int(t)), f"{name} append {i}")
    check_logits(gs.prefill(tokens[:24]), os_.prefill(tokens[:24]), f"{name} long prefill")
    gs.close()


def test_generate_greedy_matches_oracle(oracle):
    """The device-resident decode loop (mc_generate) on config 2: 80 tokens after 48."""
    spec = small_spec(2)
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n = 64
    prompts = synth.prompts_uniform_fast(n, 48, spec.vocab, seed=2)
    lens = np.full(n, 48, np.int32)
    wt, wp, wl = om.generate_greedy(prompts, lens, 80, logits=True)
    b = gm.new_batch(n, 0, 48)
    gt, gp = b.generate(prompts, lens, 80)
    compare_streams(gt, wt, wl)
    same = gt == wt
    assert np.allclose(gp[same], wp[same], rtol=1e-4, atol=0)
    # the same batch again gives the same result (state fully reset by the prefill)
    gt2, _ = b.generate(prompts, lens, 80)
    assert np.array_equal(gt, gt2)
    b.close()


def test_one_token_prompts_match_oracle(oracle):
    """A prefill whose longest prompt has one token runs through the decode kernels, which read
    each session's token from the decode input: the prompt tokens must be the ones there, for
    mc_prefill (logits after the token), mc_generate and mc_score_targets alike."""
    spec = small_spec(2, vocab=512)
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n = 40
    prompts = synth.prompts_uniform_fast(n, 1, spec.vocab, seed=17)
    lens = np.ones(n, np.int32)
    b = gm.new_batch(n, 0, 8)
    # the decode input holds something else before the prefill
    b.append(np.full(n, 9, np.int32))
    logits, _, _ = b.prefill(prompts, lens, want_logits=True)
    for s in (0, 1, n - 1):
        check_logits(logits[s], om.call(prompts[s, :1]), f"prefill of one token, session {s}")
    wt, _, wl = om.generate_greedy(prompts, lens, 6, logits=True)
    gt, _ = b.generate(prompts, lens, 6)
    compare_streams(gt, wt, wl)
    tg = np.full((n, 1), 11, np.int32)
    lp = b.score_targets(prompts, tg, lens)
    for s in (0, n - 1):
        l = np.asarray(om.call(prompts[s, :1]), np.float64)
        want = l[11] - l.max() - np.log(np.sum(np.exp(l - l.max())))
        assert abs(lp[s, 0] - want) <= 2e-3 * np.max(np.abs(l))
    b.close()


def test_generate_stops_end_sessions_before_the_stop_token():
    """mc_generate_stops: greedyLoop's stop tokens (generate/greedy.go:63-87). A session ends
    before the first stop token it would emit, in the prefill's selection or in any decode step;
    the others go on unchanged. Sessions never interact and the stopped ones take no further
    steps, so every row equals the run without stops up to its first stop token, then -1 / 0, and
    its length is that position. Stops apply to one call only."""
    spec = small_spec(2, vocab=512)
    gm = quant.Model.decode(synth.build_model_file(spec))
    n, n_new = 200, 24
    prompts = synth.prompts_uniform_fast(n, 48, spec.vocab, seed=23)
    lens = synth.prompt_lengths(n, 1, 48, seed=23)
    lens[3] = 0
    act = lens > 0
    b = gm.new_batch(n, 0, 48)
    t0, p0 = b.generate(prompts, lens, n_new)
    vals, counts = np.unique(t0[act], return_counts=True)
    stops = vals[np.argsort(-counts, kind="stable")[:2]]
    t1, p1, got_len = b.generate(prompts, lens, n_new, stops=stops)
    stopped = 0
    for s in range(n):
        if not act[s]:
            assert got_len[s] == 0 and np.all(t1[s] == -1)
            continue
        hit = np.nonzero(np.isin(t0[s], stops))[0]
        k = int(hit[0]) if hit.size else n_new
        stopped += k < n_new
        assert got_len[s] == k, (s, got_len[s], k)
        assert np.array_equal(t1[s, :k], t0[s, :k]) and np.all(t1[s, k:] == -1)
        assert np.array_equal(p1[s, :k], p0[s, :k]) and np.all(p1[s, k:] == 0)
    assert stopped > 0
    t2, _ = b.generate(prompts, lens, n_new)
    assert np.array_equal(t2[act], t0[act])
    b.close()
    gm.close()


def test_ragged_prompts_and_idle_sessions(oracle):
    """Prompts of different lengths in one batch; a zero-length prompt leaves its session idle."""
    spec = small_spec(2, vocab=512)
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n = 40
    lens = synth.prompt_lengths(n, 1, 64, seed=3)
    lens[7] = 0
    prompts = synth.prompts_uniform_fast(n, 64, spec.vocab, seed=3)
    wt, wp, wl = om.generate_greedy(prompts, lens, 6, logits=True)
    gt, gp, gl = run_steps(gm, prompts, lens, 6)
    for s in range(n):
        if lens[s] == 0:
            continue
        check_logits(gl[s, 0], wl[s, 0], f"ragged session {s}")
    mask = lens > 0
    compare_streams(gt[mask], wt[mask], wl[mask])


def _cdf_margin(logits, temperature, topk, u):
    """Distance of the draw from the nearest bucket edge of the top-k CDF, relative to its total
    (the truncated branch of SampleRawLogitsAdvanced, generate/sample.go:91-172, on these logits)."""
    l = np.asarray(logits, np.float64)
    order = np.lexsort((np.arange(l.size), -l))[:topk]  # value descending, index ascending
    v = l[order] / temperature
    cdf = np.cumsum(np.exp(v - v[0]))
    return float(np.min(np.abs(cdf - u * cdf[-1])) / cdf[-1])


def test_sampling_matches_oracle(oracle):
    """Config-3 shapes (D=384, streamed activation tiles), T=0.8, top-k 40, Philox per session:
    the sampled streams equal the oracle's (the same draws). A stream may leave the oracle's only
    at a step where the oracle's own draw falls within 5e-3 of a CDF bucket edge (the logits
    agree to 1e-3 of their maximum, so only such draws can flip), and at most a quarter may."""
    spec = small_spec(3, vocab=1024)
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n, steps, T, K = 16, 12, 0.8, 40
    lens = synth.prompt_lengths(n, 16, 64, seed=3)
    prompts = synth.prompts_uniform_fast(n, 64, spec.vocab, seed=3)
    wt, wl = om.generate_sample(prompts, lens, steps, T, K, session0=0, logits=True)
    b = gm.new_batch(n, 0, 64, top_k=K)
    gt, _ = b.generate(prompts, lens, steps, temperature=T, session0=0)
    b.close()
    diverged = 0
    for s in range(n):
        diff = np.nonzero(gt[s] != wt[s])[0]
        if diff.size == 0:
            continue
        t = int(diff[0])
        diverged += 1
        m = _cdf_margin(wl[s, t], T, K, synth.sample_uniform(s, t))
        assert m < 5e-3, f"session {s} step {t}: {gt[s, t]} != {wt[s, t]} with the draw {m:.3g} from a bucket edge"
    assert diverged <= n // 4, diverged


def test_score_matches_oracle(oracle):
    """mc_score on config-4 shapes (D=192, 6 blocks x 2 rule steps, dilation up to 32, attention
    4 x 48): the log-probability of every next token from one prefill pass, against the oracle's
    logProb of Call(prefix) for every prefix (eval/suite.go:201-209). log p = l_t - logsumexp(l)
    moves by at most 2 max|dlogit|, so the bar is 2e-3 * max|logit|. Ragged, one-token and empty
    sequences included; afterwards the sessions continue like prefilled ones."""
    spec = small_spec(4, vocab=512)
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    n, L = 24, 64
    seqs = synth.prompts_uniform_fast(n, L, spec.vocab, seed=4)
    want = om.score(seqs)
    lens = np.full(n, L, np.int32)
    lens[5], lens[9], lens[11] = 1, 0, 30
    b = gm.new_batch(n, 0, L)
    got = b.score(seqs, lens)
    scale = max(float(np.max(np.abs(om.call(seqs[s])))) for s in range(4))
    for s in range(n):
        k = max(int(lens[s]) - 1, 0)
        err = float(np.max(np.abs(got[s, :k] - want[s, :k]), initial=0.0))
        assert err <= 2e-3 * scale, f"sequence {s}: max |dlogprob| {err:.3g} > {2e-3 * scale:.3g}"
        assert np.all(got[s, k:] == 0.0)
    # continuation: session 0 appends one token as after a prefill of its sequence
    tok = np.full(n, 7, np.int32)
    logits, _, _ = b.append(tok, want_logits=True)
    os_ = om.new_session(0)
    os_.prefill(seqs[0])
    check_logits(logits[0], os_.append(7), "append after score")
    b.close()


@pytest.mark.parametrize("cfg,vocab,dec_r", [(2, None, None), (1, None, None), (3, 1024, None), (4, 512, None),
                                             (2, None, "32")])
def test_decode_kernel_matches_block_kernel_bitwise(monkeypatch, cfg, vocab, dec_r):
    """Decode steps run on block_decode_kernel (weights on the MMA's M side, 32 sessions per CTA);
    block_kernel (128 session rows per CTA) computes the same float32 operations in the same
    order, so the two give bit-identical logits, tokens and probabilities (MC_DECODE_KERNEL=block
    selects block_kernel for a batch opened under it). Ragged and idle sessions included.
    Configs 1 and 2 run the 16-sessions-per-CTA instance (two CTAs per multiprocessor at state
    width 128), configs 3 and 4 the wide one; dec_r "32": the model is loaded under
    MC_DECODE_R=32, the 32-sessions-per-CTA instance."""
    spec = small_spec(cfg, vocab)
    data = synth.build_model_file(spec)
    if dec_r:
        monkeypatch.setenv("MC_DECODE_R", dec_r)
    gm = quant.Model.decode(data)
    monkeypatch.delenv("MC_DECODE_R", raising=False)
    n = 200
    prompts = synth.prompts_uniform_fast(n, 48, spec.vocab, seed=5)
    lens = np.full(n, 48, np.int32)
    lens[3] = 0
    lens[50] = 7
    lens[199] = 1
    got = {}
    for kern in ("decode", "block"):
        if kern == "block":
            monkeypatch.setenv("MC_DECODE_KERNEL", "block")
        else:
            monkeypatch.delenv("MC_DECODE_KERNEL", raising=False)
        got[kern] = run_steps(gm, prompts, lens, 6)
    monkeypatch.delenv("MC_DECODE_KERNEL", raising=False)
    act = lens > 0
    for i, name in enumerate(("tokens", "probs", "logits")):
        a, b = got["decode"][i][act], got["block"][i][act]
        assert np.array_equal(a, b), f"{name}: {np.sum(a != b)} entries differ"
    gm.close()


def test_perplexity_matches_reference_loop(oracle):
    """quant.perplexity / perplexity_per_doc (eval.Perplexity, eval.go:49-62; PerplexityPerDoc,
    perdoc.go:16-32) against the reference's nll.score loop (eval.go:27-43) restated with the
    oracle: every target t predicted from a fresh Call of the last context_size tokens before it.
    Streams longer than the context exercise mc_score_targets' windows past the first pass; batch
    size 8 splits the windows over several calls. Mean loss within 2e-3 * max|logit| (the
    per-token log-probability bar), bits per byte with it, token counts exact."""
    spec = small_spec(2, vocab=512)
    data = synth.build_model_file(spec)
    om, gm = oracle.Model(data), quant.Model.decode(data)
    ctx = 16
    rng = np.random.default_rng(21)
    text = rng.integers(5, spec.vocab, size=45)
    docs = [rng.integers(5, spec.vocab, size=k) for k in (9, 30, 1)]
    token_bytes = rng.integers(1, 5, size=spec.vocab)

    def ref(streams):
        nats, count, nbytes, scale = 0.0, 0, 0, 0.0
        for T in streams:
            for t in range(1, len(T)):
                logits = np.asarray(om.call(np.asarray(T[max(0, t - ctx):t], np.int32)), np.float64)
                m = logits.max()
                nats -= logits[T[t]] - m - np.log(np.sum(np.exp(logits - m)))
                count += 1
                nbytes += int(token_bytes[T[t]])
                scale = max(scale, float(np.max(np.abs(logits))))
        return nats / count, nats / (np.log(2.0) * nbytes), count, scale

    for got, streams in ((quant.perplexity(gm, text, ctx, token_bytes=token_bytes, batch_size=8), [list(text)]),
                         (quant.perplexity_per_doc(gm, docs, ctx, eos_id=4, token_bytes=token_bytes, batch_size=8),
                          [[4] + list(d) for d in docs])):
        loss, bpb, count, scale = ref(streams)
        assert got.tokens == count
        assert abs(got.loss - loss) <= 2e-3 * scale, (got.loss, loss)
        assert abs(got.ppl - np.exp(loss)) <= np.exp(loss) * 2e-3 * scale * 1.01
        assert abs(got.bpb - bpb) <= 2e-3 * scale / np.log(2.0)  # every token covers >= 1 byte
    gm.close()


def test_fused_head_matches_head_kernel(monkeypatch):
    """Greedy decode steps without logits run the head and the selection inside the final decode
    launch. The separate head_kernel + select_kernel path (MC_NO_FUSED_HEAD, read when a step is
    enqueued) computes the same logits, so the tokens are identical (first index of the maximum)
    and the probabilities agree to float rounding of the sum of exponentials."""
    spec = small_spec(2)
    gm = quant.Model.decode(synth.build_model_file(spec))
    n = 300
    prompts = synth.prompts_uniform_fast(n, 48, spec.vocab, seed=9)
    lens = synth.prompt_lengths(n, 1, 48, seed=9)
    lens[17] = 0
    got = {}
    for fused in (True, False):
        if fused:
            monkeypatch.delenv("MC_NO_FUSED_HEAD", raising=False)
        else:
            monkeypatch.setenv("MC_NO_FUSED_HEAD", "1")
        b = gm.new_batch(n, 0, 48)
        got[fused] = b.generate(prompts, lens, 24)
        b.close()
    monkeypatch.delenv("MC_NO_FUSED_HEAD", raising=False)
    act = lens > 0
    assert np.array_equal(got[True][0][act], got[False][0][act])
    assert np.allclose(got[True][1][act], got[False][1][act], rtol=1e-5, atol=0)
    gm.close()


def test_model_file_errors():
    """Damaged files are rejected by the engine's own reader (binary_test.go:58-75)."""
    qm = synth.build_model_uniform(16, 8, 8, synth.build_block_configs(2, 3, 2), 0, 0, 16, seed=1)
    good = synth.encode_model(qm)
    quant.Model.decode(good).close()
    from mignon_ai_b200._lib import MignonCudaError
    for data in (good[:-5], good[:20], good + b"\x01\x02\x03", good[:4] + b"\x09\x00" + good[6:],
                 good[:6] + b"\x07" + good[7:]):
        with pytest.raises(MignonCudaError):
            quant.Model.decode(data)
