"""Pins the oracle's engine to the reference's own engine tests.

Restates internal/quant/session_test.go, equivalence_test.go, binary_test.go and
internal/binfmt/binfmt_test.go with models from this package's seeded generator (the reference
draws its test weights from Go's math/rand, which is not available here).
"""
import numpy as np
import pytest

from mignon_ai_b200 import synth

import dense_ref

VOCAB, STATE, HIDDEN = 16, 8, 12
ONE = [synth.BlockConfig(3, 2, 1)]
TWO = [synth.BlockConfig(2, 2, 1), synth.BlockConfig(2, 2, 2)]
# quantEquivCases (equivalence_test.go:35-49): name, blocks, maxContext, heads, window
CASES = [("1blk", ONE, 64, 0, 0), ("2blk", TWO, 64, 0, 0), ("2blk ctx=256", TWO, 256, 0, 0),
         ("1blk attn", ONE, 64, 2, 0), ("2blk attn", TWO, 64, 2, 0), ("2blk attn window", TWO, 64, 4, 3)]


def case_model(case, tied=True):
    name, blocks, ctx, heads, window = case
    return synth.build_model_uniform(VOCAB, STATE, HIDDEN, blocks, heads, window, ctx, seed=3, tied=tied)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_session_matches_call(oracle, case):
    """TestQuantSessionMatchesCall (session_test.go:18-52): cached logits are bit-identical to a
    full pass, before and after the 12-token window overflows, and for a long prefill."""
    qm = case_model(case)
    m = oracle.Model(synth.encode_model(qm))
    tokens = synth.uniform_ints(40, 0, VOCAB - 1, 9, 77, 0).astype(np.int32)
    sess = m.new_session(12)
    window = list(tokens[:5])
    assert np.array_equal(sess.prefill(window), m.call(window))
    for t in tokens[5:]:
        window.append(t)
        assert np.array_equal(sess.append(t), m.call(window))
    long = tokens[:24]
    assert np.array_equal(sess.prefill(long), m.call(long[-12:]))


def test_session_state_is_bounded(oracle):
    """TestQuantSessionStateIsBounded (session_test.go:56-73)."""
    case = CASES[1]
    m = oracle.Model(synth.encode_model(case_model(case)))
    sess = m.new_session(12)
    sess.prefill([1, 2])
    before = sess.state_bytes()
    for i in range(10 * case[2]):
        sess.append(i % VOCAB)
    assert sess.state_bytes() == before
    assert m.ring == max(m.dilations()) + 1
    assert sess.position() == 2 + 10 * case[2]  # the session streams past its window


def test_windowed_attention_state_is_bounded(oracle):
    """TestQuantSessionWindowedAttentionIsBounded (session_test.go:77-90)."""
    case = CASES[5]
    m = oracle.Model(synth.encode_model(case_model(case)))
    sess = m.new_session(12)
    sess.prefill([1, 2])
    before = sess.state_bytes()
    for i in range(10 * case[2]):
        sess.append(i % VOCAB)
    assert sess.state_bytes() == before
    assert m.attn_cache == case[4]


def test_empty_prefill_returns_nil(oracle):
    m = oracle.Model(synth.encode_model(case_model(CASES[0])))
    assert m.new_session(12).prefill([]) is None
    assert m.call([]) is None


def test_out_of_range_tokens_read_token_zero(oracle):
    """appendPosition clamps ids outside [0, vocab) to 0 (stream.go:144-146)."""
    m = oracle.Model(synth.encode_model(case_model(CASES[4])))
    assert np.array_equal(m.call([3, -1, VOCAB + 5]), m.call([3, 0, 0]))


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_quantized_matches_dequantized(oracle, case):
    """TestQuantizedMatchesDequantized (equivalence_test.go:75-98): the INT8 engine against a
    float64 engine on the dequantized weights, every prefix, max |dlogit| <= 1e-3."""
    qm = case_model(case)
    m = oracle.Model(synth.encode_model(qm))
    context = [2, 5, 7, 1, 9, 3, 11, 4, 0, 15]
    for n in range(1, len(context) + 1):
        got = m.call(context[:n]).astype(np.float64)
        want = dense_ref.forward_all(qm, context[:n], max_context=case[2])[-1]
        assert np.max(np.abs(got - want)) <= 1e-3, (case[0], n)


@pytest.mark.parametrize("tied", [True, False], ids=["tied", "untied"])
def test_binary_file_matches_json(oracle, tied):
    """TestBinaryFileMatchesJSON (binary_test.go:14-56): the binary and JSON files load to the
    same model; the binary one is less than half the size."""
    qm = synth.build_model_uniform(80, 16, 24, synth.build_block_configs(2, 3, 2), 2, 8, 32, seed=3, tied=tied)
    b = synth.encode_model(qm)
    j = synth.encode_model_json(qm)
    assert len(b) < len(j) / 2
    mb, mj = oracle.Model(b), oracle.Model(j)
    ctx = [2, 7, 14, 3, 9]
    assert np.array_equal(mb.call(ctx), mj.call(ctx))


def test_binary_file_rejects_damage(oracle):
    """TestBinaryFileRejectsDamage (binary_test.go:58-75)."""
    qm = synth.build_model_uniform(16, 8, 8, synth.build_block_configs(2, 3, 2), 0, 0, 16, seed=1)
    good = synth.encode_model(qm)
    oracle.Model(good)
    damaged = {
        "cut in the arrays": good[:-5],
        "cut in the header": good[:20],
        "trailing bytes": good + bytes([1, 2, 3]),
        "wrong version": good[:4] + bytes([9, 0]) + good[6:],
        "wrong kind": good[:6] + bytes([7]) + good[7:],
    }
    for name, data in damaged.items():
        with pytest.raises(ValueError):
            oracle.Model(data)


def test_model_file_header_round_trip(oracle):
    """The package's writer and the oracle's reader agree on every config's shapes."""
    for k, spec in synth.CONFIGS.items():
        small = synth.ModelSpec(**{**spec.__dict__, "vocab": 64})
        m = oracle.Model(synth.build_model_file(small))
        assert (m.vocab, m.state, m.hidden, m.blocks) == (64, spec.state, spec.hidden, spec.blocks)
        assert (m.attn_heads, m.attn_window, m.max_context) == (spec.attn_heads, spec.attn_window, 128)
    m4 = oracle.Model(synth.build_model_file(synth.ModelSpec(**{**synth.CONFIGS[4].__dict__, "vocab": 64})))
    assert list(m4.dilations()) == [1, 2, 2, 4, 4, 8, 8, 16, 16, 32, 32, 32]
    assert m4.ring == 33


def test_score_matches_call_per_prefix(oracle):
    """Per-token log-probs of one streaming pass equal logProb of a Call per prefix
    (eval.go:27-40 scores each prefix with a full Call)."""
    qm = case_model(CASES[5])
    m = oracle.Model(synth.encode_model(qm))
    seq = synth.uniform_ints(20, 0, VOCAB - 1, 4, 1, 0).astype(np.int32)
    lp = m.score(seq[None, :])[0]
    for t in range(1, 20):
        assert lp[t - 1] == oracle.log_prob(m.call(seq[:t]), int(seq[t]))
