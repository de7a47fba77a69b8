"""mc_load_model_full: a full-precision model file quantized on the GPU (pkg/model.Decode then
quant.Quantize, internal/quant/convert.go:8-98) must give the model that the INT8 file of the same
weights gives — the host statement of Quantize (synth.quantize_float_model, NewTensorF32 restated
and pinned in test_oracle_kernels.py) — so the logits of both are bit-identical."""
import numpy as np
import pytest

from mignon_ai_b200 import quant, synth
from mignon_ai_b200._lib import MignonCudaError

pytestmark = pytest.mark.gpu

SHAPES = [
    # vocab, state, hidden, blocks, steps, base, tied, heads, window
    (512, 128, 256, 2, 1, 2, True, 4, 16),
    (300, 64, 96, 3, 2, 2, False, 2, 0),
    (256, 64, 128, 2, 3, 2, False, 0, 0),   # DefaultTwoBlockConfig
    (1000, 192, 512, 1, 2, 2, True, 4, 32),
]


@pytest.mark.parametrize("shape", SHAPES)
def test_full_model_quantized_on_device_matches_int8_file(shape):
    V, D, H, nb, steps, base, tied, heads, window = shape
    fm = synth.build_float_model(V, D, H, nb, steps, base, tied=tied, attn_heads=heads, attn_window=window,
                                 context=64, seed=V + D)
    full = quant.Model.decode_full(synth.encode_full_model(fm))
    ref = quant.Model.decode(synth.encode_model(synth.quantize_float_model(fm)))
    for k in ("vocab", "state", "hidden", "blocks", "max_context", "attn_heads", "attn_window", "total_steps", "ring"):
        assert getattr(full, k) == getattr(ref, k), k
    n, P = 16, 24
    prompts = synth.prompts_uniform_fast(n, P, V, seed=3)
    lens = np.arange(1, n + 1, dtype=np.int32)
    outs = []
    for m in (full, ref):
        b = m.new_batch(n, 0, P)
        logits, nxt, prob = b.prefill(prompts, lens, want_logits=True)
        toks, _ = b.generate(prompts, lens, 6)
        b.close()
        outs.append((logits, nxt, toks))
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    np.testing.assert_array_equal(outs[0][2], outs[1][2])
    full.close()
    ref.close()


def test_full_model_context_and_errors():
    fm = synth.build_float_model(64, 32, 48, 1, 2, 2, attn_heads=2, context=96)
    data = synth.encode_full_model(fm)
    assert quant.Model.decode_full(data).max_context == 96
    assert quant.Model.decode_full(data, max_context=80).max_context == 80
    # quant.NewModel raises a context below 64 to its default 128 (internal/quant/model.go:92-93)
    assert quant.Model.decode_full(data, max_context=40).max_context == 128
    with pytest.raises(MignonCudaError, match="not a full-precision"):
        quant.Model.decode_full(synth.encode_model(synth.quantize_float_model(fm)))
    bad = bytearray(data)
    n = int.from_bytes(bad[8:12], "little")
    bad[12 + n:16 + n] = (fm.weights.size - 1).to_bytes(4, "little")
    with pytest.raises(MignonCudaError):
        quant.Model.decode_full(bytes(bad[:-4]))
    fm2 = synth.build_float_model(64, 32, 48, 1, 2, 2)
    fm2.weights = fm2.weights[:-1]
    with pytest.raises(MignonCudaError, match="architecture mismatch"):
        quant.Model.decode_full(synth.encode_full_model(fm2))
