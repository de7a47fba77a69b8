"""The full-precision model layout (ca.NewLayout, internal/ca/layout.go:103-161) and the host
statement of quant.Quantize (internal/quant/convert.go:8-98) that the device quantizer is tested
against. CPU only."""
import numpy as np
import pytest

from mignon_ai_b200 import synth

SHAPES = [
    # vocab, state, hidden, blocks, steps, base, tied, heads
    (12, 16, 24, 2, 3, 2, True, 2),    # TestOptimParamsCoverMatrices' layout (layout_test.go:8-10)
    (50, 8, 12, 3, 2, 2, False, 0),
    (40, 12, 20, 1, 4, 3, False, 3),
    (30, 8, 8, 2, 5, 2, True, 0),      # DefaultTwoBlockConfig: 3 steps per block despite steps = 5
]


@pytest.mark.parametrize("shape", SHAPES)
def test_layout_parameters_partition_the_vector(shape):
    """Every weight index is read by exactly one parameter, and the matrices hold no bias, gain or
    norm: the property TestOptimParamsCoverMatrices checks (layout_test.go:8-36), extended to the
    whole vector."""
    V, D, H, nb, steps, base, tied, heads = shape
    fm = synth.build_float_model(V, D, H, nb, steps, base, tied=tied, attn_heads=heads)
    fm.weights = np.arange(fm.weights.size, dtype=np.float32)  # exact indices below 2^24
    p = synth.float_model_parts(fm)
    mats, vecs = [p["embed"]], [p["final_norm"], p["head_b"]]
    if not tied:
        mats.append(p["head_w"])
    for b in p["blocks"]:
        mats += [b["w1"], b["w2"], b["wsel"]] + ([b["qkv"], b["out"]] if "qkv" in b else [])
        vecs += [b["b1"], b["b2"], b["gamma"]] + ([b["attn_norm"]] if "qkv" in b else [])
    idx = np.concatenate(mats + vecs).astype(np.int64)
    assert np.array_equal(np.sort(idx), np.arange(fm.weights.size))
    assert len(p["blocks"]) == len(synth.layout_block_configs(nb, steps, base))
    for b in p["blocks"]:
        assert b["w1"].size == 2 * H * 3 * D and b["w2"].size == 2 * D * H and b["wsel"].size == D * D


def test_default_two_block_config():
    """BuildBlockConfigs' special case (internal/ca/model.go:25-41) and NewLayout's defaults."""
    cfg = synth.layout_block_configs(2, 5, 2)
    assert [(c.steps, c.dilation_base, c.initial_dilation) for c in cfg] == [(3, 2, 1), (3, 2, 4)]
    cfg = synth.layout_block_configs(3, 2, 0)
    assert [(c.dilation_base, c.initial_dilation) for c in cfg] == [(2, 1), (2, 1), (2, 1)]


def test_quantized_model_loads_in_the_oracle(oracle):
    """The host statement of Quantize gives an INT8 file the oracle reads, with the file's
    context as maxContext, and its logits follow the float model's dequantized weights."""
    fm = synth.build_float_model(64, 16, 24, 2, 2, 2, tied=False, attn_heads=2, attn_window=8, context=32)
    q = synth.quantize_float_model(fm)
    om = oracle.Model(synth.encode_model(q))
    assert om.vocab == 64
    logits = om.call([5, 6, 7, 8])
    assert logits is not None and np.isfinite(logits).all()


def test_full_file_header():
    fm = synth.build_float_model(20, 8, 8, 1, 2, 2)
    data = synth.encode_full_model(fm)
    assert data[:4] == b"MGNN" and data[6] == 1
    n = int.from_bytes(data[8:12], "little")
    assert int.from_bytes(data[12 + n:16 + n], "little") == fm.weights.size
    assert len(data) == 16 + n + 4 * fm.weights.size
