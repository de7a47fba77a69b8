"""Seeded synthetic INT8 models and prompts for the benchmark configurations.

The reference has no N(0, 0.02) initialiser and its own init draws from Go's global
``math/rand``, so the benchmark models are produced here by a documented generator and written
in the reference's own INT8 model file format (``mignon.model/1``), which is the interchange both
this engine and the CPU oracle load.

* Random numbers: Philox4x32-10 (Salmon et al., SC'11, "Parallel random numbers: as easy as
  1, 2, 3"), key = (seed, stream), counter = (i, 0, 0, 0).
* Normals: Box-Muller on pairs of Philox words, u = (x + 0.5) * 2^-32.
* Quantizer: restates ``NewTensorF32`` (internal/quant/tensor.go:12-42): per-tensor
  scale = maxAbs/127 in float32, q = clamp(round_half_away(float32(w / scale)), -127, 127).
* File: ``binfmt.Encode`` (internal/binfmt/binfmt.go:47-78) of the header JSON of
  ``CheckpointJSON.withoutArrays`` (internal/quant/checkpoint.go:16-29,106-123) followed by the
  arrays in the order of ``CheckpointJSON.arrays`` (internal/quant/checkpoint.go:77-89).
* Block schedule: ``ca.BuildBlockConfigs`` (internal/ca/model.go:33-59).
"""
from __future__ import annotations

import dataclasses
import json
import struct
from typing import List, Optional, Sequence

import numpy as np

# Philox4x32-10 constants (Random123).
_PHILOX_M0 = np.uint64(0xD2511F53)
_PHILOX_M1 = np.uint64(0xCD9E8D57)
_PHILOX_W0 = 0x9E3779B9
_PHILOX_W1 = 0xBB67AE85
_MASK32 = np.uint64(0xFFFFFFFF)

# Streams of the synthetic generator (second key word).
STREAM_PROMPT = 0x50524F4D  # "PROM"
STREAM_LENGTH = 0x4C454E53  # "LENS"
STREAM_SAMPLE = 0x53414D50  # "SAMP"

MAX_CA_DILATION = 32          # internal/ca/config.go:59
DEFAULT_MIN_CONTEXT = 64      # internal/ca/config.go:55
NUM_SPECIAL_TOKENS = 5        # <PAD>,<UNK>,<USER>,<BOT>,<EOS> (internal/tokenizer/tokenizer.go:29-31)


def philox4x32(counters: np.ndarray, key0: int, key1: int) -> np.ndarray:
    """Philox4x32-10 on an array of counters of shape (n, 4) (uint32); returns (n, 4) uint32."""
    c = counters.astype(np.uint64) & _MASK32
    c0, c1, c2, c3 = c[:, 0], c[:, 1], c[:, 2], c[:, 3]
    k0, k1 = key0 & 0xFFFFFFFF, key1 & 0xFFFFFFFF
    for _ in range(10):
        p0 = _PHILOX_M0 * c0
        p1 = _PHILOX_M1 * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK32
        c0, c1, c2, c3 = (hi1 ^ c1 ^ np.uint64(k0)), lo1, (hi0 ^ c3 ^ np.uint64(k1)), lo0
        k0 = (k0 + _PHILOX_W0) & 0xFFFFFFFF
        k1 = (k1 + _PHILOX_W1) & 0xFFFFFFFF
    return np.stack([c0, c1, c2, c3], axis=1).astype(np.uint32)


def philox_words(n: int, key0: int, key1: int, row: int = 0) -> np.ndarray:
    """The first n uint32 words of the stream (key0, key1) with counters (i, row, 0, 0)."""
    calls = (n + 3) // 4
    ctr = np.zeros((calls, 4), dtype=np.uint64)
    ctr[:, 0] = np.arange(calls, dtype=np.uint64)
    ctr[:, 1] = row
    return philox4x32(ctr, key0, key1).reshape(-1)[:n]


def normal_f32(n: int, seed: int, stream: int, std: float) -> np.ndarray:
    """n float32 draws of N(0, std^2): Box-Muller over Philox words (u1,u2),(u3,u4) per call."""
    w = philox_words(((n + 3) // 4) * 4, seed, stream).astype(np.float64)
    u = (w + 0.5) * (2.0 ** -32)
    u1, u2 = u[0::2], u[1::2]
    r = np.sqrt(-2.0 * np.log(u1))
    t = 2.0 * np.pi * u2
    z = np.empty(u.shape[0], dtype=np.float64)
    z[0::2] = r * np.cos(t)
    z[1::2] = r * np.sin(t)
    return (std * z[:n]).astype(np.float32)


def uniform_ints(n: int, lo: int, hi: int, seed: int, stream: int, row: int) -> np.ndarray:
    """n integers uniform in [lo, hi] (inclusive) from one Philox row of the stream."""
    w = philox_words(n, seed, stream, row).astype(np.uint64)
    return (np.uint64(lo) + w % np.uint64(hi - lo + 1)).astype(np.int64)


# ---------------------------------------------------------------------------------------------
# Quantizer (restates internal/quant/tensor.go:12-42)
# ---------------------------------------------------------------------------------------------

def quantize_tensor(weights: np.ndarray):
    """Symmetric per-tensor int8 quantization, exactly as ``quant.NewTensorF32``."""
    w = np.ascontiguousarray(weights, dtype=np.float32).reshape(-1)
    if w.size == 0:
        return np.zeros(0, dtype=np.int8), np.float32(0.0)
    max_abs = np.float32(np.max(np.abs(w)))
    if max_abs == 0:
        return np.zeros(w.size, dtype=np.int8), np.float32(1.0)
    scale = np.float32(max_abs / np.float32(127.0))
    q = (w / scale).astype(np.float32).astype(np.float64)  # float32 division, widened
    r = np.sign(q) * np.floor(np.abs(q) + 0.5)                # math.Round: half away from zero
    r = np.clip(r, -127, 127)
    return r.astype(np.int8), scale


def dequantize_tensor(data: np.ndarray, scale) -> np.ndarray:
    """``Tensor.DequantizeF32`` (internal/quant/tensor.go:45-51)."""
    return data.astype(np.float32) * np.float32(scale)


# ---------------------------------------------------------------------------------------------
# Architecture
# ---------------------------------------------------------------------------------------------

@dataclasses.dataclass
class BlockConfig:
    steps: int
    dilation_base: int
    initial_dilation: int


def build_block_configs(num_blocks: int, steps: int, dilation_base: int) -> List[BlockConfig]:
    """Restates ``ca.BuildBlockConfigs`` (internal/ca/model.go:33-59, DefaultTwoBlockConfig :25-30)."""
    if num_blocks <= 1:
        return [BlockConfig(steps, dilation_base, 1)]
    if num_blocks == 2 and steps in (3, 5) and dilation_base == 2:
        return [BlockConfig(3, 2, 1), BlockConfig(3, 2, 4)]
    out, cur = [], 1
    for _ in range(num_blocks):
        out.append(BlockConfig(steps, dilation_base, cur))
        for _ in range(steps - 1):
            cur *= dilation_base
            if cur > MAX_CA_DILATION:
                cur = MAX_CA_DILATION
                break
    return out


def step_dilation(initial: int, base: int, step: int) -> int:
    """``ca.StepDilation`` (internal/ca/layout.go:24-30)."""
    d = initial
    s = 0
    while s < step and d < MAX_CA_DILATION:
        d *= base
        s += 1
    return min(d, MAX_CA_DILATION)


@dataclasses.dataclass
class ModelSpec:
    vocab: int
    state: int
    hidden: int
    blocks: int
    steps: int
    dilation_base: int = 2
    attn_heads: int = 0
    attn_window: int = 0
    context: int = 128
    seed: int = 0
    std: float = 0.02
    tied: bool = True


# The benchmark configurations 1-4 (shapes; prompts are generated by the workload helpers below).
CONFIGS = {
    1: ModelSpec(vocab=1024, state=64, hidden=128, blocks=2, steps=1, attn_heads=0, attn_window=0),
    2: ModelSpec(vocab=2048, state=128, hidden=256, blocks=4, steps=1, attn_heads=4, attn_window=64),
    3: ModelSpec(vocab=4096, state=384, hidden=1024, blocks=8, steps=1, attn_heads=6, attn_window=64),
    4: ModelSpec(vocab=2048, state=192, hidden=512, blocks=6, steps=2, attn_heads=4, attn_window=64),
}


@dataclasses.dataclass
class QTensor:
    data: np.ndarray  # int8
    scale: np.float32


@dataclasses.dataclass
class QBlock:
    cfg: BlockConfig
    w1: QTensor
    b1: np.ndarray
    w2: QTensor
    b2: np.ndarray
    gamma: np.ndarray
    wsel: QTensor
    attn_norm: Optional[np.ndarray] = None
    qkv: Optional[QTensor] = None
    out: Optional[QTensor] = None


@dataclasses.dataclass
class QModel:
    vocab: int
    state: int
    hidden: int
    tied: bool
    embed: QTensor
    blocks: List[QBlock]
    final_norm: np.ndarray
    head_w: QTensor
    head_b: np.ndarray
    context: int
    attn_heads: int
    attn_window: int


def build_model(spec: ModelSpec) -> QModel:
    """Seeded random-init model quantized with the restated ``NewTensorF32``.

    Every matrix (embedding, W1, W2, W_select, QKV, Out) is N(0, std^2) from its own Philox
    stream (key = (seed, tensor index), tensor index in file order). The other parameters follow
    the structure of the reference init (internal/ca/model.go:107-186, internal/nn/attention.go:42-52):
    norm gains 1, b1 = 0, b2 = 0 for the delta half and -1.386 for the gate half, head bias 0.
    """
    D, H, V = spec.state, spec.hidden, spec.vocab
    tensor_index = 0

    def mat(n):
        nonlocal tensor_index
        w = normal_f32(n, spec.seed, tensor_index, spec.std)
        tensor_index += 1
        d, s = quantize_tensor(w)
        return QTensor(d, s)

    embed = mat(V * D)
    blocks = []
    for bc in build_block_configs(spec.blocks, spec.steps, spec.dilation_base):
        w1 = mat(2 * H * 3 * D)
        w2 = mat(2 * D * H)
        wsel = mat(D * D)
        b1 = np.zeros(2 * H, dtype=np.float32)
        b2 = np.concatenate([np.zeros(D, np.float32), np.full(D, -1.386, np.float32)])
        gamma = np.ones(D, dtype=np.float32)
        qb = QBlock(bc, w1, b1, w2, b2, gamma, wsel)
        if spec.attn_heads > 0:
            qb.attn_norm = np.ones(D, dtype=np.float32)
            qb.qkv = mat(3 * D * D)
            qb.out = mat(D * D)
        blocks.append(qb)
    return QModel(vocab=V, state=D, hidden=H, tied=True, embed=embed, blocks=blocks,
                  final_norm=np.ones(D, dtype=np.float32),
                  head_w=QTensor(np.zeros(0, np.int8), np.float32(0.0)),
                  head_b=np.zeros(V, dtype=np.float32), context=spec.context,
                  attn_heads=spec.attn_heads, attn_window=spec.attn_window)


# ---------------------------------------------------------------------------------------------
# mignon.model/1 writer (internal/binfmt/binfmt.go:47-78, internal/quant/checkpoint.go:106-135)
# ---------------------------------------------------------------------------------------------

def go_float32_json(x) -> str:
    """Formats a float32 the way Go's encoding/json does: shortest round-trip digits, 'f' form
    unless |x| < 1e-6 or >= 1e21, where the 'e' form is used with a one-digit negative exponent
    cleaned up (e-07 -> e-7)."""
    f = np.float32(x)
    a = abs(float(f))
    if a != 0 and (a < 1e-6 or a >= 1e21):
        s = np.format_float_scientific(f, unique=True, trim='-')
        mant, exp = s.split('e')
        sign = exp[0]
        digits = exp[1:].lstrip('0') or '0'
        if sign == '+':
            exp = 'e+' + (digits if len(digits) >= 2 else '0' + digits)
        else:
            exp = 'e-' + digits
        return mant + exp
    return np.format_float_positional(f, unique=True, trim='-')


def _tensor_header(t: QTensor) -> str:
    return '{"data":null,"scale":%s}' % go_float32_json(t.scale)


def header_json(m: QModel, metadata: Optional[dict] = None) -> bytes:
    """The binary file's header: ``json.Marshal(cp.withoutArrays())`` with Go's field order."""
    blocks = []
    for b in m.blocks:
        s = ('{"steps":%d,"dilation_base":%d,"initial_dilation":%d,"rule_w1":%s,"rule_b1":null,'
             '"rule_w2":%s,"rule_b2":null,"rule_w_select":%s' % (
                 b.cfg.steps, b.cfg.dilation_base, b.cfg.initial_dilation,
                 _tensor_header(b.w1), _tensor_header(b.w2), _tensor_header(b.wsel)))
        if b.qkv is not None:
            s += ',"attn":{"norm":null,"qkv":%s,"out":%s}' % (_tensor_header(b.qkv), _tensor_header(b.out))
        blocks.append(s + '}')
    meta = {"context_size": m.context, "tied_embed": m.tied or None,
            "attn_heads": m.attn_heads or None, "attn_window": m.attn_window or None}
    if metadata:
        meta.update(metadata)
    meta_order = ["blocks", "state_size", "hidden_size", "steps", "dilation_base", "context_size",
                  "task", "tied_embed", "attn_heads", "attn_window", "tokenizer_version"]
    meta_items = [(k, meta[k]) for k in meta_order if meta.get(k)]
    meta_s = "{" + ",".join('"%s":%s' % (k, json.dumps(v)) for k, v in meta_items) + "}"
    head = ('{"vocab_size":%d,"state_size":%d,"hidden_size":%d,"tied_embed":%s,"embed":%s,'
            '"blocks":[%s],"head_w":%s,"head_b":null,"vocab":null,"metadata":%s}' % (
                m.vocab, m.state, m.hidden, "true" if m.tied else "false", _tensor_header(m.embed),
                ",".join(blocks), _tensor_header(m.head_w), meta_s))
    return head.encode()


def model_arrays(m: QModel) -> List[np.ndarray]:
    """``CheckpointJSON.arrays`` order (internal/quant/checkpoint.go:77-89)."""
    out = [m.embed.data]
    for b in m.blocks:
        out += [b.w1.data, b.b1, b.w2.data, b.b2, b.gamma, b.wsel.data]
        if b.qkv is not None:
            out += [b.attn_norm, b.qkv.data, b.out.data]
    out += [m.final_norm, m.head_w.data, m.head_b]
    return out


def encode_model(m: QModel, metadata: Optional[dict] = None) -> bytes:
    """The binary INT8 model file of m (``quant.Encode``)."""
    header = header_json(m, metadata)
    parts = [b"MGNN", struct.pack("<HBB", 1, 2, 0), struct.pack("<I", len(header)), header]
    for a in model_arrays(m):
        a = np.ascontiguousarray(a)
        parts.append(struct.pack("<I", a.size))
        if a.dtype == np.int8:
            parts.append(a.tobytes())
        else:
            parts.append(a.astype("<f4").tobytes())
    return b"".join(parts)


def build_model_file(spec: ModelSpec) -> bytes:
    return encode_model(build_model(spec))


# ---------------------------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------------------------

def prompts_uniform(n_sessions: int, length: int, vocab: int, seed: int) -> np.ndarray:
    """n_sessions prompts of `length` ids uniform over the non-special ids [5, vocab-1]."""
    out = np.empty((n_sessions, length), dtype=np.int32)
    for s in range(n_sessions):
        out[s] = uniform_ints(length, NUM_SPECIAL_TOKENS, vocab - 1, seed, STREAM_PROMPT, s)
    return out


def prompts_uniform_fast(n_sessions: int, length: int, vocab: int, seed: int) -> np.ndarray:
    """Same values as ``prompts_uniform``, generated in one vectorised Philox pass."""
    calls = (length + 3) // 4
    ctr = np.zeros((n_sessions * calls, 4), dtype=np.uint64)
    ctr[:, 0] = np.tile(np.arange(calls, dtype=np.uint64), n_sessions)
    ctr[:, 1] = np.repeat(np.arange(n_sessions, dtype=np.uint64), calls)
    w = philox4x32(ctr, seed, STREAM_PROMPT).reshape(n_sessions, calls * 4)[:, :length]
    span = np.uint64(vocab - NUM_SPECIAL_TOKENS)
    return (np.uint64(NUM_SPECIAL_TOKENS) + w.astype(np.uint64) % span).astype(np.int32)


def prompt_lengths(n_sessions: int, lo: int, hi: int, seed: int) -> np.ndarray:
    """Per-session prompt lengths uniform in [lo, hi] (config 3)."""
    ctr = np.zeros((n_sessions, 4), dtype=np.uint64)
    ctr[:, 0] = np.arange(n_sessions, dtype=np.uint64)
    w = philox4x32(ctr, seed, STREAM_LENGTH)[:, 0].astype(np.uint64)
    return (np.uint64(lo) + w % np.uint64(hi - lo + 1)).astype(np.int32)


def sample_uniform(session: int, step: int) -> float:
    """The sampler's uniform draw in [0, 1) for (session, step): Philox4x32-10 with key
    (session, "SAMP") and counter (step, 0, 0, 0); 53 bits from the first two words."""
    ctr = np.array([[step, 0, 0, 0]], dtype=np.uint64)
    w = philox4x32(ctr, session, STREAM_SAMPLE)[0].astype(np.uint64)
    return float(((int(w[0]) >> 5) * 67108864 + (int(w[1]) >> 6)) * (2.0 ** -53))


def build_model_uniform(vocab: int, state: int, hidden: int, block_configs: Sequence[BlockConfig],
                        attn_heads: int = 0, attn_window: int = 0, context: int = 64, seed: int = 3,
                        scale: float = 0.5, tied: bool = True) -> QModel:
    """Every full-precision parameter uniform in [-scale, scale) (norm gains and biases included),
    then quantized: the shape of the reference's equivalence-test models
    (internal/quant/equivalence_test.go:64-73), drawn from Philox instead of Go's math/rand."""
    D, H, V = state, hidden, vocab
    idx = 0

    def uni(n):
        nonlocal idx
        w = philox_words(n, seed, 0x554E4900 + idx).astype(np.float64)
        idx += 1
        return (((w + 0.5) * (2.0 ** -32)) * 2.0 - 1.0).astype(np.float64) * scale

    def mat(n):
        d, s = quantize_tensor(uni(n).astype(np.float32))
        return QTensor(d, s)

    embed = mat(V * D)
    blocks = []
    for bc in block_configs:
        w1, b1 = mat(2 * H * 3 * D), uni(2 * H).astype(np.float32)
        w2, b2 = mat(2 * D * H), uni(2 * D).astype(np.float32)
        gamma = uni(D).astype(np.float32)
        wsel = mat(D * D)
        qb = QBlock(BlockConfig(bc.steps, bc.dilation_base, bc.initial_dilation), w1, b1, w2, b2, gamma, wsel)
        if attn_heads > 0:
            qb.attn_norm = uni(D).astype(np.float32)
            qb.qkv = mat(3 * D * D)
            qb.out = mat(D * D)
        blocks.append(qb)
    head_w = QTensor(np.zeros(0, np.int8), np.float32(0.0)) if tied else mat(V * D)
    return QModel(vocab=V, state=D, hidden=H, tied=tied, embed=embed, blocks=blocks,
                  final_norm=uni(D).astype(np.float32), head_w=head_w,
                  head_b=uni(V).astype(np.float32), context=context, attn_heads=attn_heads,
                  attn_window=attn_window)


def encode_model_json(m: QModel, metadata: Optional[dict] = None) -> bytes:
    """The legacy JSON checkpoint of m (``quant.Save``: the same fields with the arrays inline)."""
    def t(x: QTensor):
        return {"data": [int(v) for v in x.data] if x.data.size else None, "scale": float(x.scale)}

    def f(a):
        return [float(v) for v in a] if a is not None and len(a) else None

    blocks = []
    for b in m.blocks:
        d = {"steps": b.cfg.steps, "dilation_base": b.cfg.dilation_base,
             "initial_dilation": b.cfg.initial_dilation, "rule_w1": t(b.w1), "rule_b1": f(b.b1),
             "rule_w2": t(b.w2), "rule_b2": f(b.b2), "gamma": f(b.gamma), "rule_w_select": t(b.wsel)}
        if b.qkv is not None:
            d["attn"] = {"norm": f(b.attn_norm), "qkv": t(b.qkv), "out": t(b.out)}
        blocks.append(d)
    meta = {"context_size": m.context, "tied_embed": m.tied, "attn_heads": m.attn_heads,
            "attn_window": m.attn_window}
    meta = {k: v for k, v in meta.items() if v}
    if metadata:
        meta.update(metadata)
    cp = {"vocab_size": m.vocab, "state_size": m.state, "hidden_size": m.hidden, "tied_embed": m.tied,
          "embed": t(m.embed), "blocks": blocks, "final_norm": f(m.final_norm), "head_w": t(m.head_w),
          "head_b": f(m.head_b), "vocab": None, "metadata": meta}
    # float32 values printed with 9 significant digits round-trip exactly.
    return json.dumps(cp, default=float).encode()


# ---------------------------------------------------------------------------------------------
# Full-precision model files (binfmt kind 1: internal/checkpoint/checkpoint.go:86-94) and the
# flat weight layout of ca.NewLayout (internal/ca/layout.go:103-161)
# ---------------------------------------------------------------------------------------------

def layout_block_configs(num_blocks: int, steps: int, dilation_base: int) -> List[BlockConfig]:
    """BuildBlockConfigs as NewLayout stores it: a base <= 1 becomes 2, an initial dilation < 1
    becomes 1 (internal/ca/layout.go:115-122)."""
    return [BlockConfig(b.steps, b.dilation_base if b.dilation_base > 1 else 2, max(1, b.initial_dilation))
            for b in build_block_configs(num_blocks, steps, dilation_base)]


@dataclasses.dataclass
class FModel:
    """A full-precision model: its flat weight vector in ca.NewLayout order and its shape."""
    vocab: int
    state: int
    hidden: int
    blocks: int
    steps: int
    dilation_base: int
    tied: bool
    attn_heads: int
    attn_window: int
    context: int
    weights: np.ndarray  # float32


def full_layout(vocab: int, state: int, hidden: int, configs: Sequence[BlockConfig], tied: bool, attn_heads: int):
    """Offsets of ca.NewLayout: (block offsets [(layer1, layer2, gamma, select, attn)], final norm
    offset, head offset, total parameters)."""
    D, H, V = state, hidden, vocab
    in_dim = 3 * D
    l1, l2 = 2 * H * (in_dim + 1), 2 * D * (H + 1)
    cur = V * D
    blocks = []
    for _ in configs:
        sel = cur + l1 + l2 + D
        extra = sel + D * D
        attn = -1
        if attn_heads > 0:
            attn = extra
            extra += D + 4 * D * D
        blocks.append((cur, cur + l1, cur + l1 + l2, sel, attn))
        cur = extra
    final_norm = cur
    cur += D
    head = cur
    total = cur + (V if tied else V * (D + 1))
    return blocks, final_norm, head, total


def build_float_model(vocab: int, state: int, hidden: int, blocks: int, steps: int, dilation_base: int = 2,
                      tied: bool = True, attn_heads: int = 0, attn_window: int = 0, context: int = 64,
                      seed: int = 11, scale: float = 0.5) -> FModel:
    """Every parameter uniform in [-scale, scale) from Philox, one stream per parameter slot."""
    configs = layout_block_configs(blocks, steps, dilation_base)
    total = full_layout(vocab, state, hidden, configs, tied, attn_heads)[3]
    w = philox_words(total, seed, 0x46554C4C).astype(np.float64)
    weights = ((((w + 0.5) * (2.0 ** -32)) * 2.0 - 1.0) * scale).astype(np.float32)
    return FModel(vocab, state, hidden, blocks, steps, dilation_base, tied, attn_heads, attn_window, context, weights)


def float_model_parts(fm: FModel) -> dict:
    """The parameters quant.Quantize reads from the flat vector (internal/quant/convert.go:8-98):
    'embed', per block 'w1', 'b1', 'w2', 'b2', 'gamma', 'wsel' (+ 'attn_norm', 'qkv', 'out'),
    'final_norm', 'head_w' (untied) and 'head_b'; W1 and W2 rows carry their bias after their
    weights, and so do the rows of an untied head."""
    D, H, V = fm.state, fm.hidden, fm.vocab
    w = fm.weights
    configs = layout_block_configs(fm.blocks, fm.steps, fm.dilation_base)
    offs, fno, ho, total = full_layout(V, D, H, configs, fm.tied, fm.attn_heads)
    if w.size != total:
        raise ValueError("architecture mismatch: %d weights, the model needs %d" % (w.size, total))

    def rows(off, n, width):  # n rows of `width` weights followed by one bias each
        r = w[off:off + n * (width + 1)].reshape(n, width + 1)
        return r[:, :width].reshape(-1), r[:, width].copy()

    parts = {"embed": w[:V * D], "configs": configs, "blocks": []}
    for o1, o2, og, osel, oa in offs:
        b = {}
        b["w1"], b["b1"] = rows(o1, 2 * H, 3 * D)
        b["w2"], b["b2"] = rows(o2, 2 * D, H)
        b["gamma"], b["wsel"] = w[og:og + D], w[osel:osel + D * D]
        if oa >= 0:
            b["attn_norm"] = w[oa:oa + D]
            b["qkv"] = w[oa + D:oa + D + 3 * D * D]
            b["out"] = w[oa + D + 3 * D * D:oa + D + 4 * D * D]
        parts["blocks"].append(b)
    parts["final_norm"] = w[fno:fno + D]
    if fm.tied:
        parts["head_b"] = w[ho:ho + V]
    else:
        parts["head_w"], parts["head_b"] = rows(ho, V, D)
    return parts


def quantize_float_model(fm: FModel, max_context: int = 0) -> QModel:
    """quant.Quantize (internal/quant/convert.go:8-98) of a full-precision model, with the
    restated NewTensorF32; max_context <= 0 takes the model's context."""
    p = float_model_parts(fm)

    def qt(a):
        d, sc = quantize_tensor(np.ascontiguousarray(a, np.float32))
        return QTensor(d, sc)

    qblocks = []
    for bc, b in zip(p["configs"], p["blocks"]):
        qb = QBlock(bc, qt(b["w1"]), b["b1"].copy(), qt(b["w2"]), b["b2"].copy(), b["gamma"].copy(), qt(b["wsel"]))
        if "qkv" in b:
            qb.attn_norm, qb.qkv, qb.out = b["attn_norm"].copy(), qt(b["qkv"]), qt(b["out"])
        qblocks.append(qb)
    head_w = qt(p["head_w"]) if not fm.tied else QTensor(np.zeros(0, np.int8), np.float32(0.0))
    return QModel(vocab=fm.vocab, state=fm.state, hidden=fm.hidden, tied=fm.tied, embed=qt(p["embed"]),
                  blocks=qblocks, final_norm=p["final_norm"].copy(), head_w=head_w, head_b=p["head_b"].copy(),
                  context=max_context if max_context > 0 else fm.context, attn_heads=fm.attn_heads,
                  attn_window=fm.attn_window)


def encode_full_model(fm: FModel) -> bytes:
    """The binary full-precision model file (checkpoint.Encode): header
    ``json.Marshal(File{Vocab, Merges, Metadata})`` with a placeholder vocabulary of the model's
    size, then one float32 array of all weights."""
    meta = {"blocks": fm.blocks, "state_size": fm.state, "hidden_size": fm.hidden, "steps": fm.steps,
            "dilation_base": fm.dilation_base, "context_size": fm.context, "tied_embed": fm.tied,
            "attn_heads": fm.attn_heads, "attn_window": fm.attn_window, "tokenizer_version": 1}
    meta_s = "{" + ",".join('"%s":%s' % (k, json.dumps(v)) for k, v in meta.items() if v) + "}"
    vocab = ["<PAD>", "<UNK>", "<USER>", "<BOT>", "<EOS>"] + ["t%d" % i for i in range(5, fm.vocab)]
    header = ('{"weights":null,"vocab":%s,"metadata":%s}' % (json.dumps(vocab[:fm.vocab]), meta_s)).encode()
    w = np.ascontiguousarray(fm.weights, "<f4")
    return b"".join([b"MGNN", struct.pack("<HBB", 1, 1, 0), struct.pack("<I", len(header)), header,
                     struct.pack("<I", w.size), w.tobytes()])
