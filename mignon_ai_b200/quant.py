"""Host-side mirror of the reference's INT8 session API, running on the B200 engine.

The names and meanings follow internal/quant and internal/infer of mignon-ai:

* ``Model.decode(data)`` / ``Model.load(path)``   quant.Decode / quant.Load (checkpoint.go:148-212)
* ``Model.call(window)`` = ``Model.forward``       quant.(*Model).Call / Forward (model.go:122-137)
* ``Model.new_session(context_size)``              quant.(*Model).NewSession (session.go:20-28)
* ``Session.prefill(tokens)`` / ``append(token)``  infer.Session (internal/infer/infer.go:12-17)
* ``Model.new_batch(...)``                         the batched extension: many sessions stepped
                                                   together, which is what makes the GPU fast.

Logits come back as float64 arrays widened from float32, as the reference returns them
(stream.go:244-246). Every call goes through libmignoncuda.so; there is no CPU path.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import numpy as np

from . import _lib
from ._lib import c_vp

_i = ctypes.c_int
_lib.register({
    "mc_open": [c_vp, ctypes.POINTER(c_vp)],
    "mc_close": [c_vp],
    "mc_load_model": [c_vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(c_vp)],
    "mc_load_model_full": [c_vp, ctypes.c_char_p, ctypes.c_size_t, _i, ctypes.POINTER(c_vp)],
    "mc_model_free": [c_vp],
    "mc_model_info": [c_vp, c_vp],
    "mc_batch_open": [c_vp, _i, _i, _i, _i, ctypes.POINTER(c_vp)],
    "mc_batch_close": [c_vp],
    "mc_prefill": [c_vp, c_vp, c_vp, _i, c_vp, c_vp, c_vp],
    "mc_score": [c_vp, c_vp, c_vp, _i, c_vp],
    "mc_score_targets": [c_vp, c_vp, c_vp, _i, c_vp, c_vp],
    "mc_append": [c_vp, c_vp, c_vp, c_vp, c_vp],
    "mc_generate": [c_vp, c_vp, c_vp, _i, _i, ctypes.c_double, ctypes.c_uint32, c_vp, c_vp],
    "mc_generate_stops": [c_vp, c_vp, c_vp, _i, _i, ctypes.c_double, ctypes.c_uint32, c_vp, _i, c_vp, c_vp, c_vp],
    "mc_generate_limits": [c_vp, c_vp, c_vp, _i, c_vp, _i, ctypes.c_double, ctypes.c_uint32, c_vp, c_vp, c_vp],
    "mc_generate_limits_dev": [c_vp, c_vp, c_vp, _i, _i, c_vp, _i, ctypes.c_double, ctypes.c_uint32, c_vp, c_vp],
    "mc_generate_dev": [c_vp, c_vp, c_vp, _i, _i, _i, ctypes.c_double, ctypes.c_uint32, c_vp, c_vp],
    "mc_batch_stream": [c_vp, _i, ctypes.POINTER(c_vp)],
    "mc_batch_error": [c_vp],
    "mc_probe_mma_i8": [_i, _i, _i, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)],
    "mc_generate_policy": [c_vp, c_vp, c_vp, _i, _i, c_vp, _i, c_vp, _i, c_vp, ctypes.c_uint32, c_vp, _i, c_vp, c_vp,
                           c_vp],
    "mc_sample_rows": [_i, c_vp, _i, _i, c_vp, c_vp, _i, c_vp, c_vp, c_vp, ctypes.c_uint32, ctypes.c_uint32, c_vp,
                       c_vp],
    "mc_sched_open": [c_vp, _i, _i, _i, _i, c_vp, _i, c_vp, _i, ctypes.POINTER(c_vp)],
    "mc_sched_close": [c_vp],
    "mc_sched_submit": [c_vp, c_vp, _i, _i, ctypes.c_uint32, ctypes.POINTER(ctypes.c_int64)],
    "mc_sched_step": [c_vp, _i, ctypes.POINTER(_i)],
    "mc_sched_run": [c_vp, _i],
    "mc_sched_result": [c_vp, ctypes.c_int64, c_vp, c_vp, _i, ctypes.POINTER(_i)],
    "mc_sched_stats": [c_vp, c_vp],
    "mc_sched_set_admit_min": [c_vp, _i],
})

# sampleContinuation's repetition window (internal/generate/constants.go:11)
CHAT_REPETITION_WINDOW = 6


class Sampling(ctypes.Structure):
    """mc_sampling: the knobs of generate.Sampling (internal/generate/chat.go:45-56).

    ``temperature`` <= 0.001 is argmax; ``rep_penalty`` > 1 penalises the distinct tokens of the
    last ``rep_window`` tokens (all when <= 0); ``top_k`` <= 0 and ``top_p`` outside (0, 1) are off;
    ``ban_trigrams`` turns on sampleContinuation's 3-gram repetition block."""
    _fields_ = [("temperature", ctypes.c_double), ("rep_penalty", ctypes.c_double), ("top_k", ctypes.c_int),
                ("top_p", ctypes.c_double), ("rep_window", ctypes.c_int), ("ban_trigrams", ctypes.c_int)]

    def __init__(self, temperature: float = 0.0, rep_penalty: float = 1.0, top_k: int = 0, top_p: float = 1.0,
                 rep_window: int = CHAT_REPETITION_WINDOW, ban_trigrams: bool = True):
        super().__init__(float(temperature), float(rep_penalty), int(top_k), float(top_p), int(rep_window),
                         int(bool(ban_trigrams)))


def sample_rows(logits, sampling: Sampling, recent=None, recent_lens=None, allowed=None, u=None, session0: int = 0,
                step: int = 0, device: int = 0):
    """SampleRawLogitsAdvanced (internal/generate/sample.go:33-172) over the rows of a float32
    [n x vocab] logits array on one GPU: (tokens [n], probs [n]). ``recent`` [n x m] with
    ``recent_lens`` are each row's recent tokens (the penalty window's source and, with
    ``ban_trigrams``, the generated tokens of the 3-gram block); ``allowed`` [n x vocab] masks
    tokens where < 0; ``u`` [n] are the uniform draws (default: Philox of (session0 + r, step))."""
    lg = np.ascontiguousarray(logits, np.float32)
    if lg.ndim != 2:
        raise ValueError("logits must be [n x vocab]")
    n, V = lg.shape
    rc = rl = None
    stride = 0
    if recent is not None:
        rc = np.ascontiguousarray(recent, np.int32).reshape(n, -1)
        stride = rc.shape[1]
        rl = (np.full(n, stride, np.int32) if recent_lens is None else np.ascontiguousarray(recent_lens, np.int32))
    al = np.ascontiguousarray(allowed, np.int32).reshape(n, V) if allowed is not None else None
    uu = np.ascontiguousarray(u, np.float64) if u is not None else None
    toks = np.zeros(n, np.int32)
    probs = np.zeros(n, np.float32)
    _lib.check(_lib.lib().mc_sample_rows(device, _lib.ptr(lg), n, V, _lib.ptr(rc), _lib.ptr(rl), stride,
                                         _lib.ptr(al), ctypes.byref(sampling), _lib.ptr(uu), session0, step,
                                         _lib.ptr(toks), _lib.ptr(probs)))
    return toks, probs


class _Options(ctypes.Structure):
    _fields_ = [("n_devices", ctypes.c_int), ("devices", ctypes.POINTER(ctypes.c_int))]


class Context:
    """One process's view of the GPUs it drives (mc_open)."""

    def __init__(self, devices: Sequence[int] = (0,)):
        self.devices = list(devices)
        arr = (ctypes.c_int * len(self.devices))(*self.devices)
        opt = _Options(len(self.devices), arr)
        h = c_vp()
        _lib.check(_lib.lib().mc_open(ctypes.byref(opt), ctypes.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().mc_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except (AttributeError, TypeError):  # interpreter shutdown: the module globals are gone
            pass


_default_ctx: Optional[Context] = None


def default_context() -> Context:
    global _default_ctx
    if _default_ctx is None:
        _default_ctx = Context((0,))
    return _default_ctx


class Model:
    """An INT8 model replicated on the context's GPUs."""

    def __init__(self, handle, ctx: Context):
        self._h = handle
        self.ctx = ctx
        info = np.zeros(10, np.int32)
        _lib.check(_lib.lib().mc_model_info(self._h, _lib.ptr(info)))
        (self.vocab, self.state, self.hidden, self.blocks, self.max_context, self.attn_heads, self.attn_window,
         self.total_steps, self.ring, self.attn_cache) = [int(v) for v in info]

    @classmethod
    def decode(cls, data: bytes, ctx: Optional[Context] = None) -> "Model":
        ctx = ctx or default_context()
        h = c_vp()
        _lib.check(_lib.lib().mc_load_model(ctx._h, data, len(data), ctypes.byref(h)))
        return cls(h, ctx)

    @classmethod
    def load(cls, path: str, ctx: Optional[Context] = None) -> "Model":
        with open(path, "rb") as f:
            return cls.decode(f.read(), ctx)

    @classmethod
    def decode_full(cls, data: bytes, max_context: int = 0, ctx: Optional[Context] = None) -> "Model":
        """A full-precision model file quantized on the GPU: pkg/model.Decode then
        quant.Quantize (internal/quant/convert.go:8-98) with maxContext = max_context (<= 0: the
        file's context size)."""
        ctx = ctx or default_context()
        h = c_vp()
        _lib.check(_lib.lib().mc_load_model_full(ctx._h, data, len(data), max_context, ctypes.byref(h)))
        return cls(h, ctx)

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().mc_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except (AttributeError, TypeError):  # interpreter shutdown: the module globals are gone
            pass

    def vocab_size(self) -> int:
        return self.vocab

    def state_size(self) -> int:
        return self.state

    def hidden_size(self) -> int:
        return self.hidden

    def num_blocks(self) -> int:
        return self.blocks

    def new_batch(self, count: int, context_size: int = 0, max_prompt: int = 128, top_k: int = 0) -> "SessionBatch":
        return SessionBatch(self, count, context_size, max_prompt, top_k)

    def new_session(self, context_size: int) -> "Session":
        return Session(self, context_size)

    def call(self, window: Sequence[int]) -> Optional[np.ndarray]:
        """Logits after the last token of window (most recent max_context tokens kept)."""
        if len(window) == 0:
            return None
        w = np.asarray(window, np.int32)[-self.max_context:]
        b = self.new_batch(1, 0, len(w))
        logits, _, _ = b.prefill(w[None, :], [len(w)], want_logits=True)
        b.close()
        return logits[0].astype(np.float64)

    forward = call


class SessionBatch:
    """count sessions of one model, stepped together on the GPU(s)."""

    def __init__(self, model: Model, count: int, context_size: int, max_prompt: int, top_k: int):
        self.model = model
        self.count = count
        h = c_vp()
        _lib.check(_lib.lib().mc_batch_open(model._h, count, context_size, max_prompt, top_k, ctypes.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().mc_batch_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except (AttributeError, TypeError):  # interpreter shutdown: the module globals are gone
            pass

    def prefill(self, prompts, lens, want_logits: bool = False):
        p = np.ascontiguousarray(prompts, np.int32)
        if p.ndim == 1:
            p = p[None, :]
        lens = np.ascontiguousarray(lens, np.int32)
        logits = np.zeros((self.count, self.model.vocab), np.float32) if want_logits else None
        nxt = np.zeros(self.count, np.int32)
        prob = np.zeros(self.count, np.float32)
        _lib.check(_lib.lib().mc_prefill(self._h, _lib.ptr(p), _lib.ptr(lens), p.shape[1], _lib.ptr(logits),
                                         _lib.ptr(nxt), _lib.ptr(prob)))
        return logits, nxt, prob

    def append(self, tokens, want_logits: bool = False):
        t = np.ascontiguousarray(tokens, np.int32)
        logits = np.zeros((self.count, self.model.vocab), np.float32) if want_logits else None
        nxt = np.zeros(self.count, np.int32)
        prob = np.zeros(self.count, np.float32)
        _lib.check(_lib.lib().mc_append(self._h, _lib.ptr(t), _lib.ptr(logits), _lib.ptr(nxt), _lib.ptr(prob)))
        return logits, nxt, prob

    def score(self, seqs, lens=None):
        """Per-token log-probabilities: out[s, t] = log p(seqs[s, t+1] | seqs[s, :t+1]) for
        t < lens[s] - 1 (eval.logProb over every prefix, one prefill pass); other entries 0."""
        q = np.ascontiguousarray(seqs, np.int32)
        if q.ndim == 1:
            q = q[None, :]
        lens = np.full(self.count, q.shape[1], np.int32) if lens is None else np.ascontiguousarray(lens, np.int32)
        out = np.zeros((self.count, max(q.shape[1] - 1, 0)), np.float64)
        _lib.check(_lib.lib().mc_score(self._h, _lib.ptr(q), _lib.ptr(lens), q.shape[1], _lib.ptr(out)))
        return out

    def score_targets(self, seqs, targets, lens=None):
        """Per-position log-probabilities of given targets: out[s, t] = log p(targets[s, t] |
        seqs[s, :t+1]) for t < lens[s] (nll.score, internal/eval/eval.go:27-43); other entries 0."""
        q = np.ascontiguousarray(seqs, np.int32)
        tg = np.ascontiguousarray(targets, np.int32)
        if q.ndim == 1:
            q, tg = q[None, :], tg[None, :]
        if tg.shape != q.shape:
            raise ValueError("targets must have the shape of seqs")
        lens = np.full(self.count, q.shape[1], np.int32) if lens is None else np.ascontiguousarray(lens, np.int32)
        out = np.zeros((self.count, q.shape[1]), np.float64)
        _lib.check(_lib.lib().mc_score_targets(self._h, _lib.ptr(q), _lib.ptr(lens), q.shape[1], _lib.ptr(tg),
                                               _lib.ptr(out)))
        return out

    def generate(self, prompts, lens, n_new: int, temperature: float = 0.0, session0: int = 0, stops=None):
        """n_new tokens per session after its prompt (greedy, or sampled with temperature > 0):
        (tokens, probs). With stops (at most 8 token ids): each session ends before the first stop
        token it would emit, as greedyLoop does (generate/greedy.go:63-87); returns (tokens, probs,
        lengths) with -1 / 0 past each session's length."""
        p = np.ascontiguousarray(prompts, np.int32)
        lens = np.ascontiguousarray(lens, np.int32)
        toks = np.zeros((self.count, n_new), np.int32)
        probs = np.zeros((self.count, n_new), np.float32)
        if stops is None:
            _lib.check(_lib.lib().mc_generate(self._h, _lib.ptr(p), _lib.ptr(lens), p.shape[1], n_new, temperature,
                                              session0, _lib.ptr(toks), _lib.ptr(probs)))
            return toks, probs
        st = np.ascontiguousarray(list(stops), np.int32)
        out_lens = np.zeros(self.count, np.int32)
        _lib.check(_lib.lib().mc_generate_stops(self._h, _lib.ptr(p), _lib.ptr(lens), p.shape[1], n_new, temperature,
                                                session0, _lib.ptr(st) if st.size else None, int(st.size),
                                                _lib.ptr(toks), _lib.ptr(probs), _lib.ptr(out_lens)))
        return toks, probs, out_lens

    def generate_limits(self, prompts, lens, max_tokens, temperature: float = 0.0, session0: int = 0):
        """max_tokens[s] tokens for session s after its prompt (pkg/infer.Generate's MaxTokens per
        session; greedy, or sampled with temperature > 0 like ``generate``): (tokens, probs,
        lengths), tokens [count x max(max_tokens)] with -1 past each session's limit."""
        p = np.ascontiguousarray(prompts, np.int32)
        lens = np.ascontiguousarray(lens, np.int32)
        lim = np.ascontiguousarray(max_tokens, np.int32)
        n_max = int(lim.max())
        toks = np.zeros((self.count, n_max), np.int32)
        probs = np.zeros((self.count, n_max), np.float32)
        out_lens = np.zeros(self.count, np.int32)
        _lib.check(_lib.lib().mc_generate_limits(self._h, _lib.ptr(p), _lib.ptr(lens), p.shape[1], _lib.ptr(lim), n_max,
                                                 temperature, session0, _lib.ptr(toks), _lib.ptr(probs),
                                                 _lib.ptr(out_lens)))
        return toks, probs, out_lens

    def generate_policy(self, prompts, lens, n_new: int, sampling: Sampling, penalize_prompt: bool = False,
                        dfa=None, dfa_start=None, session0: int = 0, stops=()):
        """sampleContinuation (internal/generate/sample.go:196-247) for every session, the whole
        policy on the device: (tokens, probs, lengths), -1 / 0 past each session's length.
        ``penalize_prompt`` makes the prompt the penalty prefix (chat.go:72); ``dfa``
        [n_states x vocab] (next state, -1 = not allowed) with ``dfa_start`` [count] is the
        constraint automaton."""
        p = np.ascontiguousarray(prompts, np.int32)
        lens = np.ascontiguousarray(lens, np.int32)
        toks = np.zeros((self.count, n_new), np.int32)
        probs = np.zeros((self.count, n_new), np.float32)
        out_lens = np.zeros(self.count, np.int32)
        st = np.ascontiguousarray(list(stops), np.int32)
        d = ds = None
        n_states = 0
        if dfa is not None:
            d = np.ascontiguousarray(dfa, np.int32)
            n_states = d.shape[0]
            ds = np.ascontiguousarray(dfa_start, np.int32)
        _lib.check(_lib.lib().mc_generate_policy(self._h, _lib.ptr(p), _lib.ptr(lens), p.shape[1], n_new,
                                                 ctypes.byref(sampling), int(bool(penalize_prompt)), _lib.ptr(d),
                                                 n_states, _lib.ptr(ds), session0, _lib.ptr(st) if st.size else None,
                                                 int(st.size), _lib.ptr(toks), _lib.ptr(probs), _lib.ptr(out_lens)))
        return toks, probs, out_lens


class Scheduler:
    """Continuous batching over ``slots`` GPU session slots (mc_sched_*): requests queue on the
    host, are admitted into free slots by prefill passes while the other slots keep their state,
    and decode together; each ends at its own ``n_new`` or a stop token. Every request runs
    sampleContinuation (internal/generate/sample.go:196-247) with ``sampling``; its draws are
    keyed by ``draw_key`` (default: its id) and its token index, so its tokens do not depend on
    the slot it ran in or on the other requests."""

    def __init__(self, model: Model, slots: int, sampling: Optional[Sampling] = None, context_size: int = 0,
                 max_prompt: int = 128, max_new: int = 128, penalize_prompt: bool = False, stops=()):
        sampling = sampling if sampling is not None else Sampling()
        st = np.ascontiguousarray(list(stops), np.int32)
        h = c_vp()
        _lib.check(_lib.lib().mc_sched_open(model._h, slots, context_size, max_prompt, max_new, ctypes.byref(sampling),
                                            int(bool(penalize_prompt)), _lib.ptr(st) if st.size else None,
                                            int(st.size), ctypes.byref(h)))
        self._h = h
        self.model = model
        self.max_new = max_new
        self._submitted = 0

    def close(self):
        if self._h:
            _lib.lib().mc_sched_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except (AttributeError, TypeError):  # interpreter shutdown: the module globals are gone
            pass

    def submit(self, prompt: Sequence[int], n_new: int, draw_key: Optional[int] = None) -> int:
        """Queues a request; returns its id."""
        p = np.ascontiguousarray(list(prompt), np.int32)
        rid = ctypes.c_int64()
        key = self._submitted if draw_key is None else draw_key
        _lib.check(_lib.lib().mc_sched_submit(self._h, _lib.ptr(p) if p.size else None, int(p.size), int(n_new),
                                              ctypes.c_uint32(key & 0xFFFFFFFF), ctypes.byref(rid)))
        self._submitted += 1
        return int(rid.value)

    def step(self, steps: int = 8) -> int:
        """One round (admission where due, ``steps`` decode steps, collection); returns the
        number of requests still queued or running."""
        left = _i()
        _lib.check(_lib.lib().mc_sched_step(self._h, steps, ctypes.byref(left)))
        return int(left.value)

    def run(self, steps_per_poll: int = 8):
        _lib.check(_lib.lib().mc_sched_run(self._h, steps_per_poll))

    def set_admit_min(self, admit_min: int):
        _lib.check(_lib.lib().mc_sched_set_admit_min(self._h, admit_min))

    def result(self, rid: int):
        """(tokens, probs) of a finished request, None while it is queued or running."""
        n = _i()
        toks = np.zeros(self.max_new, np.int32)
        probs = np.zeros(self.max_new, np.float32)
        _lib.check(_lib.lib().mc_sched_result(self._h, rid, _lib.ptr(toks), _lib.ptr(probs), self.max_new,
                                              ctypes.byref(n)))
        if n.value < 0:
            return None
        return toks[:n.value].copy(), probs[:n.value].copy()

    def stats(self) -> dict:
        out = np.zeros(10, np.int64)
        _lib.check(_lib.lib().mc_sched_stats(self._h, _lib.ptr(out)))
        return dict(zip(("prefill_passes", "decode_steps", "tokens", "finished", "in_flight", "admit_us", "decode_us",
                         "step_us", "admit_host_us", "admitted"), map(int, out)))


class Session:
    """quantSession (internal/quant/session.go:11-68) on a one-session batch: a window of the most
    recent tokens, rebuilt by a prefill when the session was never prefilled."""

    def __init__(self, model: Model, context_size: int):
        self.model = model
        window = model.max_context
        if 0 < context_size < window:
            window = context_size
        self.window = window
        self._batch = model.new_batch(1, context_size, min(window, 128))
        self.tokens: list = []
        self.fed = 0
        self.n = 0

    def prefill(self, tokens: Sequence[int]) -> Optional[np.ndarray]:
        tokens = list(tokens)[-self.window:] if len(tokens) > self.window else list(tokens)
        self.tokens = tokens
        if not tokens:
            return None
        return self._prefill()

    def _prefill(self) -> np.ndarray:
        self.fed = len(self.tokens)
        t = np.asarray(self.tokens, np.int32)
        logits, _, _ = self._batch.prefill(t[None, :], [len(t)], want_logits=True)
        self.n = len(t)
        return logits[0].astype(np.float64)

    def append(self, token: int) -> np.ndarray:
        self.tokens.append(int(token))
        if len(self.tokens) > self.window:
            self.tokens = self.tokens[1:]
        if self.fed == 0 or self.n != self.fed:
            return self._prefill()
        logits, _, _ = self._batch.append(np.array([token], np.int32), want_logits=True)
        self.n += 1
        self.fed += 1
        return logits[0].astype(np.float64)

    def close(self):
        self._batch.close()


def greedy_continuation(sess: Session, context: Sequence[int], max_tokens: int, stops: Sequence[int] = ()):
    """generate.greedyLoop (internal/generate/greedy.go:63-87) over a Session: ids and the
    probability of each (argmaxProb, :90-102)."""
    ids, probs = [], []
    logits = sess.prefill(context)
    while len(ids) < max_tokens and logits is not None and len(logits) > 0:
        best = int(np.argmax(logits))  # first index of the maximum
        prob = 1.0 / float(np.sum(np.exp(logits - logits[best])))
        if best in stops:
            break
        ids.append(best)
        probs.append(prob)
        if len(ids) < max_tokens:
            logits = sess.append(best)
    return ids, probs


class HeldOut:
    """eval.HeldOut (internal/eval/eval.go): mean loss in nats per scored token, perplexity
    exp(loss), bits per byte (when token byte lengths are given) and the number of tokens."""

    def __init__(self, nats: float = 0.0, tokens: int = 0, nbytes: int = 0, with_bytes: bool = False):
        self.tokens = tokens
        self.loss = nats / tokens if tokens else 0.0
        self.ppl = float(np.exp(self.loss)) if tokens else 0.0
        self.bpb = (nats / np.log(2.0) / nbytes if nbytes else 0.0) if with_bytes and tokens else None

    def __repr__(self):
        return f"HeldOut(loss={self.loss:.6f}, ppl={self.ppl:.4f}, bpb={self.bpb}, tokens={self.tokens})"


def _nll(model: "Model", streams, context_size: int, token_bytes=None, batch_size: int = 1024) -> HeldOut:
    """nll.score (internal/eval/eval.go:27-43) over token streams, from position 1 to the end:
    token t is predicted from window(stream[:t], context_size), the last context_size tokens.
    Targets t <= context_size share one prefix pass per stream; each later target gets its own
    window of context_size tokens. The windows run batch_size at a time on the engine."""
    V = model.vocab
    ctx = min(int(context_size), model.max_context)
    jobs = []  # (sequence, targets, positions to read)
    for T in streams:
        T = np.asarray(T, np.int64)
        L = len(T)
        if L < 2:
            continue
        n = min(L - 1, ctx)
        jobs.append((T[:n], T[1:n + 1], np.arange(n)))
        for t in range(ctx + 1, L):
            w = T[t - ctx:t]
            jobs.append((w, np.concatenate([T[t - ctx + 1:t], T[t:t + 1]]), np.array([ctx - 1])))
    nats, count, nbytes = 0.0, 0, 0
    batch = model.new_batch(max(1, min(batch_size, len(jobs))), ctx, ctx)
    try:
        for j0 in range(0, len(jobs), batch.count):
            chunk = jobs[j0:j0 + batch.count]
            seqs = np.zeros((batch.count, ctx), np.int32)
            tgts = np.zeros((batch.count, ctx), np.int32)
            lens = np.zeros(batch.count, np.int32)
            for i, (q, tg, _) in enumerate(chunk):
                seqs[i, :len(q)] = q
                tgts[i, :len(q)] = np.clip(tg, 0, V - 1)  # out-of-range targets are skipped below
                lens[i] = len(q)
            lp = batch.score_targets(seqs, tgts, lens)
            for i, (q, tg, read) in enumerate(chunk):
                for p in read:
                    target = int(tg[p])
                    if 0 <= target < V:  # the reference skips targets outside the logits
                        nats -= float(lp[i, p])
                        count += 1
                        if token_bytes is not None:
                            nbytes += int(token_bytes[target])
    finally:
        batch.close()
    return HeldOut(nats, count, nbytes, token_bytes is not None)


def perplexity(model: "Model", tokens: Sequence[int], context_size: int, max_tokens: int = 0, token_bytes=None,
               batch_size: int = 1024) -> HeldOut:
    """eval.Perplexity (internal/eval/eval.go:49-62) on an already tokenized text: one continuous
    stream, every token after the first predicted from the context_size tokens before it (at most
    max_tokens of them when > 0). token_bytes[id]: the byte length of each token, for bits per byte."""
    T = list(tokens)
    if len(T) < 2:
        return HeldOut()
    n = len(T) - 1
    if max_tokens > 0 and n > max_tokens:
        n = max_tokens
    return _nll(model, [T[:n + 1]], context_size, token_bytes, batch_size)


def perplexity_per_doc(model: "Model", docs: Sequence[Sequence[int]], context_size: int, eos_id: int,
                       max_docs: int = 0, token_bytes=None, batch_size: int = 1024) -> HeldOut:
    """eval.PerplexityPerDoc (internal/eval/perdoc.go:16-32) on already tokenized documents: each
    document scored on its own, starting from EOS, every token of it (the first included)."""
    docs = list(docs)
    if max_docs > 0:
        docs = docs[:max_docs]
    return _nll(model, [[eos_id] + list(d) for d in docs], context_size, token_bytes, batch_size)
