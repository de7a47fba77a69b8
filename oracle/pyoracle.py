"""ctypes binding of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Loaded by tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``; never by
the product package. The oracle restates the reference's Go INT8 engine (see ``oracle.h``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i8p = ctypes.POINTER(ctypes.c_int8)


class Sampling(ctypes.Structure):
    """or_sampling: the knobs of generate.Sampling (internal/generate/chat.go:45-56)."""
    _fields_ = [("temperature", ctypes.c_double), ("rep_penalty", ctypes.c_double), ("top_k", ctypes.c_int),
                ("top_p", ctypes.c_double), ("rep_window", ctypes.c_int), ("ban_trigrams", ctypes.c_int)]

    def __init__(self, temperature=0.0, rep_penalty=1.0, top_k=0, top_p=1.0, rep_window=0, ban_trigrams=0):
        super().__init__(float(temperature), float(rep_penalty), int(top_k), float(top_p), int(rep_window),
                         int(ban_trigrams))


def build(force: bool = False) -> str:
    """Builds liboracle.so with the committed Makefile (the system gcc)."""
    if force or not os.path.exists(_LIB_PATH) or any(
            os.path.getmtime(os.path.join(_HERE, f)) > os.path.getmtime(_LIB_PATH)
            for f in os.listdir(_HERE) if f.endswith((".c", ".h", "Makefile"))):
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "liboracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        L.or_dot_i8_f32.restype = ctypes.c_float
        L.or_dot_i8_f32.argtypes = [_f32p, _i8p, ctypes.c_int]
        L.or_dot_i8_f32_scalar_order.restype = ctypes.c_float
        L.or_dot_i8_f32_scalar_order.argtypes = [_f32p, _i8p, ctypes.c_int]
        L.or_dot_f32.restype = ctypes.c_float
        L.or_dot_f32.argtypes = [_f32p, _f32p, ctypes.c_int]
        L.or_dot_f32_scalar_order.restype = ctypes.c_float
        L.or_dot_f32_scalar_order.argtypes = [_f32p, _f32p, ctypes.c_int]
        L.or_add_scaled_f32.argtypes = [_f32p, _f32p, ctypes.c_float, ctypes.c_int]
        L.or_vec_exp_f32.argtypes = [_f32p, _f32p, ctypes.c_int]
        L.or_fast_exp_f32.restype = ctypes.c_float
        L.or_fast_exp_f32.argtypes = [ctypes.c_float]
        L.or_matvec_i8.argtypes = [_f32p, ctypes.c_int, _i8p, ctypes.c_int, ctypes.c_float, _f32p, ctypes.c_int, _f32p]
        L.or_sigmoid_clamped.restype = ctypes.c_float
        L.or_sigmoid_clamped.argtypes = [ctypes.c_float]
        L.or_step_dilation.restype = ctypes.c_int
        L.or_step_dilation.argtypes = [ctypes.c_int] * 3
        L.or_latch_base_logits.argtypes = [ctypes.c_int, _f32p]
        L.or_quantize_tensor.restype = ctypes.c_float
        L.or_quantize_tensor.argtypes = [_f32p, ctypes.c_size_t, _i8p]
        L.or_model_decode.restype = ctypes.c_void_p
        L.or_model_decode.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
        L.or_model_free.argtypes = [ctypes.c_void_p]
        L.or_model_info.argtypes = [ctypes.c_void_p, _i32p]
        L.or_model_dilations.argtypes = [ctypes.c_void_p, _i32p]
        L.or_model_call.restype = ctypes.c_int
        L.or_model_call.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int, _f32p]
        L.or_session_new.restype = ctypes.c_void_p
        L.or_session_new.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.or_session_free.argtypes = [ctypes.c_void_p]
        L.or_session_prefill.restype = ctypes.c_int
        L.or_session_prefill.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int, _f32p]
        L.or_session_append.restype = ctypes.c_int
        L.or_session_append.argtypes = [ctypes.c_void_p, ctypes.c_int32, _f32p]
        L.or_session_state_bytes.restype = ctypes.c_long
        L.or_session_state_bytes.argtypes = [ctypes.c_void_p]
        L.or_session_position.restype = ctypes.c_int
        L.or_session_position.argtypes = [ctypes.c_void_p]
        L.or_argmax_prob.restype = ctypes.c_int
        L.or_argmax_prob.argtypes = [_f32p, ctypes.c_int, _f64p]
        L.or_log_prob.restype = ctypes.c_double
        L.or_log_prob.argtypes = [_f32p, ctypes.c_int, ctypes.c_int]
        L.or_philox4x32.argtypes = [ctypes.POINTER(ctypes.c_uint32)] * 3
        L.or_sample_uniform.restype = ctypes.c_double
        L.or_sample_uniform.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        L.or_sample_topk.restype = ctypes.c_int
        L.or_sample_topk.argtypes = [_f32p, ctypes.c_int, ctypes.c_double, ctypes.c_int, ctypes.c_double]
        L.or_generate_greedy.restype = ctypes.c_int
        L.or_generate_greedy.argtypes = [ctypes.c_void_p, ctypes.c_int, _i32p, ctypes.c_int, _i32p, ctypes.c_int,
                                         ctypes.c_int, _i32p, _f32p, _f32p, ctypes.c_int]
        L.or_generate_sample.restype = ctypes.c_int
        L.or_generate_sample.argtypes = [ctypes.c_void_p, ctypes.c_int, _i32p, ctypes.c_int, _i32p, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_double, ctypes.c_int, ctypes.c_uint32, _i32p, _f32p,
                                         ctypes.c_int]
        L.or_sample_policy.restype = ctypes.c_int
        L.or_sample_policy.argtypes = [_f64p, ctypes.c_int, _i32p, ctypes.c_int, _i32p, ctypes.c_int,
                                       ctypes.POINTER(Sampling), _i32p, ctypes.c_double, _f64p]
        L.or_generate_policy.restype = ctypes.c_int
        L.or_generate_policy.argtypes = [ctypes.c_void_p, ctypes.c_int, _i32p, ctypes.c_int, _i32p, ctypes.c_int,
                                         ctypes.c_int, ctypes.POINTER(Sampling), ctypes.c_int, _i32p, _i32p,
                                         ctypes.c_uint32, _i32p, ctypes.c_int, _i32p, _f32p, _i32p, _f32p,
                                         ctypes.c_int]
        L.or_score.restype = ctypes.c_int
        L.or_score.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _i32p, _f64p, ctypes.c_int]
        L.or_set_avx2.argtypes = [ctypes.c_int]
        L.or_get_avx2.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def i8(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int8)


class Model:
    """A decoded INT8 model (quant.Decode)."""

    def __init__(self, data: bytes):
        err = ctypes.create_string_buffer(256)
        self._h = lib().or_model_decode(data, len(data), err, 256)
        if not self._h:
            raise ValueError(err.value.decode())
        info = np.zeros(10, dtype=np.int32)
        lib().or_model_info(self._h, _p(info, _i32p))
        (self.vocab, self.state, self.hidden, self.blocks, self.max_context, self.attn_heads,
         self.attn_window, self.ring, self.attn_cache, self.total_steps) = [int(x) for x in info]

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_model_free(self._h)
            self._h = None

    def dilations(self) -> np.ndarray:
        out = np.zeros(self.total_steps, dtype=np.int32)
        lib().or_model_dilations(self._h, _p(out, _i32p))
        return out

    def call(self, window) -> np.ndarray | None:
        w = i32(window)
        out = np.zeros(self.vocab, dtype=np.float32)
        if lib().or_model_call(self._h, _p(w, _i32p), w.size, _p(out, _f32p)) != 0:
            return None
        return out

    def new_session(self, context_size: int) -> "Session":
        return Session(self, context_size)

    def generate_greedy(self, prompts, lens, n_new, context_size=0, logits=False, nthreads=0):
        prompts = i32(prompts)
        lens = i32(lens)
        n = prompts.shape[0]
        toks = np.zeros((n, n_new), dtype=np.int32)
        probs = np.zeros((n, n_new), dtype=np.float32)
        lg = np.zeros((n, n_new, self.vocab), dtype=np.float32) if logits else None
        lib().or_generate_greedy(self._h, n, _p(prompts, _i32p), prompts.shape[1], _p(lens, _i32p), context_size,
                                 n_new, _p(toks, _i32p), _p(probs, _f32p),
                                 _p(lg, _f32p) if lg is not None else None, nthreads)
        return toks, probs, lg

    def generate_sample(self, prompts, lens, n_new, temperature, topk, session0=0, context_size=0,
                        logits=False, nthreads=0):
        prompts = i32(prompts)
        lens = i32(lens)
        n = prompts.shape[0]
        toks = np.zeros((n, n_new), dtype=np.int32)
        lg = np.zeros((n, n_new, self.vocab), dtype=np.float32) if logits else None
        lib().or_generate_sample(self._h, n, _p(prompts, _i32p), prompts.shape[1], _p(lens, _i32p), context_size,
                                 n_new, temperature, topk, session0, _p(toks, _i32p),
                                 _p(lg, _f32p) if lg is not None else None, nthreads)
        return toks, lg

    def generate_policy(self, prompts, lens, n_new, sampling: Sampling, penalize_prompt=False, dfa=None,
                        dfa_start=None, session0=0, stops=(), context_size=0, logits=False, nthreads=0):
        """sampleContinuation per session: tokens [n x n_new] (-1 after a session ends), probs,
        lengths and (logits=True) the float32 logits each token was drawn from."""
        prompts = i32(prompts)
        lens = i32(lens)
        n = prompts.shape[0]
        toks = np.zeros((n, n_new), dtype=np.int32)
        probs = np.zeros((n, n_new), dtype=np.float32)
        out_lens = np.zeros(n, dtype=np.int32)
        st = i32(list(stops) or [0])
        d = i32(dfa) if dfa is not None else None
        ds = i32(dfa_start) if dfa is not None else None
        lg = np.zeros((n, n_new, self.vocab), dtype=np.float32) if logits else None
        lib().or_generate_policy(self._h, n, _p(prompts, _i32p), prompts.shape[1], _p(lens, _i32p), context_size,
                                 n_new, ctypes.byref(sampling), int(penalize_prompt),
                                 _p(d, _i32p) if d is not None else None, _p(ds, _i32p) if ds is not None else None,
                                 session0, _p(st, _i32p), len(stops), _p(toks, _i32p), _p(probs, _f32p),
                                 _p(out_lens, _i32p), _p(lg, _f32p) if lg is not None else None, nthreads)
        return toks, probs, out_lens, lg

    def score(self, seqs, nthreads=0) -> np.ndarray:
        seqs = i32(seqs)
        n, L = seqs.shape
        out = np.zeros((n, L - 1), dtype=np.float64)
        lib().or_score(self._h, n, L, _p(seqs, _i32p), _p(out, _f64p), nthreads)
        return out


class Session:
    """quantSession (internal/quant/session.go:11-68)."""

    def __init__(self, model: Model, context_size: int):
        self.model = model
        self._h = lib().or_session_new(model._h, context_size)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_session_free(self._h)
            self._h = None

    def prefill(self, tokens):
        t = i32(tokens)
        out = np.zeros(self.model.vocab, dtype=np.float32)
        if lib().or_session_prefill(self._h, _p(t, _i32p), t.size, _p(out, _f32p)) == 0:
            return None
        return out

    def append(self, token: int):
        out = np.zeros(self.model.vocab, dtype=np.float32)
        lib().or_session_append(self._h, int(token), _p(out, _f32p))
        return out

    def state_bytes(self) -> int:
        return int(lib().or_session_state_bytes(self._h))

    def position(self) -> int:
        return int(lib().or_session_position(self._h))


def dot_i8_f32(x, w, n=None) -> float:
    x, w = f32(x), i8(w)
    n = min(x.size, w.size) if n is None else n
    return float(lib().or_dot_i8_f32(_p(x, _f32p), _p(w, _i8p), n))


def dot_f32(x, y) -> float:
    x, y = f32(x), f32(y)
    return float(lib().or_dot_f32(_p(x, _f32p), _p(y, _f32p), min(x.size, y.size)))


def matvec_i8(w, rows, stride, scale, x, bias=None) -> np.ndarray:
    w, x = i8(w), f32(x)
    y = np.zeros(rows, dtype=np.float32)
    b = f32(bias) if bias is not None else None
    lib().or_matvec_i8(_p(y, _f32p), rows, _p(w, _i8p), stride, scale, _p(x, _f32p), x.size,
                       _p(b, _f32p) if b is not None else None)
    return y


def quantize(w):
    w = f32(w)
    out = np.zeros(w.size, dtype=np.int8)
    s = lib().or_quantize_tensor(_p(w, _f32p), w.size, _p(out, _i8p))
    return out, np.float32(s)


def argmax_prob(logits):
    l = f32(logits)
    p = ctypes.c_double()
    b = lib().or_argmax_prob(_p(l, _f32p), l.size, ctypes.byref(p))
    return int(b), float(p.value)


def log_prob(logits, idx) -> float:
    l = f32(logits)
    return float(lib().or_log_prob(_p(l, _f32p), l.size, int(idx)))


def sample_topk(logits, temperature, topk, u) -> int:
    l = f32(logits)
    return int(lib().or_sample_topk(_p(l, _f32p), l.size, temperature, topk, u))


def sample_policy(logits, sampling: Sampling, prefix=(), gen=(), allowed=None, u=0.5):
    """One step of sampleContinuation over float64 logits: (token, probability)."""
    l = np.array(logits, dtype=np.float64)
    pre = i32(list(prefix) or [0])
    g = i32(list(gen) or [0])
    a = i32(allowed) if allowed is not None else None
    p = ctypes.c_double()
    t = lib().or_sample_policy(_p(l, _f64p), l.size, _p(pre, _i32p), len(prefix), _p(g, _i32p), len(gen),
                               ctypes.byref(sampling), _p(a, _i32p) if a is not None else None, float(u),
                               ctypes.byref(p))
    return int(t), float(p.value)


def philox(ctr, key):
    c = (ctypes.c_uint32 * 4)(*ctr)
    k = (ctypes.c_uint32 * 2)(*key)
    o = (ctypes.c_uint32 * 4)()
    lib().or_philox4x32(c, k, o)
    return list(o)
