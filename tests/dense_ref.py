"""A float64, layer-major restatement of the Hybrid-NCA forward pass on dequantized weights.

It plays the part of the full-precision engine in the reference's
TestQuantizedMatchesDequantized (internal/quant/equivalence_test.go:75-98): an independent
statement of the same mathematics (the dense forward of internal/ca/forward.go computes every
position of a step at once), so the INT8 engines can be checked against it within 1e-3.
"""
import numpy as np

from mignon_ai_b200 import synth


def _sig(x):
    out = 1.0 / (1.0 + np.exp(-np.clip(x, -30, 30)))
    out = np.where(x > 15.0, 1.0, out)
    return np.where(x < -15.0, 0.0, out)


def _rms(x, g):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + 1e-5) * g


def _deq(t):
    return synth.dequantize_tensor(t.data, t.scale).astype(np.float64)


def latch_base(D):
    minT, maxT = 1.5, 64.0
    out = np.zeros(D)
    for d in range(D):
        td = minT if D == 1 else minT * (maxT / minT) ** (d / (D - 1))
        lam = float(np.float32(2.0 ** (-1.0 / td)))
        out[d] = np.log(lam / (1 - lam))
    return out


def forward_all(m: synth.QModel, tokens, max_context=None):
    """Logits (float64) after every position of one sequence (tokens trimmed like prefill)."""
    D, H, V = m.state, m.hidden, m.vocab
    ctx = m.context if m.context >= 64 else 128
    if max_context is not None:
        ctx = max_context
    tokens = np.asarray(tokens)[-ctx:]
    N = len(tokens)
    E = _deq(m.embed).reshape(V, D)
    tok = np.where((tokens < 0) | (tokens >= V), 0, tokens)
    cur = E[tok].copy()
    block_in = cur.copy()
    base = latch_base(D)
    for bi, b in enumerate(m.blocks):
        if bi > 0:
            block_in = block_in + cur
            cur = block_in.copy()
        W1 = _deq(b.w1).reshape(2 * H, 3 * D)
        W2 = _deq(b.w2).reshape(2 * D, H)
        Ws = _deq(b.wsel).reshape(D, D)
        for step in range(b.cfg.steps):
            dil = synth.step_dilation(b.cfg.initial_dilation, b.cfg.dilation_base, step)
            n = _rms(cur, b.gamma.astype(np.float64)) if len(b.gamma) == D else cur.copy()
            lam = _sig(n @ Ws.T + base)
            latch = np.zeros_like(n)
            l = np.zeros(D)
            for t in range(N):
                l = lam[t] * l + (1 - lam[t]) * n[t]
                latch[t] = l
            left = np.zeros_like(n)
            if dil < N:
                left[dil:] = n[:-dil]
            x = np.concatenate([n, left, latch], axis=1)
            a = x @ W1.T + b.b1
            hid = a[:, :H] * _sig(a[:, H:])
            o = hid @ W2.T + b.b2
            g = _sig(o[:, D:])
            cur = (1 - g) * cur + g * o[:, :D]
        if b.qkv is not None:
            heads = m.attn_heads
            dh = D // heads
            cache = m.attn_window if m.attn_window > 0 else ctx
            na = _rms(cur, b.attn_norm.astype(np.float64))
            qkv = na @ _deq(b.qkv).reshape(3 * D, D).T
            q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
            att = np.zeros_like(cur)
            for t in range(N):
                lo = max(0, t - cache + 1)
                if m.attn_window > 0:
                    lo = max(lo, t - m.attn_window + 1)
                for h in range(heads):
                    sl = slice(h * dh, (h + 1) * dh)
                    s = k[lo:t + 1, sl] @ q[t, sl] / np.sqrt(dh)
                    p = np.exp(s - s.max())
                    p /= p.sum()
                    att[t, sl] = p @ v[lo:t + 1, sl]
            cur = cur + att @ _deq(b.out).reshape(D, D).T
    c = _rms(cur, m.final_norm.astype(np.float64)) if len(m.final_norm) == D else cur
    Wh = E if m.tied else _deq(m.head_w).reshape(V, D)
    return c @ Wh.T + m.head_b
