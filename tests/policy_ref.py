"""A plain-Python statement of the reference's decode-loop policy, for the policy tests.

py_policy follows sampleContinuation's loop body and SampleRawLogitsAdvanced line by line
(internal/generate/sample.go:213-231, :33-172, :174-191; ties in the descending sort go to the
lower index); policy_margin says how close a case lies to a decision edge, so that a stream that
leaves another engine's can be excused only there.
"""
import math

import numpy as np

NEG_MAX = -1.7976931348623157e308


def py_policy(logits, sp, prefix=(), gen=(), allowed=None, u=0.5):
    """sampleContinuation's loop body then SampleRawLogitsAdvanced, in plain Python
    (sample.go:213-231, :33-172, :174-191); ties in the descending sort go to the lower index."""
    l = [float(x) for x in logits]
    V = len(l)
    gen = list(gen)
    if sp.ban_trigrams and len(gen) >= 2:
        w1, w2 = gen[-2], gen[-1]
        for i in range(len(gen) - 2):
            if gen[i] == w1 and gen[i + 1] == w2 and 0 <= gen[i + 2] < V:
                l[gen[i + 2]] = NEG_MAX
    if allowed is not None:
        for i in range(V):
            if allowed[i] < 0:
                l[i] = -1e300
    recent = list(prefix) + gen
    if sp.rep_window > 0:
        recent = recent[-sp.rep_window:]
    if sp.rep_penalty > 1.0:
        for i, tok in enumerate(recent):
            if tok < 0 or tok >= V or tok in recent[:i]:
                continue
            l[tok] = l[tok] / sp.rep_penalty if l[tok] > 0 else l[tok] * sp.rep_penalty
    if sp.temperature <= 0.001:
        best = 0
        for i in range(1, V):
            if l[i] > l[best]:
                best = i
        s = 0.0
        for x in l:
            s += math.exp(x - l[best])
        return best, 1.0 / s
    inv_t = 1.0 / sp.temperature
    mx = NEG_MAX
    for i in range(V):
        l[i] *= inv_t
        mx = max(mx, l[i]) if l[i] > mx else mx
    if sp.top_k <= 0 and sp.top_p >= 0.9999:
        p = [math.exp(x - mx) for x in l]
        s = 0.0
        for x in p:
            s += x
        r, cum = u * s, 0.0
        for i, x in enumerate(p):
            cum += x
            if r <= cum:
                return i, x / s
        return 0, p[0] / s
    p = [math.exp(x - mx) for x in l]
    s = 0.0
    for x in p:
        s += x
    inv = 1.0 / s
    cand = sorted(((x * inv, i) for i, x in enumerate(p)), key=lambda c: (-c[0], c[1]))
    active = V
    if 0 < sp.top_k < active:
        active = sp.top_k
    if 0.0 < sp.top_p < 1.0:
        cum, cut = 0.0, 0
        for i in range(active):
            cum += cand[i][0]
            cut = i + 1
            if cum >= sp.top_p:
                break
        active = cut
    if active == 1:
        return cand[0][1], 1.0
    sp_sum = 0.0
    for i in range(active):
        sp_sum += cand[i][0]
    r, cum = u * sp_sum, 0.0
    for i in range(active):
        cum += cand[i][0]
        if r <= cum:
            return cand[i][1], cand[i][0] / sp_sum
    return cand[active - 1][1], cand[active - 1][0] / sp_sum


def _penalised(logits, sp, prefix, gen, allowed):
    l = np.array(logits, np.float64)
    V = l.size
    gen = list(gen)
    if sp.ban_trigrams and len(gen) >= 2:
        for i in range(len(gen) - 2):
            if gen[i] == gen[-2] and gen[i + 1] == gen[-1] and 0 <= gen[i + 2] < V:
                l[gen[i + 2]] = NEG_MAX
    if allowed is not None:
        l[np.asarray(allowed) < 0] = -1e300
    recent = list(prefix) + gen
    if sp.rep_window > 0:
        recent = recent[-sp.rep_window:]
    if sp.rep_penalty > 1.0:
        for i, tok in enumerate(recent):
            if 0 <= tok < V and tok not in recent[:i]:
                l[tok] = l[tok] / sp.rep_penalty if l[tok] > 0 else l[tok] * sp.rep_penalty
    return l


def policy_margin(logits, sp, prefix=(), gen=(), allowed=None, u=0.5):
    """How far this case lies from a decision edge: for argmax the gap between the two largest
    penalised logits relative to the largest magnitude; for a draw the smallest distance of the
    draw (and of the top-p threshold) from a running-sum edge, relative to the total."""
    l = _penalised(logits, sp, prefix, gen, allowed)
    if sp.temperature <= 0.001:
        top = np.sort(l)[-2:]
        return float((top[1] - top[0]) / max(1e-30, np.max(np.abs(l[l > -1e299]))))
    z = l / sp.temperature
    p = np.exp(z - z.max())
    if sp.top_k <= 0 and sp.top_p >= 0.9999:
        cdf = np.cumsum(p)
        return float(np.min(np.abs(cdf - u * cdf[-1])) / cdf[-1])
    prob = p / p.sum()
    order = np.lexsort((np.arange(prob.size), -prob))
    q = prob[order]
    active = sp.top_k if 0 < sp.top_k < q.size else q.size
    cdf = np.cumsum(q[:active])
    m = 1.0
    if 0.0 < sp.top_p < 1.0:
        m = float(np.min(np.abs(cdf - sp.top_p)))
        hit = np.nonzero(cdf >= sp.top_p)[0]
        active = int(hit[0]) + 1 if hit.size else active
        cdf = cdf[:active]
    return min(m, float(np.min(np.abs(cdf - u * cdf[-1])) / cdf[-1]))
