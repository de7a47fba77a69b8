/*
 * Oracle token selection and batch runners — TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * argmaxProb (internal/generate/greedy.go:90-102), logProb (internal/eval/suite.go:201-209),
 * the truncated branch of SampleRawLogitsAdvanced (internal/generate/sample.go:33-172) and
 * sampleFromCDF (:174-191), with the uniform draw taken from Philox4x32-10 (Salmon et al.,
 * SC'11) keyed by the session instead of Go's global math/rand. The runners drive one cached
 * session per sequence (internal/quant/session.go) like greedyLoop (greedy.go:63-87).
 */
#include "or_internal.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int or_argmax_prob(const float* logits, int n, double* prob) {
    int best = 0;
    for (int i = 0; i < n; i++)
        if ((double)logits[i] > (double)logits[best]) best = i;
    double sum = 0.0;
    for (int i = 0; i < n; i++) sum += exp((double)logits[i] - (double)logits[best]);
    if (prob) *prob = 1.0 / sum;
    return best;
}

double or_log_prob(const float* logits, int n, int id) {
    double mx = (double)logits[0];
    for (int i = 1; i < n; i++)
        if ((double)logits[i] > mx) mx = (double)logits[i];
    double sum = 0.0;
    for (int i = 0; i < n; i++) sum += exp((double)logits[i] - mx);
    return (double)logits[id] - mx - log(sum);
}

void or_philox4x32(const uint32_t c[4], const uint32_t k[2], uint32_t out[4]) {
    uint32_t c0 = c[0], c1 = c[1], c2 = c[2], c3 = c[3], k0 = k[0], k1 = k[1];
    for (int r = 0; r < 10; r++) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0, hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0;
        c1 = lo1;
        c2 = n2;
        c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0;
    out[1] = c1;
    out[2] = c2;
    out[3] = c3;
}

double or_sample_uniform(uint32_t session, uint32_t step) {
    uint32_t c[4] = {step, 0, 0, 0}, k[2] = {session, 0x53414D50u}, o[4];
    or_philox4x32(c, k, o);
    uint64_t a = o[0] >> 5, b = o[1] >> 6;
    return (double)(a * 67108864ull + b) * (1.0 / 9007199254740992.0);
}

typedef struct {
    int idx;
    double prob;
} cand;

static int cand_cmp(const void* a, const void* b) {
    const cand* x = a;
    const cand* y = b;
    if (x->prob > y->prob) return -1;
    if (x->prob < y->prob) return 1;
    return x->idx - y->idx; /* deterministic order among equal probabilities */
}

int or_sample_topk(const float* logits, int n, double temperature, int topk, double u) {
    if (n == 0) return 0;
    if (temperature <= 0.001) {
        int best = 0;
        for (int i = 1; i < n; i++)
            if ((double)logits[i] > (double)logits[best]) best = i;
        return best;
    }
    double inv_t = 1.0 / temperature;
    cand* c = malloc(sizeof(cand) * (size_t)n);
    double mx = -1.7976931348623157e308;
    for (int i = 0; i < n; i++) {
        double s = (double)logits[i] * inv_t;
        c[i].idx = i;
        c[i].prob = s;
        if (s > mx) mx = s;
    }
    double sum = 0.0;
    for (int i = 0; i < n; i++) {
        c[i].prob = exp(c[i].prob - mx);
        sum += c[i].prob;
    }
    double inv = 1.0 / sum;
    for (int i = 0; i < n; i++) c[i].prob *= inv;
    qsort(c, (size_t)n, sizeof(cand), cand_cmp);
    int active = n;
    if (topk > 0 && topk < active) active = topk;
    int chosen;
    if (active == 1) chosen = c[0].idx;
    else {
        double sp = 0.0;
        for (int i = 0; i < active; i++) sp += c[i].prob;
        double r = u * sp, cum = 0.0;
        chosen = c[active - 1].idx;
        for (int i = 0; i < active; i++) {
            cum += c[i].prob;
            if (r <= cum) {
                chosen = c[i].idx;
                break;
            }
        }
    }
    free(c);
    return chosen;
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
}

int or_generate_greedy(const or_model* m, int n_sess, const int32_t* prompts, int stride, const int32_t* lens,
                       int context_size, int n_new, int32_t* out_tokens, float* out_probs, float* out_logits,
                       int nthreads) {
    set_threads(nthreads);
#pragma omp parallel
    {
        or_session* s = or_session_new(m, context_size);
        float* logits = malloc(sizeof(float) * (size_t)m->vocab);
#pragma omp for schedule(dynamic, 1)
        for (int i = 0; i < n_sess; i++) {
            int have = or_session_prefill(s, prompts + (size_t)i * stride, lens[i], logits);
            for (int t = 0; t < n_new; t++) {
                if (!have) {
                    out_tokens[(size_t)i * n_new + t] = -1;
                    if (out_probs) out_probs[(size_t)i * n_new + t] = 0;
                    continue;
                }
                if (out_logits) memcpy(out_logits + ((size_t)i * n_new + t) * m->vocab, logits, sizeof(float) * m->vocab);
                double p;
                int best = or_argmax_prob(logits, m->vocab, &p);
                out_tokens[(size_t)i * n_new + t] = best;
                if (out_probs) out_probs[(size_t)i * n_new + t] = (float)p;
                if (t + 1 < n_new) or_session_append(s, best, logits);
            }
        }
        free(logits);
        or_session_free(s);
    }
    return 0;
}

int or_generate_sample(const or_model* m, int n_sess, const int32_t* prompts, int stride, const int32_t* lens,
                       int context_size, int n_new, double temperature, int topk, uint32_t session0,
                       int32_t* out_tokens, float* out_logits, int nthreads) {
    set_threads(nthreads);
#pragma omp parallel
    {
        or_session* s = or_session_new(m, context_size);
        float* logits = malloc(sizeof(float) * (size_t)m->vocab);
#pragma omp for schedule(dynamic, 1)
        for (int i = 0; i < n_sess; i++) {
            int have = or_session_prefill(s, prompts + (size_t)i * stride, lens[i], logits);
            for (int t = 0; t < n_new; t++) {
                if (!have) {
                    out_tokens[(size_t)i * n_new + t] = -1;
                    continue;
                }
                if (out_logits) memcpy(out_logits + ((size_t)i * n_new + t) * m->vocab, logits, sizeof(float) * m->vocab);
                double u = or_sample_uniform(session0 + (uint32_t)i, (uint32_t)t);
                int tok = or_sample_topk(logits, m->vocab, temperature, topk, u);
                out_tokens[(size_t)i * n_new + t] = tok;
                if (t + 1 < n_new) or_session_append(s, tok, logits);
            }
        }
        free(logits);
        or_session_free(s);
    }
    return 0;
}

int or_score(const or_model* m, int n_seq, int len, const int32_t* tokens, double* out_logprobs, int nthreads) {
    set_threads(nthreads);
#pragma omp parallel
    {
        or_state* st = or_state_new(m);
        or_scratch* sc = or_scratch_new(m);
        float* logits = malloc(sizeof(float) * (size_t)m->vocab);
#pragma omp for schedule(dynamic, 1)
        for (int i = 0; i < n_seq; i++) {
            const int32_t* seq = tokens + (size_t)i * len;
            st->n = 0;
            memset(st->latch, 0, sizeof(float) * (size_t)m->total_steps * m->D);
            /* The logits after every prefix equal Call(prefix) (session_test.go:18-52); one
             * streaming pass produces them all. */
            for (int t = 0; t + 1 < len; t++) {
                or_append_position(m, st, sc, seq[t], 1);
                or_head_logits(m, sc, st->cur, logits);
                out_logprobs[(size_t)i * (len - 1) + t] = or_log_prob(logits, m->vocab, seq[t + 1]);
            }
        }
        free(logits);
        or_scratch_free(sc);
        or_state_free(st);
    }
    return 0;
}

/* ---- the full decode-loop policy ---------------------------------------------------------- */

static int is_stop(int tok, const int32_t* stops, int n_stops) {
    for (int k = 0; k < n_stops; k++)
        if (stops[k] >= 0 && tok == stops[k]) return 1;
    return 0;
}

/* Token k of the concatenation prefix ++ gen. */
static int32_t hist_at(const int32_t* prefix, int n_prefix, const int32_t* gen, int k) {
    return k < n_prefix ? prefix[k] : gen[k - n_prefix];
}

/* Sum of v[0..n) in index order, and the index of the first running sum >= r (or -1). */
static int first_cum_at_least(const double* v, int n, double r) {
    double cum = 0.0;
    for (int i = 0; i < n; i++) {
        cum += v[i];
        if (r <= cum) return i;
    }
    return -1;
}

int or_sample_policy(double* logits, int n, const int32_t* prefix, int n_prefix, const int32_t* gen, int n_gen,
                     const or_sampling* sp, const int32_t* allowed, double u, double* prob) {
    const double neg_max = -1.7976931348623157e308;
    if (n <= 0) return 0;
    /* 3-gram repetition block of sampleContinuation (sample.go:213-227): a token that followed the
     * trailing pair earlier in the generated tokens gets -MaxFloat64 */
    if (sp->ban_trigrams && n_gen >= 2) {
        const int32_t w1 = gen[n_gen - 2], w2 = gen[n_gen - 1];
        for (int i = 0; i <= n_gen - 3; i++)
            if (gen[i] == w1 && gen[i + 1] == w2 && gen[i + 2] >= 0 && gen[i + 2] < n) logits[gen[i + 2]] = neg_max;
    }
    /* Constraint.Mask (sample.go:229-231): tokens without a transition get -1e300 like the
     * grammar's negInf (constrain/grammar.go:259) */
    if (allowed)
        for (int i = 0; i < n; i++)
            if (allowed[i] < 0) logits[i] = -1e300;
    /* repetition penalty over the window's distinct tokens (sample.go:48-69); the window is the
     * trailing rep_window tokens of prefix ++ generated (sample.go:207-210) */
    const int total = n_prefix + n_gen;
    const int w = sp->rep_window > 0 && sp->rep_window < total ? sp->rep_window : total;
    const int w0 = total - w;
    if (sp->rep_penalty > 1.0 && w > 0) {
        for (int i = 0; i < w; i++) {
            const int32_t tok = hist_at(prefix, n_prefix, gen, w0 + i);
            if (tok < 0 || tok >= n) continue;
            int seen = 0;
            for (int j = 0; j < i && !seen; j++) seen = hist_at(prefix, n_prefix, gen, w0 + j) == tok;
            if (seen) continue;
            if (logits[tok] > 0) logits[tok] /= sp->rep_penalty;
            else logits[tok] *= sp->rep_penalty;
        }
    }
    /* greedy argmax (sample.go:71-82); prob = 1 / sum exp(l - max) as argmaxProb reports it */
    if (sp->temperature <= 0.001) {
        int best = 0;
        for (int i = 1; i < n; i++)
            if (logits[i] > logits[best]) best = i;
        if (prob) {
            double s = 0.0;
            for (int i = 0; i < n; i++) s += exp(logits[i] - logits[best]);
            *prob = 1.0 / s;
        }
        return best;
    }
    const double inv_t = 1.0 / sp->temperature;
    double mx = neg_max;
    for (int i = 0; i < n; i++) {
        logits[i] *= inv_t;
        if (logits[i] > mx) mx = logits[i];
    }
    if (sp->top_k <= 0 && sp->top_p >= 0.9999) {
        /* pure temperature sampling in index order (sample.go:96-117) */
        double s = 0.0;
        for (int i = 0; i < n; i++) {
            logits[i] = exp(logits[i] - mx);
            s += logits[i];
        }
        int chosen = first_cum_at_least(logits, n, u * s);
        if (chosen < 0) chosen = 0;
        if (prob) *prob = logits[chosen] / s;
        return chosen;
    }
    /* truncated sampling (sample.go:119-172): probabilities sorted descending (ties by index),
     * top-k, then the shortest prefix whose mass reaches top-p, then sampleFromCDF (:174-191) */
    cand* c = malloc(sizeof(cand) * (size_t)n);
    double s = 0.0;
    for (int i = 0; i < n; i++) {
        c[i].idx = i;
        c[i].prob = exp(logits[i] - mx);
        s += c[i].prob;
    }
    const double inv = 1.0 / s;
    for (int i = 0; i < n; i++) c[i].prob *= inv;
    qsort(c, (size_t)n, sizeof(cand), cand_cmp);
    int active = n;
    if (sp->top_k > 0 && sp->top_k < active) active = sp->top_k;
    if (sp->top_p > 0.0 && sp->top_p < 1.0) {
        double cum = 0.0;
        int cut = 0;
        for (int i = 0; i < active; i++) {
            cum += c[i].prob;
            cut = i + 1;
            if (cum >= sp->top_p) break;
        }
        active = cut;
    }
    int chosen;
    double p;
    if (active == 1) {
        chosen = c[0].idx;
        p = 1.0;
    } else {
        double sp_sum = 0.0;
        for (int i = 0; i < active; i++) sp_sum += c[i].prob;
        const double r = u * sp_sum;
        double cum = 0.0;
        int k = active - 1;
        for (int i = 0; i < active; i++) {
            cum += c[i].prob;
            if (r <= cum) {
                k = i;
                break;
            }
        }
        chosen = c[k].idx;
        p = c[k].prob / sp_sum;
    }
    if (prob) *prob = p;
    free(c);
    return chosen;
}

int or_generate_policy(const or_model* m, int n_sess, const int32_t* prompts, int stride, const int32_t* lens,
                       int context_size, int n_new, const or_sampling* sp, int penalize_prompt, const int32_t* dfa,
                       const int32_t* dfa_start, uint32_t session0, const int32_t* stops, int n_stops,
                       int32_t* out_tokens, float* out_probs, int32_t* out_lens, float* out_logits, int nthreads) {
    set_threads(nthreads);
    const int V = m->vocab;
#pragma omp parallel
    {
        or_session* s = or_session_new(m, context_size);
        float* logits = malloc(sizeof(float) * (size_t)V);
        double* work = malloc(sizeof(double) * (size_t)V);
        int32_t* gen = malloc(sizeof(int32_t) * (size_t)(n_new > 0 ? n_new : 1));
#pragma omp for schedule(dynamic, 1)
        for (int i = 0; i < n_sess; i++) {
            const int32_t* prompt = prompts + (size_t)i * stride;
            int have = or_session_prefill(s, prompt, lens[i], logits);
            int n_gen = 0;
            int state = dfa ? dfa_start[i] : -1;
            /* sampleContinuation (sample.go:196-247): the penalty prefix is the prompt (chat.go:72)
             * or nothing (chat.go:122) */
            for (int t = 0; t < n_new && have; t++) {
                if (out_logits) memcpy(out_logits + ((size_t)i * n_new + t) * V, logits, sizeof(float) * V);
                for (int v = 0; v < V; v++) work[v] = (double)logits[v];
                double p = 0.0;
                const double u = or_sample_uniform(session0 + (uint32_t)i, (uint32_t)t);
                const int tok = or_sample_policy(work, V, prompt, penalize_prompt ? lens[i] : 0, gen, n_gen, sp,
                                                 state >= 0 ? dfa + (size_t)state * V : NULL, u, &p);
                if (is_stop(tok, stops, n_stops)) break;
                if (state >= 0) state = dfa[(size_t)state * V + tok];  /* Constraint.Advance */
                gen[n_gen++] = tok;
                out_tokens[(size_t)i * n_new + t] = tok;
                if (out_probs) out_probs[(size_t)i * n_new + t] = (float)p;
                if (n_gen < n_new) or_session_append(s, tok, logits);
            }
            for (int t = n_gen; t < n_new; t++) {
                out_tokens[(size_t)i * n_new + t] = -1;
                if (out_probs) out_probs[(size_t)i * n_new + t] = 0.f;
            }
            if (out_lens) out_lens[i] = n_gen;
        }
        free(gen);
        free(work);
        free(logits);
        or_session_free(s);
    }
    return 0;
}
