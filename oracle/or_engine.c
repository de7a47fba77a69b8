/*
 * Oracle streaming engine — TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Restates the position-major INT8 engine of internal/quant: appendPosition
 * (stream.go:141-193), updateLatch (:197-205), applyRule (:209-230), headLogits (:233-248),
 * prefill (:252-261), attendPosition (attention.go:71-104), Call (model.go:122-132) and the
 * cached session (session.go:11-68), with the reference's float32 operation order.
 */
#include "or_internal.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static float* zalloc(size_t n) { return calloc(n ? n : 1, sizeof(float)); }

or_state* or_state_new(const or_model* m) {
    or_state* st = calloc(1, sizeof(or_state));
    int D = m->D;
    st->norm = zalloc((size_t)m->total_steps * m->ring * D);
    st->latch = zalloc((size_t)m->total_steps * D);
    st->attn_k = zalloc((size_t)m->nblocks * m->attn_cache * D);
    st->attn_v = zalloc((size_t)m->nblocks * m->attn_cache * D);
    st->attn_scores = zalloc((size_t)m->attn_cache);
    st->attn_scratch = zalloc((size_t)m->attn_cache);
    st->bufs = zalloc((size_t)3 * D);
    st->cur = st->bufs;
    st->next = st->bufs + D;
    st->block_in = st->bufs + 2 * D;
    return st;
}

void or_state_free(or_state* st) {
    if (!st) return;
    free(st->norm);
    free(st->latch);
    free(st->attn_k);
    free(st->attn_v);
    free(st->attn_scores);
    free(st->attn_scratch);
    free(st->bufs);
    free(st);
}

or_scratch* or_scratch_new(const or_model* m) {
    or_scratch* s = calloc(1, sizeof(or_scratch));
    int D = m->D, H = m->H;
    s->mlp_input = zalloc((size_t)3 * D);
    s->mlp_hidden = zalloc((size_t)H);
    s->mlp_output = zalloc((size_t)2 * D);
    s->xhat = zalloc((size_t)D);
    s->norm_scratch = zalloc((size_t)D);
    s->logits = zalloc((size_t)m->vocab);
    s->mlp_gate = zalloc((size_t)H);
    s->latch_logit = zalloc((size_t)D);
    s->a_norm = zalloc((size_t)D);
    s->a_xhat = zalloc((size_t)D);
    s->a_qkv = zalloc((size_t)3 * D);
    s->a_att = zalloc((size_t)D);
    s->a_proj = zalloc((size_t)D);
    return s;
}

void or_scratch_free(or_scratch* s) {
    if (!s) return;
    free(s->mlp_input);
    free(s->mlp_hidden);
    free(s->mlp_output);
    free(s->xhat);
    free(s->norm_scratch);
    free(s->logits);
    free(s->mlp_gate);
    free(s->latch_logit);
    free(s->a_norm);
    free(s->a_xhat);
    free(s->a_qkv);
    free(s->a_att);
    free(s->a_proj);
    free(s);
}

static void reset_state(const or_model* m, or_state* st) {
    st->n = 0;
    memset(st->latch, 0, sizeof(float) * (size_t)m->total_steps * m->D);
}

/* updateLatch (stream.go:197-205) */
static const float* update_latch(const or_model* m, or_scratch* sc, float* gl, const or_block* bl, const float* norm_cell) {
    int D = m->D;
    or_matvec_i8(sc->latch_logit, D, bl->wsel.data, D, bl->wsel.scale, norm_cell, D, m->latch_base);
    for (int d = 0; d < D; d++) {
        float lam = or_sigmoid_clamped(sc->latch_logit[d]);
        float a = lam * gl[d];
        float b = (1.0f - lam) * norm_cell[d];
        gl[d] = a + b;
    }
    return gl;
}

/* applyRule (stream.go:209-230) with AssembleNeighborhood (ca/neighborhood.go:16-25) */
static void apply_rule(const or_model* m, or_scratch* sc, const or_block* bl, const float* norm_cell, const float* left,
                       const float* latch, const float* self, float* next) {
    int D = m->D, H = m->H, in_dim = 3 * D;
    float* x = sc->mlp_input;
    memcpy(x, norm_cell, sizeof(float) * D);
    if (left) memcpy(x + D, left, sizeof(float) * D);
    else memset(x + D, 0, sizeof(float) * D);
    memcpy(x + 2 * D, latch, sizeof(float) * D);
    or_matvec_i8(sc->mlp_hidden, H, bl->w1.data, in_dim, bl->w1.scale, x, in_dim, bl->b1);
    or_matvec_i8(sc->mlp_gate, H, bl->w1.data + (size_t)H * in_dim, in_dim, bl->w1.scale, x, in_dim, bl->b1 + H);
    for (int h = 0; h < H; h++) sc->mlp_hidden[h] *= or_sigmoid_clamped(sc->mlp_gate[h]);
    or_matvec_i8(sc->mlp_output, 2 * D, bl->w2.data, H, bl->w2.scale, sc->mlp_hidden, H, bl->b2);
    for (int s = 0; s < D; s++) {
        float gate = or_sigmoid_clamped(sc->mlp_output[D + s]);
        float a = (1.0f - gate) * self[s];
        float b = gate * sc->mlp_output[s];
        next[s] = a + b;
    }
}

/* attendPosition (attention.go:71-104) */
static void attend_position(const or_model* m, or_state* st, or_scratch* sc, int b, const or_block* bl, int pos) {
    int D = m->D, heads = m->attn_heads, dh = D / heads;
    or_rmsnorm_f32(st->cur, bl->attn_norm, sc->a_norm, sc->a_xhat, D, 1e-5f);
    or_matvec_i8(sc->a_qkv, 3 * D, bl->qkv.data, D, bl->qkv.scale, sc->a_norm, D, NULL);
    int ring = m->attn_cache;
    float* keys = st->attn_k + (size_t)b * ring * D;
    float* values = st->attn_v + (size_t)b * ring * D;
    int slot = pos % ring;
    memcpy(keys + (size_t)slot * D, sc->a_qkv + D, sizeof(float) * D);
    memcpy(values + (size_t)slot * D, sc->a_qkv + 2 * D, sizeof(float) * D);
    int ws = 0; /* nn.WindowStart (nn/attention.go:55-60) */
    if (m->attn_window > 0 && pos - m->attn_window + 1 > 0) ws = pos - m->attn_window + 1;
    int lo = ws > pos - ring + 1 ? ws : pos - ring + 1;
    int span = pos - lo + 1;
    float* scores = st->attn_scores;
    float scale = (float)(1.0 / sqrt((double)dh));
    memset(sc->a_att, 0, sizeof(float) * D);
    for (int h = 0; h < heads; h++) {
        const float* q = sc->a_qkv + h * dh;
        for (int j = lo; j <= pos; j++) {
            size_t k = (size_t)(j % ring) * D;
            scores[j - lo] = or_dot_f32(q, keys + k + h * dh, dh) * scale;
        }
        or_softmax_f32(scores, st->attn_scratch, span);
        float* out = sc->a_att + h * dh;
        for (int j = lo; j <= pos; j++) {
            size_t v = (size_t)(j % ring) * D;
            or_add_scaled_f32(out, values + v + h * dh, scores[j - lo], dh);
        }
    }
    or_matvec_i8(sc->a_proj, D, bl->out.data, D, bl->out.scale, sc->a_att, D, NULL);
    for (int d = 0; d < D; d++) st->cur[d] += sc->a_proj[d];
}

/* appendPosition (stream.go:141-193) */
void or_append_position(const or_model* m, or_state* st, or_scratch* sc, int token, int need_output) {
    int D = m->D;
    int pos = st->n;
    if (token < 0 || token >= m->vocab) token = 0;
    size_t off = (size_t)token * D;
    for (int d = 0; d < D; d++) {
        float v = (float)m->embed.data[off + d] * m->embed.scale;
        st->cur[d] = v;
        st->block_in[d] = v;
    }
    for (int b = 0; b < m->nblocks; b++) {
        const or_block* bl = &m->blocks[b];
        if (b > 0)
            for (int d = 0; d < D; d++) {
                st->block_in[d] += st->cur[d];
                st->cur[d] = st->block_in[d];
            }
        for (int step = 0; step < bl->steps; step++) {
            int bs = m->step_offset[b] + step;
            float* norm_cell = st->norm + ((size_t)bs * m->ring + (size_t)(pos % m->ring)) * D;
            if (bl->n_gamma == (size_t)D) or_rmsnorm_f32(st->cur, bl->gamma, norm_cell, sc->xhat, D, 1e-5f);
            else memcpy(norm_cell, st->cur, sizeof(float) * D);
            const float* latch = update_latch(m, sc, st->latch + (size_t)bs * D, bl, norm_cell);
            if (!need_output && b == m->nblocks - 1 && step == bl->steps - 1 && !bl->has_attn) break;
            const float* left = NULL;
            int left_idx = pos - or_step_dilation(bl->initial_dilation, bl->dilation_base, step);
            if (left_idx >= 0) left = st->norm + ((size_t)bs * m->ring + (size_t)(left_idx % m->ring)) * D;
            apply_rule(m, sc, bl, norm_cell, left, latch, st->cur, st->next);
            float* t = st->cur;
            st->cur = st->next;
            st->next = t;
        }
        if (bl->has_attn) attend_position(m, st, sc, b, bl, pos);
    }
    st->n++;
}

/* headLogits (stream.go:233-248); out receives the float32 logits. */
void or_head_logits(const or_model* m, or_scratch* sc, const float* cell, float* out) {
    int D = m->D;
    if (m->n_final_norm == (size_t)D) {
        or_rmsnorm_f32(cell, m->final_norm, sc->norm_scratch, sc->xhat, D, 1e-5f);
        cell = sc->norm_scratch;
    }
    const int8_t* w = m->tied ? m->embed.data : m->head_w.data;
    float scale = m->tied ? m->embed.scale : m->head_w.scale;
    or_matvec_i8(out, m->vocab, w, D, scale, cell, D, m->head_b);
}

/* prefill (stream.go:252-261) */
void or_prefill(const or_model* m, or_state* st, or_scratch* sc, const int32_t* tokens, int n, float* out) {
    if (n > m->max_context) {
        tokens += n - m->max_context;
        n = m->max_context;
    }
    reset_state(m, st);
    for (int i = 0; i < n; i++) or_append_position(m, st, sc, tokens[i], i == n - 1);
    or_head_logits(m, sc, st->cur, out);
}

int or_model_call(const or_model* m, const int32_t* window, int n, float* logits) {
    if (n == 0) return -1;
    or_state* st = or_state_new(m);
    or_scratch* sc = or_scratch_new(m);
    or_prefill(m, st, sc, window, n, logits);
    or_state_free(st);
    or_scratch_free(sc);
    return 0;
}

/* quantSession (session.go:11-68) */
struct or_session {
    const or_model* m;
    or_state* st;
    or_scratch* sc;
    int window;
    int32_t* tokens;
    int ntok;
    int fed;
};

or_session* or_session_new(const or_model* m, int context_size) {
    or_session* s = calloc(1, sizeof(or_session));
    s->m = m;
    s->st = or_state_new(m);
    s->sc = or_scratch_new(m);
    s->window = m->max_context;
    if (context_size > 0 && context_size < s->window) s->window = context_size;
    s->tokens = calloc((size_t)s->window + 1, sizeof(int32_t));
    return s;
}

void or_session_free(or_session* s) {
    if (!s) return;
    or_state_free(s->st);
    or_scratch_free(s->sc);
    free(s->tokens);
    free(s);
}

int or_session_prefill(or_session* s, const int32_t* tokens, int n, float* logits) {
    if (n > s->window) {
        tokens += n - s->window;
        n = s->window;
    }
    memmove(s->tokens, tokens, sizeof(int32_t) * (size_t)n);
    s->ntok = n;
    if (n == 0) return 0;
    s->fed = n;
    or_prefill(s->m, s->st, s->sc, s->tokens, n, logits);
    return 1;
}

int or_session_append(or_session* s, int32_t token, float* logits) {
    s->tokens[s->ntok++] = token;
    if (s->ntok > s->window) {
        memmove(s->tokens, s->tokens + 1, sizeof(int32_t) * (size_t)(s->ntok - 1));
        s->ntok--;
    }
    if (s->fed == 0 || s->st->n != s->fed) {
        s->fed = s->ntok;
        or_prefill(s->m, s->st, s->sc, s->tokens, s->ntok, logits);
        return 1;
    }
    or_append_position(s->m, s->st, s->sc, token, 1);
    s->fed++;
    or_head_logits(s->m, s->sc, s->st->cur, logits);
    return 1;
}

/* quantSeqState.bytes (stream.go:88-102): float32 working vectors and caches counted as the
 * reference counts them. */
long or_session_state_bytes(const or_session* s) {
    const or_model* m = s->m;
    long n = 3L * m->D + (long)m->total_steps * m->ring * m->D + (long)m->total_steps * m->D;
    long n32 = 0;
    int any_attn = 0;
    for (int b = 0; b < m->nblocks; b++)
        if (m->blocks[b].has_attn) {
            any_attn = 1;
            n32 += 2L * m->attn_cache * m->D;
        }
    if (any_attn) n32 += 2L * m->attn_cache;
    return n * 8 + n32 * 4;
}

int or_session_position(const or_session* s) { return s->st->n; }
