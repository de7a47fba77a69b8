/*
 * Oracle model file reader — TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Restates quant.Decode (internal/quant/checkpoint.go:162-212): a binary mignon.model/1 file
 * (internal/binfmt/binfmt.go:1-14, Decode :88-107, Fill :111-144) whose header is the checkpoint
 * JSON without arrays, arrays in the order of CheckpointJSON.arrays (checkpoint.go:77-89); or a
 * legacy JSON checkpoint with the arrays inline. The shape check is checkBlockShapes (:216-225).
 */
#include "or_internal.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------------------------ */
/* Minimal JSON tree                                                                           */
/* ------------------------------------------------------------------------------------------ */
typedef enum { JNULL, JBOOL, JNUM, JSTR, JARR, JOBJ } jtype;
typedef struct jval {
    jtype t;
    double num;
    float f32; /* the number parsed directly to float32, as strconv.ParseFloat(s, 32) */
    int b;
    char* str;
    struct jval** items; /* array items or object values */
    char** keys;         /* object keys */
    int n;
} jval;

typedef struct {
    const char* s;
    size_t n, i;
    int err;
} jparser;

static void jfree(jval* v) {
    if (!v) return;
    for (int i = 0; i < v->n; i++) {
        jfree(v->items[i]);
        if (v->keys) free(v->keys[i]);
    }
    free(v->items);
    free(v->keys);
    free(v->str);
    free(v);
}

static void jws(jparser* p) {
    while (p->i < p->n && (p->s[p->i] == ' ' || p->s[p->i] == '\n' || p->s[p->i] == '\t' || p->s[p->i] == '\r'))
        p->i++;
}

static jval* jparse_value(jparser* p, int depth);

static char* jparse_string(jparser* p) {
    if (p->i >= p->n || p->s[p->i] != '"') {
        p->err = 1;
        return NULL;
    }
    p->i++;
    size_t cap = 16, len = 0;
    char* out = malloc(cap);
    while (p->i < p->n && p->s[p->i] != '"') {
        char c = p->s[p->i++];
        if (c == '\\') {
            if (p->i >= p->n) break;
            char e = p->s[p->i++];
            switch (e) {
            case 'n': c = '\n'; break;
            case 't': c = '\t'; break;
            case 'r': c = '\r'; break;
            case 'b': c = '\b'; break;
            case 'f': c = '\f'; break;
            case 'u': /* keep escaped code points as '?': names are ASCII */
                p->i += 4;
                c = '?';
                break;
            default: c = e;
            }
        }
        if (len + 1 >= cap) out = realloc(out, cap *= 2);
        out[len++] = c;
    }
    if (p->i >= p->n) {
        p->err = 1;
        free(out);
        return NULL;
    }
    p->i++;
    out[len] = 0;
    return out;
}

static jval* jnew(jtype t) {
    jval* v = calloc(1, sizeof(jval));
    v->t = t;
    return v;
}

static void jpush(jval* v, char* key, jval* item, int* cap) {
    if (v->n == *cap) {
        *cap = *cap ? *cap * 2 : 8;
        v->items = realloc(v->items, sizeof(jval*) * (size_t)*cap);
        if (v->t == JOBJ) v->keys = realloc(v->keys, sizeof(char*) * (size_t)*cap);
    }
    v->items[v->n] = item;
    if (v->t == JOBJ) v->keys[v->n] = key;
    v->n++;
}

static jval* jparse_value(jparser* p, int depth) {
    if (depth > 64) {
        p->err = 1;
        return NULL;
    }
    jws(p);
    if (p->i >= p->n) {
        p->err = 1;
        return NULL;
    }
    char c = p->s[p->i];
    if (c == '{') {
        jval* v = jnew(JOBJ);
        int cap = 0;
        p->i++;
        jws(p);
        if (p->i < p->n && p->s[p->i] == '}') {
            p->i++;
            return v;
        }
        for (;;) {
            jws(p);
            char* k = jparse_string(p);
            if (p->err) break;
            jws(p);
            if (p->i >= p->n || p->s[p->i] != ':') {
                free(k);
                p->err = 1;
                break;
            }
            p->i++;
            jval* item = jparse_value(p, depth + 1);
            if (p->err) {
                free(k);
                jfree(item);
                break;
            }
            jpush(v, k, item, &cap);
            jws(p);
            if (p->i < p->n && p->s[p->i] == ',') {
                p->i++;
                continue;
            }
            if (p->i < p->n && p->s[p->i] == '}') {
                p->i++;
                return v;
            }
            p->err = 1;
            break;
        }
        jfree(v);
        return NULL;
    }
    if (c == '[') {
        jval* v = jnew(JARR);
        int cap = 0;
        p->i++;
        jws(p);
        if (p->i < p->n && p->s[p->i] == ']') {
            p->i++;
            return v;
        }
        for (;;) {
            jval* item = jparse_value(p, depth + 1);
            if (p->err) {
                jfree(item);
                break;
            }
            jpush(v, NULL, item, &cap);
            jws(p);
            if (p->i < p->n && p->s[p->i] == ',') {
                p->i++;
                continue;
            }
            if (p->i < p->n && p->s[p->i] == ']') {
                p->i++;
                return v;
            }
            p->err = 1;
            break;
        }
        jfree(v);
        return NULL;
    }
    if (c == '"') {
        jval* v = jnew(JSTR);
        v->str = jparse_string(p);
        if (p->err) {
            jfree(v);
            return NULL;
        }
        return v;
    }
    if (p->n - p->i >= 4 && !strncmp(p->s + p->i, "null", 4)) {
        p->i += 4;
        return jnew(JNULL);
    }
    if (p->n - p->i >= 4 && !strncmp(p->s + p->i, "true", 4)) {
        p->i += 4;
        jval* v = jnew(JBOOL);
        v->b = 1;
        return v;
    }
    if (p->n - p->i >= 5 && !strncmp(p->s + p->i, "false", 5)) {
        p->i += 5;
        return jnew(JBOOL);
    }
    /* number */
    char buf[64];
    size_t k = 0;
    while (p->i < p->n && k < sizeof(buf) - 1 &&
           (strchr("+-0123456789.eE", p->s[p->i]) != NULL))
        buf[k++] = p->s[p->i++];
    buf[k] = 0;
    if (k == 0) {
        p->err = 1;
        return NULL;
    }
    char* end;
    double d = strtod(buf, &end);
    if (*end) {
        p->err = 1;
        return NULL;
    }
    jval* v = jnew(JNUM);
    v->num = d;
    v->f32 = strtof(buf, NULL);
    return v;
}

static jval* jget(const jval* o, const char* key) {
    if (!o || o->t != JOBJ) return NULL;
    for (int i = 0; i < o->n; i++)
        if (!strcmp(o->keys[i], key)) return o->items[i];
    return NULL;
}

static double jnum(const jval* o, const char* key, double dflt) {
    const jval* v = jget(o, key);
    return (v && v->t == JNUM) ? v->num : dflt;
}

static int jbool(const jval* o, const char* key) {
    const jval* v = jget(o, key);
    return v && v->t == JBOOL && v->b;
}

/* ------------------------------------------------------------------------------------------ */
/* Model                                                                                       */
/* ------------------------------------------------------------------------------------------ */
typedef struct {
    int is_i8;
    int8_t** i8;
    float** f32;
    size_t* n;
} arr_ref;

static void ferr(char* err, size_t len, const char* msg) {
    if (err && len) snprintf(err, len, "%s", msg);
}

/* Reads a JSON array of numbers into a freshly allocated int8 or float32 array. */
static int json_array(const jval* v, arr_ref a) {
    size_t n = (v && v->t == JARR) ? (size_t)v->n : 0;
    if (v && v->t != JARR && v->t != JNULL) return -1;
    *a.n = n;
    if (a.is_i8) {
        *a.i8 = malloc(n ? n : 1);
        for (size_t i = 0; i < n; i++) {
            if (v->items[i]->t != JNUM) return -1;
            (*a.i8)[i] = (int8_t)v->items[i]->num;
        }
    } else {
        *a.f32 = malloc((n ? n : 1) * sizeof(float));
        for (size_t i = 0; i < n; i++) {
            if (v->items[i]->t != JNUM) return -1;
            (*a.f32)[i] = v->items[i]->f32;
        }
    }
    return 0;
}

void or_model_free(or_model* m) {
    if (!m) return;
    free(m->embed.data);
    for (int b = 0; b < m->nblocks; b++) {
        or_block* bl = &m->blocks[b];
        free(bl->w1.data);
        free(bl->w2.data);
        free(bl->wsel.data);
        free(bl->b1);
        free(bl->b2);
        free(bl->gamma);
        free(bl->attn_norm);
        free(bl->qkv.data);
        free(bl->out.data);
    }
    free(m->blocks);
    free(m->final_norm);
    free(m->head_w.data);
    free(m->head_b);
    free(m->latch_base);
    free(m->step_offset);
    free(m);
}

static void tensor_scale(const jval* t, or_tensor* out) {
    const jval* v = jget(t, "scale");
    out->scale = (v && v->t == JNUM) ? v->f32 : 0.0f;
}

or_model* or_model_decode(const uint8_t* data, size_t n, char* err, size_t errlen) {
    int binary = n >= 4 && !memcmp(data, "MGNN", 4);
    const char* hdr = (const char*)data;
    size_t hlen = n;
    const uint8_t* rest = NULL;
    size_t rest_n = 0;
    if (binary) {
        if (n < 12) {
            ferr(err, errlen, "binary model file is truncated");
            return NULL;
        }
        uint16_t ver = (uint16_t)(data[4] | (data[5] << 8));
        if (ver != 1) {
            ferr(err, errlen, "binary model file version is not supported");
            return NULL;
        }
        if (data[6] != 1 && data[6] != 2) {
            ferr(err, errlen, "unknown model kind");
            return NULL;
        }
        if (data[6] != 2) {
            ferr(err, errlen, "not an INT8 model file");
            return NULL;
        }
        uint32_t h = (uint32_t)data[8] | ((uint32_t)data[9] << 8) | ((uint32_t)data[10] << 16) | ((uint32_t)data[11] << 24);
        if ((size_t)h + 12 > n) {
            ferr(err, errlen, "binary model file is truncated (header)");
            return NULL;
        }
        hdr = (const char*)data + 12;
        hlen = h;
        rest = data + 12 + h;
        rest_n = n - 12 - h;
    }
    jparser p = {hdr, hlen, 0, 0};
    jval* root = jparse_value(&p, 0);
    if (p.err || !root || root->t != JOBJ) {
        jfree(root);
        ferr(err, errlen, "malformed model header JSON");
        return NULL;
    }
    or_model* m = calloc(1, sizeof(or_model));
    m->vocab = (int)jnum(root, "vocab_size", 0);
    m->D = (int)jnum(root, "state_size", 0);
    m->H = (int)jnum(root, "hidden_size", 0);
    m->tied = jbool(root, "tied_embed");
    const jval* meta = jget(root, "metadata");
    int ctx = (int)jnum(meta, "context_size", 0);
    m->attn_heads = (int)jnum(meta, "attn_heads", 0);
    m->attn_window = (int)jnum(meta, "attn_window", 0);
    m->max_context = ctx < 64 ? 128 : ctx; /* NewModel, model.go:93-95 */
    const jval* jembed = jget(root, "embed");
    tensor_scale(jembed, &m->embed);
    const jval* jblocks = jget(root, "blocks");
    m->nblocks = (jblocks && jblocks->t == JARR) ? jblocks->n : 0;
    m->blocks = calloc((size_t)(m->nblocks ? m->nblocks : 1), sizeof(or_block));
    for (int b = 0; b < m->nblocks; b++) {
        const jval* jb = jblocks->items[b];
        or_block* bl = &m->blocks[b];
        bl->steps = (int)jnum(jb, "steps", 0);
        bl->dilation_base = (int)jnum(jb, "dilation_base", 0);
        bl->initial_dilation = (int)jnum(jb, "initial_dilation", 0);
        tensor_scale(jget(jb, "rule_w1"), &bl->w1);
        tensor_scale(jget(jb, "rule_w2"), &bl->w2);
        tensor_scale(jget(jb, "rule_w_select"), &bl->wsel);
        const jval* ja = jget(jb, "attn");
        if (ja && ja->t == JOBJ) {
            bl->has_attn = 1;
            tensor_scale(jget(ja, "qkv"), &bl->qkv);
            tensor_scale(jget(ja, "out"), &bl->out);
        }
    }
    tensor_scale(jget(root, "head_w"), &m->head_w);

    /* Array list in file order (checkpoint.go:77-89). */
    int cap = 8 + m->nblocks * 9;
    arr_ref* arrs = calloc((size_t)cap, sizeof(arr_ref));
    const jval** jsrc = calloc((size_t)cap, sizeof(jval*));
    int na = 0;
#define ADD_I8(T, J) (arrs[na].is_i8 = 1, arrs[na].i8 = &(T).data, arrs[na].n = &(T).n, jsrc[na] = (J), na++)
#define ADD_F32(P, N, J) (arrs[na].is_i8 = 0, arrs[na].f32 = &(P), arrs[na].n = &(N), jsrc[na] = (J), na++)
    ADD_I8(m->embed, jget(jembed, "data"));
    for (int b = 0; b < m->nblocks; b++) {
        const jval* jb = jblocks->items[b];
        or_block* bl = &m->blocks[b];
        ADD_I8(bl->w1, jget(jget(jb, "rule_w1"), "data"));
        ADD_F32(bl->b1, bl->n_b1, jget(jb, "rule_b1"));
        ADD_I8(bl->w2, jget(jget(jb, "rule_w2"), "data"));
        ADD_F32(bl->b2, bl->n_b2, jget(jb, "rule_b2"));
        ADD_F32(bl->gamma, bl->n_gamma, jget(jb, "gamma"));
        ADD_I8(bl->wsel, jget(jget(jb, "rule_w_select"), "data"));
        if (bl->has_attn) {
            const jval* ja = jget(jb, "attn");
            ADD_F32(bl->attn_norm, bl->n_attn_norm, jget(ja, "norm"));
            ADD_I8(bl->qkv, jget(jget(ja, "qkv"), "data"));
            ADD_I8(bl->out, jget(jget(ja, "out"), "data"));
        }
    }
    ADD_F32(m->final_norm, m->n_final_norm, jget(root, "final_norm"));
    ADD_I8(m->head_w, jget(jget(root, "head_w"), "data"));
    ADD_F32(m->head_b, m->n_head_b, jget(root, "head_b"));
#undef ADD_I8
#undef ADD_F32

    int ok = 1;
    if (binary) {
        size_t off = 0;
        for (int i = 0; i < na && ok; i++) {
            if (rest_n - off < 4) {
                ferr(err, errlen, "binary model file is truncated (array)");
                ok = 0;
                break;
            }
            uint32_t cnt = (uint32_t)rest[off] | ((uint32_t)rest[off + 1] << 8) | ((uint32_t)rest[off + 2] << 16) |
                           ((uint32_t)rest[off + 3] << 24);
            off += 4;
            if (arrs[i].is_i8) {
                if (cnt > rest_n - off) {
                    ferr(err, errlen, "binary model file is truncated (array)");
                    ok = 0;
                    break;
                }
                *arrs[i].i8 = malloc(cnt ? cnt : 1);
                memcpy(*arrs[i].i8, rest + off, cnt);
                off += cnt;
            } else {
                if (cnt > (rest_n - off) / 4) {
                    ferr(err, errlen, "binary model file is truncated (array)");
                    ok = 0;
                    break;
                }
                *arrs[i].f32 = malloc((cnt ? cnt : 1) * sizeof(float));
                memcpy(*arrs[i].f32, rest + off, (size_t)cnt * 4); /* little-endian host */
                off += (size_t)cnt * 4;
            }
            *arrs[i].n = cnt;
        }
        if (ok && off != rest_n) {
            ferr(err, errlen, "binary model file has unexpected trailing bytes");
            ok = 0;
        }
    } else {
        for (int i = 0; i < na && ok; i++)
            if (json_array(jsrc[i], arrs[i]) != 0) {
                ferr(err, errlen, "malformed array in JSON model file");
                ok = 0;
            }
    }
    free(arrs);
    free(jsrc);
    jfree(root);
    if (!ok) {
        or_model_free(m);
        return NULL;
    }
    /* checkBlockShapes (checkpoint.go:216-225) */
    for (int b = 0; b < m->nblocks; b++)
        if (m->blocks[b].w1.n != (size_t)(2 * m->H * 3 * m->D)) {
            ferr(err, errlen, "rule_w1 shape does not match 2*hidden*3*state");
            or_model_free(m);
            return NULL;
        }
    if (m->tied) {
        free(m->head_w.data);
        m->head_w.data = NULL;
        m->head_w.n = 0;
    }
    /* Derived layout. */
    m->latch_base = malloc(sizeof(float) * (size_t)(m->D ? m->D : 1));
    or_latch_base_logits(m->D, m->latch_base);
    m->step_offset = malloc(sizeof(int) * (size_t)(m->nblocks ? m->nblocks : 1));
    int total = 0, longest = 0;
    for (int b = 0; b < m->nblocks; b++) {
        m->step_offset[b] = total;
        total += m->blocks[b].steps;
        for (int s = 0; s < m->blocks[b].steps; s++) {
            int d = or_step_dilation(m->blocks[b].initial_dilation, m->blocks[b].dilation_base, s);
            if (d > longest) longest = d;
        }
    }
    m->total_steps = total;
    m->ring = longest + 1;
    m->attn_cache = m->attn_window > 0 ? m->attn_window : m->max_context;
    return m;
}

void or_model_info(const or_model* m, int* o) {
    o[0] = m->vocab;
    o[1] = m->D;
    o[2] = m->H;
    o[3] = m->nblocks;
    o[4] = m->max_context;
    o[5] = m->attn_heads;
    o[6] = m->attn_window;
    o[7] = m->ring;
    o[8] = m->attn_cache;
    o[9] = m->total_steps;
}

void or_model_dilations(const or_model* m, int* out) {
    int k = 0;
    for (int b = 0; b < m->nblocks; b++)
        for (int s = 0; s < m->blocks[b].steps; s++)
            out[k++] = or_step_dilation(m->blocks[b].initial_dilation, m->blocks[b].dilation_base, s);
}
