/* Oracle internals — TEST INFRASTRUCTURE ONLY (see oracle.h). */
#ifndef MIGNON_OR_INTERNAL_H
#define MIGNON_OR_INTERNAL_H

#include "oracle.h"

typedef struct {
    int8_t* data;
    size_t n;
    float scale;
} or_tensor;

/* quant.Block (internal/quant/model.go:15-26) and blockAttention (attention.go:16-20) */
typedef struct {
    int steps, dilation_base, initial_dilation;
    or_tensor w1, w2, wsel;
    float *b1, *b2, *gamma;
    size_t n_b1, n_b2, n_gamma;
    int has_attn;
    float* attn_norm;
    size_t n_attn_norm;
    or_tensor qkv, out;
} or_block;

/* quant.Model (internal/quant/model.go:34-68), weights only; scratch lives in or_scratch. */
struct or_model {
    int vocab, D, H, tied, nblocks;
    or_tensor embed;
    or_block* blocks;
    float* final_norm;
    size_t n_final_norm;
    or_tensor head_w;
    float* head_b;
    size_t n_head_b;
    int max_context, attn_heads, attn_window;
    float* latch_base;
    int* step_offset;
    int total_steps, ring, attn_cache;
};

/* quantSeqState (internal/quant/stream.go:21-35) */
typedef struct {
    int n;
    float* norm;  /* [total_steps][ring][D] */
    float* latch; /* [total_steps][D] */
    float* attn_k;/* [nblocks][attn_cache*D] */
    float* attn_v;
    float* attn_scores;  /* attn_cache */
    float* attn_scratch; /* attn_cache */
    float *cur, *next, *block_in;
    float* bufs; /* backing store of cur/next/block_in */
} or_state;

/* The per-model scratch vectors of quant.Model (model.go:52-66, attention.go:57-67). */
typedef struct {
    float *mlp_input, *mlp_hidden, *mlp_output, *xhat, *norm_scratch, *logits, *mlp_gate, *latch_logit;
    float *a_norm, *a_xhat, *a_qkv, *a_att, *a_proj;
} or_scratch;

or_state* or_state_new(const or_model* m);
void or_state_free(or_state* st);
or_scratch* or_scratch_new(const or_model* m);
void or_scratch_free(or_scratch* s);
void or_append_position(const or_model* m, or_state* st, or_scratch* sc, int token, int need_output);
void or_head_logits(const or_model* m, or_scratch* sc, const float* cell, float* out);
void or_prefill(const or_model* m, or_state* st, or_scratch* sc, const int32_t* tokens, int n, float* out);

#endif
