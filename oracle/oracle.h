/*
 * CPU oracle for mignon-ai's INT8 inference path — TEST INFRASTRUCTURE ONLY.
 *
 * A C restatement of the reference's Go INT8 streaming engine (internal/quant) and the kernels it
 * calls (internal/kernels, internal/nn, internal/ca helpers), following the reference's float32
 * operation order, including the AVX2/FMA summation order of its Go-assembler kernels
 * (internal/kernels/vec_amd64.s). Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it; it is the checker, never the product path.
 *
 * Parity pinning: the reference is Go and no Go toolchain exists on these machines, so no output
 * of the reference itself could be recorded. The restatement is pinned by the known-answer cases
 * and properties of the reference's own tests (see tests/test_oracle_*.py): int8 dot products
 * (internal/kernels/int8_test.go), matvec, FastExp accuracy (accuracy_test.go), quantizer
 * round trip (internal/quant/tensor_test.go), model file round trip and damage rejection
 * (internal/quant/binary_test.go, internal/binfmt/binfmt_test.go), session == full pass bit
 * identity (internal/quant/session_test.go), bounded session state, dilation schedule
 * (internal/ca/layout_test.go) and greedy probabilities (internal/generate/greedy_test.go).
 */
#ifndef MIGNON_ORACLE_H
#define MIGNON_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct or_model or_model;
typedef struct or_session or_session;

/* ---- kernels (internal/kernels, internal/nn) ---- */
/* Selects the AVX2-order implementations (1, default) or the pure-Go-order ones (0), like the
 * reference's HasAVX2 switch (internal/kernels/cpu_features.go:8). */
void or_set_avx2(int on);
int or_get_avx2(void);
float or_dot_i8_f32(const float* x, const int8_t* w, int n);
float or_dot_f32(const float* x, const float* y, int n);
void or_add_scaled_f32(float* y, const float* x, float alpha, int n);
void or_vec_exp_f32(float* dst, const float* src, int n);
float or_fast_exp_f32(float x);
void or_matvec_i8(float* y, int rows, const int8_t* w, int stride, float scale, const float* x, int cols,
                  const float* bias);
float or_rmsnorm_f32(const float* x, const float* gamma, float* out, float* xhat, int d, float eps);
void or_softmax_f32(float* logits, float* scratch, int n);
float or_sigmoid_clamped(float x);

/* ---- layout helpers (internal/ca) ---- */
int or_step_dilation(int initial, int base, int step);
void or_latch_base_logits(int d, float* out);

/* ---- quantizer (internal/quant/tensor.go) ---- */
float or_quantize_tensor(const float* w, size_t n, int8_t* out);

/* ---- model file (internal/quant/checkpoint.go, internal/binfmt) ---- */
/* Parses a binary (MGNN) or JSON INT8 model file. Returns NULL and fills err on failure. */
or_model* or_model_decode(const uint8_t* data, size_t n, char* err, size_t errlen);
void or_model_free(or_model* m);
/* vocab, state, hidden, blocks, max_context, attn_heads, attn_window, ring, attn_cache, total_steps */
void or_model_info(const or_model* m, int* out10);
/* Writes the dilation of every (block, step) in order. */
void or_model_dilations(const or_model* m, int* out);

/* ---- engine (internal/quant/stream.go, attention.go, model.go, session.go) ---- */
/* quant.(*Model).Call: logits (float32, vocab entries) for the last position of window. Returns 0,
 * or -1 for an empty window. Uses per-call scratch (thread safe). */
int or_model_call(const or_model* m, const int32_t* window, int n, float* logits);
or_session* or_session_new(const or_model* m, int context_size);
void or_session_free(or_session* s);
/* Session.Prefill: returns 1 with logits filled, 0 when tokens is empty (nil logits). */
int or_session_prefill(or_session* s, const int32_t* tokens, int n, float* logits);
/* Session.Append: always returns 1 with logits filled. */
int or_session_append(or_session* s, int32_t token, float* logits);
/* quantSession.StateBytes (session.go:65-68) */
long or_session_state_bytes(const or_session* s);
int or_session_position(const or_session* s);

/* ---- token selection (internal/generate, internal/eval) ---- */
/* argmaxProb (greedy.go:90-102) over float64 logits widened from float32. */
int or_argmax_prob(const float* logits, int n, double* prob);
/* logProb (eval/suite.go:201-209) */
double or_log_prob(const float* logits, int n, int id);
/* Philox4x32-10: out[4] for counter c[4] and key k[2]. */
void or_philox4x32(const uint32_t c[4], const uint32_t k[2], uint32_t out[4]);
double or_sample_uniform(uint32_t session, uint32_t step);
/* Truncated sampling of SampleRawLogitsAdvanced (generate/sample.go:33-172) with repPenalty 1 and
 * topP 1, the uniform draw u supplied by the caller (the reference uses math/rand). */
int or_sample_topk(const float* logits, int n, double temperature, int topk, double u);

/* Sampling parameters of sampleContinuation / SampleRawLogitsAdvanced (generate/chat.go:45-56). */
typedef struct {
    double temperature; /* <= 0.001: argmax */
    double rep_penalty; /* > 1: the window's distinct tokens are penalised */
    int top_k;          /* <= 0: off */
    double top_p;       /* in (0, 1): nucleus cutoff; else off */
    int rep_window;     /* trailing tokens of prefix ++ generated the penalty sees; <= 0: all */
    int ban_trigrams;   /* the 3-gram repetition block of sampleContinuation (sample.go:213-227) */
} or_sampling;
/* One token of sampleContinuation's loop body (sample.go:206-232) over float64 logits, modified in
 * place: 3-gram ban over gen, constraint mask (allowed[i] < 0 masks token i; NULL: none),
 * repetition penalty over the window of prefix ++ gen, then SampleRawLogitsAdvanced
 * (sample.go:33-172) with the draw u. *prob = the chosen token's probability in the distribution
 * it was drawn from (argmax: 1 / sum exp(l - max)). */
int or_sample_policy(double* logits, int n, const int32_t* prefix, int n_prefix, const int32_t* gen, int n_gen,
                     const or_sampling* sp, const int32_t* allowed, double u, double* prob);

/* ---- batch runners (OpenMP over sessions; one engine state per session) ---- */
/* Greedy generation (greedyLoop, greedy.go:63-87, no stop tokens): for each session s,
 * prompts[s*stride : s*stride+lens[s]]; writes n_new tokens and probs per session, and if
 * logits != NULL the float32 logits of every step (n_sess*n_new*vocab). Returns 0. */
int or_generate_greedy(const or_model* m, int n_sess, const int32_t* prompts, int stride, const int32_t* lens,
                       int context_size, int n_new, int32_t* out_tokens, float* out_probs, float* out_logits,
                       int nthreads);
/* Sampled generation with T/top-k and the per-session Philox draw or_sample_uniform(s0+s, step). */
int or_generate_sample(const or_model* m, int n_sess, const int32_t* prompts, int stride, const int32_t* lens,
                       int context_size, int n_new, double temperature, int topk, uint32_t session0,
                       int32_t* out_tokens, float* out_logits, int nthreads);
/* sampleContinuation (generate/sample.go:196-247) per session: the policy of or_sample_policy
 * with the draw or_sample_uniform(s0 + s, step), the prompt as penalty prefix when
 * penalize_prompt, a token automaton dfa[n_states][vocab] (next state, -1 = not allowed; NULL:
 * none) starting in dfa_start[s] (< 0: unconstrained), and stop tokens that end a session before
 * they are emitted. Unused columns: token -1, prob 0; out_lens[s] = tokens emitted. */
int or_generate_policy(const or_model* m, int n_sess, const int32_t* prompts, int stride, const int32_t* lens,
                       int context_size, int n_new, const or_sampling* sp, int penalize_prompt, const int32_t* dfa,
                       const int32_t* dfa_start, uint32_t session0, const int32_t* stops, int n_stops,
                       int32_t* out_tokens, float* out_probs, int32_t* out_lens, float* out_logits, int nthreads);
/* Scoring: for each sequence, the log-prob of tokens[t] given tokens[:t] for t = 1..len-1. */
int or_score(const or_model* m, int n_seq, int len, const int32_t* tokens, double* out_logprobs, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
