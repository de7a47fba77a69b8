/*
 * libmignoncuda — C-ABI of the B200 (sm_100a) engine for mignon-ai's INT8 inference path.
 *
 * Plain C types only: pointers, sizes, status codes. Every function returns an mc_status
 * (0 = MC_OK); mc_last_error() returns a thread-local message for the last failure. The caller
 * owns host buffers; the library owns device memory it allocates. Functions whose names end in
 * _dev take device pointers and a CUDA stream (cudaStream_t passed as void*) and do not
 * synchronize; all others take host pointers and return when their results are in host memory.
 *
 * Each entry point names the reference interface it replaces (paths relative to the
 * mignon-ai repository).
 */
#ifndef MIGNON_CUDA_H
#define MIGNON_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  MC_OK = 0,
  MC_INVALID_ARGUMENT = 1,
  MC_CUDA_ERROR = 2,
  MC_BAD_MODEL = 3,
  MC_OUT_OF_MEMORY = 4,
  MC_DEVICE_TIMEOUT = 5,
  MC_UNSUPPORTED = 6
} mc_status;

/* Message of the last failed call on this thread ("" after a success). */
const char* mc_last_error(void);

/* Library version: major*10000 + minor*100 + patch. */
int mc_version(void);

/* ---------------------------------------------------------------------------------------------
 * Isolated INT8 GEMMs (the INT8 product kernels.MatVecInt8, internal/kernels/int8.go:31-41,
 * batched over rows; the config-5 sweep entry point).
 * ------------------------------------------------------------------------------------------- */

/* C[m,n] = sum_k A[m,k] * W[n,k] with int8 A [M x K] and W [N x K] (row-major, K contiguous),
 * exact s32 accumulators. Writes c_i32 [M x N] if non-null and
 * y[m,n] = ((float)C[m,n] * row_scale[m]) * col_scale[n] + bias[n] if y is non-null (null scales
 * count as 1, a null bias as 0). Requires N % 256 == 0, K % 16 == 0. Device pointers. */
int mc_gemm_i8_dev(const int8_t* a, const int8_t* w, int m, int n, int k, const float* row_scale,
                   const float* col_scale, const float* bias, int32_t* c_i32, float* y, void* stream);

/* y[m,n] = dot(x[m,:], W[n,:]) * w_scale + bias[n] with float32 activations x [M x K], as
 * MatVecInt8 (int8.go:33-41) computes it per row. Each row is sliced into three int8 digit
 * planes; if slices is non-null the three exact s32 plane accumulators are written to it
 * ([3 x M x N]). row_max_scratch: device float[M]. Requires N % 128 == 0, K % 16 == 0. */
int mc_gemm_f32a_dev(const float* x, const int8_t* w, int m, int n, int k, float w_scale, const float* bias,
                     float* y, int32_t* slices, float* row_max_scratch, void* stream);

/* mc_gemm_f32a_dev without any device allocation, for callers that cannot allocate GPU memory
 * (a host runtime limited to buffers it registered in advance, or a service whose GPU memory is
 * budgeted once at start-up). It has no counterpart in the reference. Its only scratch, one float
 * per activation row, is a fixed device array of 65536 entries (256 KB, held by every GPU that
 * loads the library until exit): m above 65536 fails with MC_INVALID_ARGUMENT, as do the shapes
 * mc_gemm_f32a_dev rejects, before any CUDA call. The first call on each device looks up that
 * array's device address and sets the kernels' shared-memory attribute on it (no allocation;
 * serialized by a lock, so first calls from several host threads are safe); make it before any
 * stream capture. Device ordinals 0..63. All calls share the array; calls that overlap on the GPU
 * race on it and must be serialized by the caller. */
int mc_gemm_f32a_noalloc_dev(const float* x, const int8_t* w, int m, int n, int k, float w_scale, const float* bias,
                             float* y, void* stream);

/* Host-pointer form of mc_gemm_i8_dev: copies in, runs on `device`, copies out. */
int mc_gemm_i8(int device, const int8_t* a, const int8_t* w, int m, int n, int k, const float* row_scale,
               const float* col_scale, const float* bias, int32_t* c_i32, float* y);

/* ---------------------------------------------------------------------------------------------
 * Engine: models, session batches, prefill / append / generate.
 * ------------------------------------------------------------------------------------------- */
typedef struct mc_ctx mc_ctx;
typedef struct mc_model mc_model;
typedef struct mc_batch mc_batch;

typedef struct {
  int n_devices;       /* 0: device 0 only */
  const int* devices;  /* CUDA device ordinals; a batch's sessions are split evenly across them */
} mc_options;

/* Opens a context over one or more GPUs of this process. */
int mc_open(const mc_options* opt, mc_ctx** out);
int mc_close(mc_ctx* ctx);

/* Parses an INT8 model file (binary mignon.model/1 or legacy JSON) and uploads a replica of the
 * weights to every device of the context. Replaces quant.Decode (internal/quant/checkpoint.go:162)
 * followed by quant.NewModel (model.go:91). Damaged files fail with MC_BAD_MODEL. */
int mc_load_model(mc_ctx* ctx, const uint8_t* data, size_t n, mc_model** out);
/* A full-precision (float32) model file instead of an INT8 one: pkg/model.Decode of a binfmt
 * kind-1 file (pkg/model/model.go:85-103; checkpoint.Encode, internal/checkpoint/checkpoint.go:86-94)
 * followed by quant.Quantize (internal/quant/convert.go:8-98), the quantization on the context's
 * first device: per-matrix max|w| and NewTensorF32's rounding (internal/quant/tensor.go:12-42)
 * run as kernels over the uploaded weight vector. max_context is Quantize's maxContext (<= 0: the
 * file's context_size, or 64 when it has none, as pkg/model normalizes it). The result is the
 * model an INT8 file of the same weights would give. */
int mc_load_model_full(mc_ctx* ctx, const uint8_t* data, size_t n, int max_context, mc_model** out);
int mc_model_free(mc_model* model);

/* out[10] = vocab, state, hidden, blocks, max_context, attn_heads, attn_window, total rule steps,
 * norm ring length (longest dilation + 1), attention cache length. (quant.Model accessors,
 * model.go:71-89, and the cache sizes of stream.go:39-47, attention.go:46-52.) */
int mc_model_info(const mc_model* model, int32_t* out);

/* Opens `count` sessions of one model: count x quant.(*Model).NewSession(context_size)
 * (internal/quant/session.go:20-28; window = min(context_size, max_context), context_size <= 0
 * meaning max_context). max_prompt bounds the prompts of later prefill/generate calls (<= 128);
 * top_k (0..64) sizes the sampler. The sessions' state lives in device memory. */
int mc_batch_open(mc_model* model, int count, int context_size, int max_prompt, int top_k, mc_batch** out);
int mc_batch_close(mc_batch* batch);

/* Session.Prefill for every session (session.go:30-39): session s restarts from
 * tokens[s*stride .. s*stride+lens[s]) trimmed to its last `window` tokens. Writes, per session,
 * the logits after the last token (if logits != NULL, [count x vocab] float32 — the reference
 * returns them widened to float64), the greedy next token and its probability (argmaxProb,
 * internal/generate/greedy.go:90-102). Sessions with lens[s] == 0 are left idle (nil logits). */
int mc_prefill(mc_batch* batch, const int32_t* tokens, const int32_t* lens, int stride, float* logits, int32_t* next,
               float* prob);

/* Session.Append for every session (session.go:41-56, the streaming path appendPosition +
 * headLogits): appends tokens[s] to session s and writes the logits after it, the greedy next
 * token and its probability. */
int mc_append(mc_batch* batch, const int32_t* tokens, float* logits, int32_t* next, float* prob);

/* Per-token log-probabilities of whole sequences (the scoring workload): session s restarts from
 * seqs[s*stride .. s*stride+lens[s]) and out[s*(stride-1) + t] = log p(seqs[t+1] | seqs[0..t])
 * for t < lens[s]-1 — logProb (internal/eval/suite.go:201-209) of the logits Call(prefix) gives
 * (model.go:122-132), all prefixes in one prefill pass; other entries are 0. Requires
 * lens[s] <= the sessions' window and the batch's max_prompt, and target ids inside the
 * vocabulary. Afterwards the sessions continue as after mc_prefill of the same tokens. */
int mc_score(mc_batch* batch, const int32_t* seqs, const int32_t* lens, int stride, double* out);

/* mc_score with the scored tokens given: out[s*stride + t] = log p(targets[s*stride + t] |
 * seqs[s][0..t]) for t < lens[s] — the loss terms of nll.score (internal/eval/eval.go:27-43) for
 * windows whose last target lies past the window itself (Perplexity / PerplexityPerDoc beyond the
 * context, eval.go:55-60, perdoc.go:16-32); other entries are 0. Same limits as mc_score
 * (lens[s] <= window and max_prompt; targets inside the vocabulary); afterwards the sessions
 * continue as after mc_prefill of seqs. */
int mc_score_targets(mc_batch* batch, const int32_t* seqs, const int32_t* lens, int stride, const int32_t* targets,
                     double* out);

/* The decode loop of generate.greedyLoop (internal/generate/greedy.go:63-87) without stop tokens,
 * or with temperature > 0 the sampled loop of sampleContinuation (generate/sample.go:196-247)
 * with top-k = the batch's top_k, no repetition penalty, top-p 1: prefill each prompt, then
 * n_new tokens per session, all steps on the device (one CUDA graph per step). Sampling draws
 * its uniform from Philox4x32-10 keyed by (session0 + s, "SAMP") with counter = step.
 * Writes out_tokens [count x n_new] and, if non-null, out_probs [count x n_new] (greedy only). */
int mc_generate(mc_batch* batch, const int32_t* prompts, const int32_t* lens, int stride, int n_new, double temperature,
                uint32_t session0, int32_t* out_tokens, float* out_probs);

/* mc_generate with stop tokens (greedyLoop's `stops`, internal/generate/greedy.go:63-87): a
 * session ends before the first token among stops[0..n_stops) it would emit (n_stops <= 8); its
 * remaining out_tokens entries are -1 (out_probs 0) and out_lens[s] is the number of tokens it
 * emitted (n_new when no stop came). The session stays after its last emitted token. */
int mc_generate_stops(mc_batch* batch, const int32_t* prompts, const int32_t* lens, int stride, int n_new,
                      double temperature, uint32_t session0, const int32_t* stops, int n_stops, int32_t* out_tokens,
                      float* out_probs, int32_t* out_lens);

/* mc_generate with a token limit per session: pkg/infer.Generate with Options.MaxTokens
 * (pkg/infer/infer.go:64-96) per session, greedy (temperature <= 0.001) or sampled like
 * mc_generate (top-k = the batch's top_k, Philox keyed by (session0 + s, "SAMP"), counter = the
 * token index). Session s emits max_tokens[s] tokens (1 <= max_tokens[s] <= n_max); out_tokens
 * [count x n_max] holds them, then -1; out_lens (if non-null) the counts. A session that has
 * emitted its tokens sits out the remaining steps (its attention rows are not read). */
int mc_generate_limits(mc_batch* batch, const int32_t* prompts, const int32_t* lens, int stride,
                       const int32_t* max_tokens, int n_max, double temperature, uint32_t session0,
                       int32_t* out_tokens, float* out_probs, int32_t* out_lens);

/* The knobs of generate.Sampling (internal/generate/chat.go:45-56) for the policy calls below. */
typedef struct {
  double temperature; /* <= 0.001: argmax (sample.go:71-82) */
  double rep_penalty; /* > 1: each distinct token of the window is divided (logit > 0) or multiplied by it */
  int top_k;          /* <= 0: off */
  double top_p;       /* in (0, 1): nucleus cutoff; otherwise off */
  int rep_window;     /* trailing tokens the penalty sees (sampleContinuation: ChatRepetitionWindow = 6,
                         generate/constants.go:11); <= 0: all */
  int ban_trigrams;   /* non-zero: sampleContinuation's 3-gram repetition block (sample.go:213-227) */
} mc_sampling;

/* sampleContinuation (internal/generate/sample.go:196-247) for every session: prefill the prompt,
 * then up to n_new tokens, each chosen on the device by the whole policy — 3-gram block,
 * constraint mask, repetition penalty over the last rep_window tokens of (the prompt when
 * penalize_prompt, chat.go:72; else nothing, chat.go:122) ++ the generated tokens, then
 * SampleRawLogitsAdvanced (sample.go:33-172) with temperature, top-k, top-p and the draw of
 * sampleFromCDF (:174-191) from Philox4x32-10 keyed like mc_generate. The constraint
 * (Constraint.Mask / Advance, chat.go:58-62) is a token automaton: dfa[state * vocab + token] is
 * the next state, or -1 for a token that is not allowed (its logit becomes -1e300 like
 * constrain/grammar.go:259); dfa_start[s] is session s's start state (< 0: unconstrained);
 * dfa == NULL: no constraint. Stop tokens (<= 8) end a session before it would emit one. Writes
 * out_tokens [count x n_new] (-1 after a session ended), out_probs (the chosen token's
 * probability in the distribution it was drawn from) and out_lens (tokens emitted) when non-null.
 * Vocabulary <= 16384. */
int mc_generate_policy(mc_batch* batch, const int32_t* prompts, const int32_t* lens, int stride, int n_new,
                       const mc_sampling* sampling, int penalize_prompt, const int32_t* dfa, int n_states,
                       const int32_t* dfa_start, uint32_t session0, const int32_t* stops, int n_stops,
                       int32_t* out_tokens, float* out_probs, int32_t* out_lens);

/* SampleRawLogitsAdvanced (internal/generate/sample.go:33-172) over n rows of float32 logits
 * [n x vocab] on one device. recent (row stride recent_stride, recent_lens[r] tokens; NULL: none)
 * are row r's recent tokens: the penalty sees their last rep_window, and with ban_trigrams they are
 * the generated tokens the 3-gram block scans. allowed [n x vocab] (NULL: none) masks token t of
 * row r when allowed[r * vocab + t] < 0. u [n] are the uniform draws in [0, 1) (NULL: Philox of
 * (session0 + r, step)). Writes out_tokens [n] and, if non-null, out_probs [n]. Vocabulary <= 16384. */
int mc_sample_rows(int device, const float* logits, int n, int vocab, const int32_t* recent, const int32_t* recent_lens,
                   int recent_stride, const int32_t* allowed, const mc_sampling* sampling, const double* u,
                   uint32_t session0, uint32_t step, int32_t* out_tokens, float* out_probs);

/* Continuous batching: a scheduler over `slots` sessions of one model (sharded over the
 * context's devices like mc_batch_open). Requests queue on the host; whenever at least
 * admit_min slots are free (default slots / 8) or none is running, queued requests are admitted
 * into the free slots by one prefill pass in which the running slots keep their state, and all
 * running slots then decode together. Each request runs sampleContinuation
 * (internal/generate/sample.go:196-247) with the scheduler's sampling knobs, the prompt as
 * penalty prefix when penalize_prompt (which needs rep_window >= 1), its own token limit and the
 * scheduler's stop tokens, its draws keyed by its draw_key and its token index (as
 * mc_generate_policy keys session s by session0 + s), so its tokens do not depend on which slot
 * it ran in or what ran beside it. Prompts: at most max_prompt tokens after trimming to the
 * window; token limits: 1 to max_new. */
typedef struct mc_sched mc_sched;
int mc_sched_open(mc_model* model, int slots, int context_size, int max_prompt, int max_new,
                  const mc_sampling* sampling, int penalize_prompt, const int32_t* stops, int n_stops, mc_sched** out);
int mc_sched_close(mc_sched* sched);
/* Queues a request; *id = its index (0, 1, 2, ... in submission order). An empty prompt finishes
 * with no tokens (Prefill of nothing returns no logits). */
int mc_sched_submit(mc_sched* sched, const int32_t* prompt, int len, int n_new, uint32_t draw_key, int64_t* id);
/* One round: admission where due, `steps` decode steps, then the finished requests are collected.
 * *in_flight = requests queued or running afterwards. */
int mc_sched_step(mc_sched* sched, int steps, int* in_flight);
/* Rounds of steps_per_poll decode steps until no request is queued or running. */
int mc_sched_run(mc_sched* sched, int steps_per_poll);
/* A finished request's tokens (and probabilities, like mc_generate_policy's): *n = its token
 * count, of which the first `capacity` are copied; *n = -1 while it is queued or running. */
int mc_sched_result(mc_sched* sched, int64_t id, int32_t* tokens, float* probs, int capacity, int* n);
/* out[10] = prefill passes, decode steps, tokens emitted, requests finished, requests in flight,
 * then microseconds: device time of the admission passes, device time of the decode steps, wall
 * time inside mc_sched_step / mc_sched_run, host time choosing and staging admissions; then the
 * requests admitted into slots so far. */
int mc_sched_stats(const mc_sched* sched, int64_t* out);
/* Admit when at least admit_min slots are free (or none is running). */
int mc_sched_set_admit_min(mc_sched* sched, int admit_min);

/* mc_generate with device-resident inputs and outputs on a single-device batch: enqueues the
 * whole job on the batch's stream (mc_batch_stream) and returns without synchronizing.
 * pmax >= every lens[s]. Check completion and device errors with mc_batch_error. */
int mc_generate_dev(mc_batch* batch, const int32_t* d_prompts, const int32_t* d_lens, int stride, int pmax, int n_new,
                    double temperature, uint32_t session0, int32_t* d_out_tokens, float* d_out_probs);

/* mc_generate_limits with device-resident prompts, lengths, limits and outputs on a
 * single-device batch (like mc_generate_dev): enqueues the job and returns without synchronizing.
 * Limits outside [1, n_max] are not checked on the host: a session emits at least one token and
 * at most n_max. */
int mc_generate_limits_dev(mc_batch* batch, const int32_t* d_prompts, const int32_t* d_lens, int stride, int pmax,
                           const int32_t* d_max_tokens, int n_max, double temperature, uint32_t session0,
                           int32_t* d_out_tokens, float* d_out_probs);

/* The int8 rate of this device's tensor pipe, the denominator of the INT8 roofline fractions (no
 * counterpart in the reference: a measurement). One CTA per multiprocessor issues back-to-back
 * tcgen05.mma kind::i8 instructions of the largest single-CTA shape (M 128, N 256, K 32) on
 * operands resident in shared memory, with nothing else to do; `launches` launches of `iters`
 * MMA groups (4 instructions, K 128) each are timed with CUDA events. *tops = int8 tera-ops/s
 * (2 ops per multiply-add), *ms = milliseconds per launch. iters in [1, 2^22]. */
int mc_probe_mma_i8(int device, int iters, int launches, double* tops, double* ms);

/* Exercises the device-error path without a fault (no counterpart in the reference): a kernel
 * waits on a barrier that nothing completes; its bounded wait gives up after 2 s, records the
 * device error word and returns. Returns MC_DEVICE_TIMEOUT (any other status means the path is
 * broken); the device stays usable afterwards. */
int mc_selftest_wait_timeout(int device);

/* The CUDA stream (cudaStream_t) the batch's work on device shard `shard` runs on. */
int mc_batch_stream(mc_batch* batch, int shard, void** stream);

/* Waits for the batch's work and reports a device-side error (MC_DEVICE_TIMEOUT) if any. */
int mc_batch_error(mc_batch* batch);

/* Runs one greedy decode step of a single-device batch launch by launch, timing each launch with
 * CUDA events: ms[i] and kinds[i] (0 block, 1 attention, 2 final block, 3 head, 4 select) for
 * i < *n_launches <= max_launches. The step advances the sessions. */
int mc_profile_step(mc_batch* batch, int max_launches, float* ms, int32_t* kinds, int* n_launches);

#ifdef __cplusplus
}
#endif
#endif /* MIGNON_CUDA_H */
