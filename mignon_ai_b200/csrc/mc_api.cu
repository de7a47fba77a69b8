// C-ABI entry points of libmignoncuda (include/mignon_cuda.h).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <vector>

#include "../../include/mignon_cuda.h"
#include "mc_engine.cuh"
#include "mc_host.h"

namespace mc {
const char* last_error_cstr();
int gemm_i8_launch(const int8_t* a, const int8_t* w, int M, int N, int K, const float* row_scale,
                   const float* col_scale, const float* bias, int32_t* c_i32, float* y, cudaStream_t stream);
int gemm_f32a_launch(const float* a, const int8_t* w, int M, int N, int K, float w_scale, const float* bias,
                     float* y, int32_t* slices, float* row_max_scratch, cudaStream_t stream);
int gemm_f32a_noalloc_launch(const float* a, const int8_t* w, int M, int N, int K, float w_scale, const float* bias,
                             float* y, cudaStream_t stream);

// Device buffer released when the scope ends.
struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};
}  // namespace mc

using namespace mc;
using namespace mc::eng;

struct mc_ctx {
  std::vector<int> devices;
};

struct mc_model {
  mc_ctx* ctx = nullptr;
  HostModel host;
  std::vector<std::unique_ptr<DevModel>> dev;  // one replica per device
};

struct mc_batch {
  mc_model* model = nullptr;
  int count = 0, window = 0, pmax = 0, topk = 0;
  std::vector<int> first;                       // first session of each device shard
  std::vector<std::unique_ptr<DevBatch>> shard;  // one per device
};

namespace {

int shard_sizes(int count, int ndev, std::vector<int>& first) {
  first.resize(ndev + 1);
  for (int g = 0; g <= ndev; ++g) first[g] = (int)((long long)count * g / ndev);
  return kOk;
}

int sync_all(mc_batch* b) {
  int st = kOk;
  for (auto& sh : b->shard) {
    if (!sh || sh->S == 0) continue;
    cudaSetDevice(sh->m->device);
    int e = check_device_error(sh->stream);
    if (e != kOk && st == kOk) st = e;
  }
  return st;
}

// Pinned host staging of a step's transfers (DevBatch::h_step): [tokens S | next S | prob S |
// device error word, padding 4 | logits S x V]. Sized before a call writes into it, so it is never
// reallocated while one of its copies is pending (every call synchronizes before returning).
int ensure_h_step(DevBatch& sh, bool logits) {
  const size_t S = (size_t)sh.S, need = 3 * S + 4 + (logits ? S * sh.m->V : 0);
  if (sh.h_step_n < need) {
    if (sh.h_step) MC_CUDA(cudaFreeHost(sh.h_step));
    sh.h_step = nullptr;
    sh.h_step_n = 0;
    MC_CUDA(cudaHostAlloc(&sh.h_step, need * 4, cudaHostAllocDefault));
    sh.h_step_n = need;
  }
  return kOk;
}

// Copies per-session host outputs back after a step that wrote column 0 of out_tok/out_prob: the
// outputs and the device error word go to each shard's pinned staging asynchronously (copies into
// the caller's pageable memory would each be staged and synchronous inside the driver), then one
// stream synchronization per shard, then plain host copies out.
int copy_step_outputs(mc_batch* b, float* logits, int32_t* next, float* prob) {
  int st;
  for (size_t g = 0; g < b->shard.size(); ++g) {
    DevBatch& sh = *b->shard[g];
    if (sh.S == 0) continue;
    MC_CUDA(cudaSetDevice(sh.m->device));
    if ((st = ensure_h_step(sh, logits != nullptr)) != kOk) return st;
    const size_t S = (size_t)sh.S, pitch = (size_t)sh.out_stride * 4;  // column 0 of [S x out_stride]
    int32_t* hs = sh.h_step;
    if (next) MC_CUDA(cudaMemcpy2DAsync(hs + S, 4, sh.out_tok, pitch, 4, S, cudaMemcpyDeviceToHost, sh.stream));
    if (prob) MC_CUDA(cudaMemcpy2DAsync(hs + 2 * S, 4, sh.out_prob, pitch, 4, S, cudaMemcpyDeviceToHost, sh.stream));
    if (logits)
      MC_CUDA(cudaMemcpyAsync(hs + 3 * S + 4, sh.logits, S * sh.m->V * 4, cudaMemcpyDeviceToHost, sh.stream));
    MC_CUDA(cudaMemcpyFromSymbolAsync(hs + 3 * S, g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, sh.stream));
  }
  st = kOk;
  for (size_t g = 0; g < b->shard.size(); ++g) {
    DevBatch& sh = *b->shard[g];
    if (sh.S == 0) continue;
    MC_CUDA(cudaSetDevice(sh.m->device));
    MC_CUDA(cudaStreamSynchronize(sh.stream));
    const size_t S = (size_t)sh.S, s0 = (size_t)b->first[g];
    const int32_t* hs = sh.h_step;
    if (hs[3 * S] != 0) {  // a bounded device wait gave up: clear the word and report it
      const int e = check_device_error(sh.stream);
      if (e != kOk && st == kOk) st = e;
      continue;
    }
    if (next) memcpy(next + s0, hs + S, S * 4);
    if (prob) memcpy(prob + s0, hs + 2 * S, S * 4);
    if (logits) memcpy(logits + s0 * sh.m->V, hs + 3 * S + 4, S * sh.m->V * 4);
  }
  return st;
}

int ensure_step_outputs(DevBatch& sh, bool logits, int stride, bool gmax = false) {
  int st;
  if (sh.out_stride < stride) {
    if ((st = sh.alloc(sh.out_tok, (size_t)sh.S * stride * 4)) || (st = sh.alloc(sh.out_prob, (size_t)sh.S * stride * 4)))
      return st;
    sh.out_stride = stride;
  }
  if (logits && !sh.logits && (st = sh.alloc(sh.logits, (size_t)sh.S * sh.m->V * 4))) return st;
  if (gmax && !sh.gmax && (st = sh.alloc(sh.gmax, (size_t)sh.S * kSelSamples * 4))) return st;
  return kOk;
}

// Uploads a prompt segment [count x stride] trimmed to each session's window into the shards'
// token buffers; sets pos = 0 and seglen = trimmed length. Returns the longest trimmed length.
int upload_prompts(mc_batch* b, const int32_t* tokens, const int32_t* lens, int stride, int* pmax_out) {
  int pmax = 0;
  for (int s = 0; s < b->count; ++s) {
    if (lens[s] < 0 || lens[s] > stride) return set_error(kInvalidArgument, "prompt length outside [0, stride]");
    pmax = std::max(pmax, std::min(lens[s], b->window));
  }
  if (pmax > b->pmax) return set_error(kInvalidArgument, "prompt longer than the batch's max_prompt");
  *pmax_out = std::max(pmax, 1);
  const int P = *pmax_out;
  for (size_t g = 0; g < b->shard.size(); ++g) {
    DevBatch& sh = *b->shard[g];
    if (sh.S == 0) continue;
    MC_CUDA(cudaSetDevice(sh.m->device));
    const int s0 = b->first[g];
    // pinned staging [tokens S*P | lengths S | zeros S | row map S], reused once the previous
    // upload's copies are done
    const size_t need = (size_t)sh.S * P + 3 * (size_t)sh.S;
    if (sh.h_stage_done) MC_CUDA(cudaEventSynchronize(sh.h_stage_done));
    else MC_CUDA(cudaEventCreateWithFlags(&sh.h_stage_done, cudaEventDisableTiming));
    if (sh.h_stage_n < need) {
      if (sh.h_stage) MC_CUDA(cudaFreeHost(sh.h_stage));
      sh.h_stage = nullptr;
      sh.h_stage_n = 0;
      MC_CUDA(cudaHostAlloc(&sh.h_stage, need * 4, cudaHostAllocDefault));
      sh.h_stage_n = need;
    }
    int32_t* tok = sh.h_stage;
    int32_t* len = tok + (size_t)sh.S * P;
    int32_t* zero = len + sh.S;
    int32_t* rowmap = zero + sh.S;
    const int spt = std::max(1, 128 / P);
    for (int i = 0; i < sh.S; ++i) {
      const int s = s0 + i;
      const int n = std::max(0, std::min(lens[s], b->window));
      const int32_t* src = tokens + (size_t)s * stride + (lens[s] - n);
      int32_t* dst = tok + (size_t)i * P;
      std::copy(src, src + n, dst);
      std::fill(dst + n, dst + P, 0);
      len[i] = n;
      zero[i] = 0;
      rowmap[i] = (i / spt) * 128 + (i % spt) * P + std::max(n - 1, 0);
    }
    MC_CUDA(cudaMemcpyAsync(sh.tok, tok, (size_t)sh.S * P * 4, cudaMemcpyHostToDevice, sh.stream));
    MC_CUDA(cudaMemcpyAsync(sh.seglen, len, sh.S * 4, cudaMemcpyHostToDevice, sh.stream));
    MC_CUDA(cudaMemcpyAsync(sh.pos, zero, sh.S * 4, cudaMemcpyHostToDevice, sh.stream));
    MC_CUDA(cudaMemcpyAsync(sh.rowmap, rowmap, sh.S * 4, cudaMemcpyHostToDevice, sh.stream));
    // a one-row segment runs through the decode kernels, which read each session's token from
    // next_tok
    if (P == 1) MC_CUDA(cudaMemcpyAsync(sh.next_tok, tok, sh.S * 4, cudaMemcpyHostToDevice, sh.stream));
    MC_CUDA(cudaEventRecord(sh.h_stage_done, sh.stream));
  }
  return kOk;
}

int run_graph_step(DevBatch& sh, int mode, double inv_temp, uint32_t session0, bool logits) {
  DevBatch::GraphKey key;
  key.mode = mode;
  key.logits = (int)logits;
  key.stride = sh.out_stride;
  key.inv_t = inv_temp;
  key.session0 = session0;
  key.out_tok = sh.out_tok;
  key.logits_buf = sh.logits;
  key.n_stops = sh.n_stops;
  for (int k = 0; k < sh.n_stops; ++k) key.stops[k] = sh.stops[k];
  key.pol = sh.pol;
  key.per_session = sh.per_session;
  if (!sh.graph || !(sh.graph_key == key)) {
    if (sh.graph) {
      cudaGraphExecDestroy(sh.graph);
      sh.graph = nullptr;
    }
    cudaGraph_t gph;
    MC_CUDA(cudaStreamBeginCapture(sh.stream, cudaStreamCaptureModeThreadLocal));
    int st = enqueue_forward(sh, 1, mode, inv_temp, session0, logits, false);
    cudaError_t e = cudaStreamEndCapture(sh.stream, &gph);
    if (st != kOk) {
      if (e == cudaSuccess) cudaGraphDestroy(gph);
      return st;
    }
    if (e != cudaSuccess) return set_error(kCudaError, std::string("stream capture: ") + cudaGetErrorString(e));
    e = cudaGraphInstantiate(&sh.graph, gph, 0);
    cudaGraphDestroy(gph);
    if (e != cudaSuccess) return set_error(kCudaError, std::string("graph instantiate: ") + cudaGetErrorString(e));
    sh.graph_key = key;
  }
  MC_CUDA(cudaGraphLaunch(sh.graph, sh.stream));
  return kOk;
}

// The n_new - 1 decode steps after a prefill: one captured step graph per step.
int run_decode_steps(DevBatch& sh, int n_new, int mode, double inv_temp, uint32_t session0) {
  for (int t = 1; t < n_new; ++t) {
    const int st = run_graph_step(sh, mode, inv_temp, session0, false);
    if (st != kOk) return st;
  }
  return kOk;
}

// Per-position log-probabilities of a prefill pass over seqs (the nll.score loop of
// internal/eval/eval.go:27-43 over every prefix, logProb of eval/suite.go:201-209).
// targets == null: position t is scored against seqs[t + 1] (t < lens - 1), out is
// [count x (stride - 1)]; else against targets[t] (t < lens), out is [count x stride].
int score_impl(mc_batch* b, const int32_t* seqs, const int32_t* lens, int stride, const int32_t* targets, double* out,
               const char* name) {
  const std::string fn(name);
  if (stride < 1) return set_error(kInvalidArgument, fn + ": stride < 1");
  const int V = b->model->dev[0]->V;
  auto target_of = [&](int s, int t) -> int32_t {
    return targets ? targets[(size_t)s * stride + t] : seqs[(size_t)s * stride + t + 1];
  };
  auto scored = [&](int s, int t) { return targets ? t < lens[s] : t + 1 < lens[s]; };
  for (int s = 0; s < b->count; ++s) {
    if (lens[s] < 0 || lens[s] > stride) return set_error(kInvalidArgument, fn + ": length outside [0, stride]");
    if (lens[s] > b->window)
      return set_error(kInvalidArgument, fn + ": sequence " + std::to_string(s) + " is longer than the session window");
    for (int t = 0; t < lens[s]; ++t)
      if (scored(s, t) && (target_of(s, t) < 0 || target_of(s, t) >= V))
        return set_error(kInvalidArgument, fn + ": target token outside the vocabulary");
  }
  int P = 1;
  int st = upload_prompts(b, seqs, lens, stride, &P);
  if (st != kOk) return st;
  const int cols = targets ? stride : stride - 1;
  std::fill(out, out + (size_t)b->count * cols, 0.0);
  for (size_t g = 0; g < b->shard.size(); ++g) {
    DevBatch& sh = *b->shard[g];
    if (sh.S == 0) continue;
    MC_CUDA(cudaSetDevice(sh.m->device));
    const int s0 = b->first[g];
    const size_t rows = (size_t)sh.S * P;
    if ((st = ensure_score_rows(sh, rows)) != kOk) return st;
    // row r = i * P + t: the final-normed row of position t of session i
    const int spt = std::max(1, 128 / P);
    std::vector<int32_t> rowmap(rows), target(rows, 0), valid(rows, 0), pos(sh.S), seglen(sh.S);
    for (int i = 0; i < sh.S; ++i) {
      const int n = lens[s0 + i];
      for (int t = 0; t < P; ++t) {
        const size_t r = (size_t)i * P + t;
        rowmap[r] = (i / spt) * 128 + (i % spt) * P + t;
        if (t < n && scored(s0 + i, t)) {
          target[r] = target_of(s0 + i, t);
          valid[r] = 1;
        }
      }
      pos[i] = n;  // afterwards the sessions continue as after mc_prefill of the same tokens
      seglen[i] = n > 0 ? 1 : 0;
    }
    MC_CUDA(cudaMemcpyAsync(sh.sc_rowmap, rowmap.data(), rows * 4, cudaMemcpyHostToDevice, sh.stream));
    MC_CUDA(cudaMemcpyAsync(sh.sc_target, target.data(), rows * 4, cudaMemcpyHostToDevice, sh.stream));
    MC_CUDA(cudaMemcpyAsync(sh.sc_valid, valid.data(), rows * 4, cudaMemcpyHostToDevice, sh.stream));
    if ((st = enqueue_score(sh, P, rows)) != kOk) return st;
    std::vector<double> lp(rows);
    MC_CUDA(cudaMemcpyAsync(lp.data(), sh.sc_logprob, rows * 8, cudaMemcpyDeviceToHost, sh.stream));
    MC_CUDA(cudaMemcpyAsync(sh.pos, pos.data(), sh.S * 4, cudaMemcpyHostToDevice, sh.stream));
    MC_CUDA(cudaMemcpyAsync(sh.seglen, seglen.data(), sh.S * 4, cudaMemcpyHostToDevice, sh.stream));
    if ((st = check_device_error(sh.stream)) != kOk) return st;  // synchronizes the stream
    for (int i = 0; i < sh.S; ++i)
      for (int t = 0; t < lens[s0 + i]; ++t)
        if (scored(s0 + i, t)) out[(size_t)(s0 + i) * cols + t] = lp[(size_t)i * P + t];
  }
  return kOk;
}

// The decode-loop policy of mc_generate_policy as the caller gave it.
struct PolicyIn {
  const mc_sampling* sp;
  int penalize_prompt;
  const int32_t* dfa;
  int n_states;
  const int32_t* dfa_start;
};

// Checks a policy and uploads what its launches read into one shard: the penalty prefix of each
// of the shard's sessions (the last tokens of its untrimmed prompt), the automaton and the
// sessions' start states. The automaton is checked entry by entry: the kernel follows it
// unchecked.
int upload_policy(mc_batch* b, size_t g, const PolicyIn& pi, const int32_t* prompts, const int32_t* lens, int stride) {
  DevBatch& sh = *b->shard[g];
  const int V = sh.m->V, s0 = b->first[g];
  const mc_sampling& sp = *pi.sp;
  int keep = 0;
  if (pi.penalize_prompt && sp.rep_penalty > 1.0)
    for (int i = 0; i < sh.S; ++i) {
      const int n = sp.rep_window > 0 ? std::min(sp.rep_window, lens[s0 + i]) : lens[s0 + i];
      keep = std::max(keep, n);
    }
  int st;
  if (keep > sh.pol_prefix_cap) {
    if ((st = sh.alloc(sh.pol_prefix, (size_t)sh.S * keep * 4)) != kOk) return st;
    sh.pol_prefix_cap = keep;
  }
  if (!sh.pol_prefix_len && ((st = sh.alloc(sh.pol_prefix_len, (size_t)sh.S * 4)) != kOk ||
                             (st = sh.alloc(sh.pol_state, (size_t)sh.S * 4)) != kOk))
    return st;
  std::vector<int32_t> plen(sh.S, 0);
  if (keep > 0) {
    std::vector<int32_t> pre((size_t)sh.S * sh.pol_prefix_cap, 0);
    for (int i = 0; i < sh.S; ++i) {
      const int len = lens[s0 + i], n = std::min(keep, len);
      const int32_t* src = prompts + (size_t)(s0 + i) * stride + (len - n);
      std::copy(src, src + n, pre.begin() + (size_t)i * sh.pol_prefix_cap);
      plen[i] = n;
    }
    MC_CUDA(cudaMemcpyAsync(sh.pol_prefix, pre.data(), pre.size() * 4, cudaMemcpyHostToDevice, sh.stream));
  }
  MC_CUDA(cudaMemcpyAsync(sh.pol_prefix_len, plen.data(), plen.size() * 4, cudaMemcpyHostToDevice, sh.stream));
  sh.pol = DevBatch::Policy();
  sh.pol.temperature = sp.temperature;
  sh.pol.rep_penalty = sp.rep_penalty;
  sh.pol.top_p = sp.top_p;
  sh.pol.top_k = sp.top_k;
  sh.pol.rep_window = sp.rep_window;
  sh.pol.ban_trigrams = sp.ban_trigrams ? 1 : 0;
  if (pi.dfa) {
    const size_t n = (size_t)pi.n_states * V;
    if (n > sh.pol_dfa_n) {
      if ((st = sh.alloc(sh.pol_dfa, n * 4)) != kOk) return st;
      sh.pol_dfa_n = n;
    }
    MC_CUDA(cudaMemcpyAsync(sh.pol_dfa, pi.dfa, n * 4, cudaMemcpyHostToDevice, sh.stream));
    MC_CUDA(cudaMemcpyAsync(sh.pol_state, pi.dfa_start + s0, (size_t)sh.S * 4, cudaMemcpyHostToDevice, sh.stream));
    sh.pol.dfa = sh.pol_dfa;
  }
  // pageable sources: the copies above have read them before returning
  return kOk;
}

int check_policy(const mc_sampling* sp, const PolicyIn* pi, int V, int count) {
  if (!sp) return set_error(kInvalidArgument, "sampling policy: null parameters");
  if (!std::isfinite(sp->temperature) || !std::isfinite(sp->rep_penalty) || !std::isfinite(sp->top_p))
    return set_error(kInvalidArgument, "sampling policy: non-finite parameter");
  if (V > kPolicyMaxVocab) return set_error(kUnsupported, "sampling policy: vocabulary above 16384");
  if (pi && pi->dfa) {
    if (pi->n_states < 1 || !pi->dfa_start) return set_error(kInvalidArgument, "sampling policy: automaton without states");
    const size_t n = (size_t)pi->n_states * V;
    for (size_t i = 0; i < n; ++i)
      if (pi->dfa[i] < -1 || pi->dfa[i] >= pi->n_states)
        return set_error(kInvalidArgument, "sampling policy: automaton entry outside [-1, n_states)");
    for (int s = 0; s < count; ++s)
      if (pi->dfa_start[s] >= pi->n_states) return set_error(kInvalidArgument, "sampling policy: start state out of range");
  }
  return kOk;
}

// The decode loop of mc_generate / mc_generate_stops (greedyLoop, generate/greedy.go:63-87, with
// stop tokens: a session ends before the first one it would emit; out_lens[s] = tokens emitted,
// the rest of its row -1), and with a policy that of mc_generate_policy (sampleContinuation,
// generate/sample.go:196-247).
// Per-session token limits (limits[s] tokens for session s, device or host pointer): the sessions
// generate through the per-session counters (gen_n: output column; limit: it ends after its last
// token) while the step loop runs n_new steps for all.
int begin_limits(DevBatch& sh, const int32_t* limits, cudaMemcpyKind kind) {
  int st;
  if (!sh.gen_n && (st = sh.alloc(sh.gen_n, (size_t)sh.S * 4)) != kOk) return st;
  if (!sh.limit && (st = sh.alloc(sh.limit, (size_t)sh.S * 4)) != kOk) return st;
  MC_CUDA(cudaMemcpyAsync(sh.limit, limits, (size_t)sh.S * 4, kind, sh.stream));
  MC_CUDA(cudaMemsetAsync(sh.gen_n, 0, (size_t)sh.S * 4, sh.stream));
  MC_CUDA(cudaMemsetAsync(sh.out_tok, 0xFF, (size_t)sh.S * sh.out_stride * 4, sh.stream));
  MC_CUDA(cudaMemsetAsync(sh.out_prob, 0, (size_t)sh.S * sh.out_stride * 4, sh.stream));
  sh.per_session = true;
  return kOk;
}

int generate_impl(mc_batch* b, const int32_t* prompts, const int32_t* lens, int stride, int n_new, double temperature,
                  uint32_t session0, const int32_t* stops, int n_stops, int32_t* out_tokens, float* out_probs,
                  int32_t* out_lens, const PolicyIn* pol = nullptr, const int32_t* limits = nullptr) {
  if (!b || !prompts || !lens || !out_tokens || n_new <= 0) return set_error(kInvalidArgument, "mc_generate: bad arguments");
  if (limits)
    for (int s = 0; s < b->count; ++s)
      if (limits[s] < 1 || limits[s] > n_new)
        return set_error(kInvalidArgument, "mc_generate_limits: a session's token limit is outside [1, n_max]");
  const int mode = pol ? 3 : temperature > 0.001 ? 1 : 0;
  if (mode == 1 && b->topk < 1)
    return set_error(kUnsupported, "mc_generate: sampling needs a batch opened with top_k in [1, 64]");
  const double inv_t = mode == 1 ? 1.0 / temperature : 0.0;
  int st;
  if (pol && (st = check_policy(pol->sp, pol, b->model->dev[0]->V, b->count)) != kOk) return st;
  int P = 1;
  if ((st = upload_prompts(b, prompts, lens, stride, &P)) != kOk) return st;
  for (size_t g = 0; g < b->shard.size(); ++g) {
    DevBatch& sh = *b->shard[g];
    if (sh.S == 0) continue;
    MC_CUDA(cudaSetDevice(sh.m->device));
    // the sampler (mode 1) and the policy (mode 3) select from materialised logits
    if ((st = ensure_step_outputs(sh, mode == 3 || mode == 1, n_new, mode == 1)) != kOk) return st;
    if (pol && (st = upload_policy(b, g, *pol, prompts, lens, stride)) != kOk) return st;
    MC_CUDA(cudaMemsetAsync(sh.step, 0, 4, sh.stream));
    sh.n_stops = n_stops;
    for (int k = 0; k < n_stops; ++k) sh.stops[k] = stops[k];
    if (n_stops > 0 || mode == 3) {  // sessions that end early leave their remaining columns at -1 / 0
      MC_CUDA(cudaMemsetAsync(sh.out_tok, 0xFF, (size_t)sh.S * sh.out_stride * 4, sh.stream));
      MC_CUDA(cudaMemsetAsync(sh.out_prob, 0, (size_t)sh.S * sh.out_stride * 4, sh.stream));
    }
    if (limits && (st = begin_limits(sh, limits + b->first[g], cudaMemcpyHostToDevice)) != kOk) return st;
    const uint32_t s0 = session0 + (uint32_t)b->first[g];
    if (tiny_job_ok(sh, mode, n_stops, limits != nullptr, pol != nullptr)) {
      st = launch_tiny_job(sh, P, n_new);  // the whole job in one launch
    } else {
      st = enqueue_forward(sh, P, mode, inv_t, s0, false, true);
      if (st == kOk) st = run_decode_steps(sh, n_new, mode, inv_t, s0);
    }
    sh.n_stops = 0;  // only this job's launches carry the stop tokens, the policy and the limits
    sh.pol = DevBatch::Policy();
    sh.per_session = false;
    if (st != kOk) return st;
  }
  for (size_t g = 0; g < b->shard.size(); ++g) {
    DevBatch& sh = *b->shard[g];
    if (sh.S == 0) continue;
    MC_CUDA(cudaSetDevice(sh.m->device));
    // out columns are laid out with stride sh.out_stride >= n_new: the first n_new of each
    // session's row go straight to the caller's rows of this shard's sessions
    const size_t row0 = (size_t)b->first[g] * n_new;
    MC_CUDA(cudaMemcpy2DAsync(out_tokens + row0, (size_t)n_new * 4, sh.out_tok, (size_t)sh.out_stride * 4,
                              (size_t)n_new * 4, sh.S, cudaMemcpyDeviceToHost, sh.stream));
    if (out_probs)
      MC_CUDA(cudaMemcpy2DAsync(out_probs + row0, (size_t)n_new * 4, sh.out_prob, (size_t)sh.out_stride * 4,
                                (size_t)n_new * 4, sh.S, cudaMemcpyDeviceToHost, sh.stream));
  }
  for (size_t g = 0; g < b->shard.size(); ++g) {
    DevBatch& sh = *b->shard[g];
    if (sh.S == 0) continue;
    MC_CUDA(cudaSetDevice(sh.m->device));
    if ((st = check_device_error(sh.stream)) != kOk) return st;
  }
  if (out_lens)
    for (int s = 0; s < b->count; ++s) {
      int n = 0;
      while (n < n_new && out_tokens[(size_t)s * n_new + n] >= 0) ++n;
      out_lens[s] = n;
    }
  return kOk;
}


// mc_generate_dev / mc_generate_limits_dev: the whole job enqueued on the batch's stream from
// device-resident prompts (and per-session limits when d_limits is non-null).
int generate_dev_impl(mc_batch* b, const int32_t* d_prompts, const int32_t* d_lens, int stride, int pmax,
                      const int32_t* d_limits, int n_new, double temperature, uint32_t session0, int32_t* d_out_tokens,
                      float* d_out_probs, const char* name) {
  const std::string fn(name);
  if (!b || !d_prompts || !d_lens || !d_out_tokens || n_new <= 0 || pmax <= 0)
    return set_error(kInvalidArgument, fn + ": bad arguments");
  if (b->shard.size() != 1) return set_error(kUnsupported, fn + ": single-device batches only");
  DevBatch& sh = *b->shard[0];
  const int P = std::min(pmax, b->window);
  if (P > b->pmax) return set_error(kInvalidArgument, fn + ": pmax above the batch's max_prompt");
  const int mode = temperature > 0.001 ? 1 : 0;
  if (mode == 1 && b->topk < 1) return set_error(kUnsupported, fn + ": sampling needs top_k >= 1");
  const double inv_t = mode ? 1.0 / temperature : 0.0;
  MC_CUDA(cudaSetDevice(sh.m->device));
  int st;
  if ((st = ensure_step_outputs(sh, mode == 1, n_new, mode == 1)) != kOk) return st;  // the sampler selects from logits
  prepare_prompts_kernel<<<(sh.S + 127) / 128, 128, 0, sh.stream>>>(d_prompts, d_lens, stride, sh.S, P, b->window, sh.tok,
                                                                      sh.seglen, sh.pos, sh.rowmap, sh.step, sh.next_tok);
  MC_CUDA(cudaGetLastError());
  if (d_limits && (st = begin_limits(sh, d_limits, cudaMemcpyDeviceToDevice)) != kOk) return st;
  if (tiny_job_ok(sh, mode, 0, d_limits != nullptr, false)) {
    st = launch_tiny_job(sh, P, n_new);  // the whole job in one launch
  } else {
    st = enqueue_forward(sh, P, mode, inv_t, session0, false, true);
    if (st == kOk) st = run_decode_steps(sh, n_new, mode, inv_t, session0);
  }
  sh.per_session = false;
  if (st != kOk) return st;
  MC_CUDA(cudaMemcpy2DAsync(d_out_tokens, (size_t)n_new * 4, sh.out_tok, (size_t)sh.out_stride * 4, (size_t)n_new * 4, sh.S,
                            cudaMemcpyDeviceToDevice, sh.stream));
  if (d_out_probs)
    MC_CUDA(cudaMemcpy2DAsync(d_out_probs, (size_t)n_new * 4, sh.out_prob, (size_t)sh.out_stride * 4, (size_t)n_new * 4,
                              sh.S, cudaMemcpyDeviceToDevice, sh.stream));
  return kOk;
}

// mc_batch_open; allow_passes: prefills larger than the scratch budget run in passes over
// contiguous sessions (a scheduler's admission passes over tile lists need every row instead).
int batch_open(mc_model* m, int count, int context_size, int max_prompt, int top_k, bool allow_passes, mc_batch** out) {
  if (!m || !out || count <= 0) return set_error(kInvalidArgument, "mc_batch_open: bad arguments");
  if (top_k < 0 || top_k > kMaxTopK) return set_error(kInvalidArgument, "mc_batch_open: top_k must be in [0, 64]");
  auto b = std::make_unique<mc_batch>();
  b->model = m;
  b->count = count;
  const DevModel& d0 = *m->dev[0];
  b->window = d0.max_context;  // NewSession (session.go:20-28)
  if (context_size > 0 && context_size < b->window) b->window = context_size;
  b->pmax = std::min(std::max(1, max_prompt > 0 ? std::min(max_prompt, b->window) : b->window), 128);
  b->topk = top_k;
  const int ndev = (int)m->dev.size();
  shard_sizes(count, ndev, b->first);
  for (int g = 0; g < ndev; ++g) {
    std::unique_ptr<DevBatch> sh;
    const int S = b->first[g + 1] - b->first[g];
    if (S == 0) {
      b->shard.push_back(std::make_unique<DevBatch>());
      b->shard.back()->m = m->dev[g].get();
      continue;
    }
    int st = batch_create(m->dev[g].get(), S, b->window, b->pmax, top_k, allow_passes, sh);
    if (st != kOk) return st;
    if ((st = ensure_step_outputs(*sh, false, 1)) != kOk) return st;
    b->shard.push_back(std::move(sh));
  }
  *out = b.release();
  return kOk;
}

}  // namespace

extern "C" {

const char* mc_last_error(void) { return last_error_cstr(); }

int mc_version(void) { return 100; }

int mc_open(const mc_options* opt, mc_ctx** out) {
  clear_error();
  DeviceRestore restore_device;
  if (!out) return set_error(kInvalidArgument, "mc_open: null output");
  auto c = std::make_unique<mc_ctx>();
  int ndev = 0;
  MC_CUDA(cudaGetDeviceCount(&ndev));
  if (opt && opt->n_devices > 0) {
    if (!opt->devices) return set_error(kInvalidArgument, "mc_open: n_devices without a device list");
    for (int i = 0; i < opt->n_devices; ++i) {
      if (opt->devices[i] < 0 || opt->devices[i] >= ndev) return set_error(kInvalidArgument, "mc_open: no such device");
      c->devices.push_back(opt->devices[i]);
    }
  } else {
    if (ndev < 1) return set_error(kCudaError, "mc_open: no CUDA device");
    c->devices.push_back(0);
  }
  *out = c.release();
  return kOk;
}

int mc_close(mc_ctx* ctx) {
  delete ctx;
  return kOk;
}

int mc_load_model(mc_ctx* ctx, const uint8_t* data, size_t n, mc_model** out) {
  clear_error();
  DeviceRestore restore_device;
  if (!ctx || !data || !out) return set_error(kInvalidArgument, "mc_load_model: null argument");
  auto m = std::make_unique<mc_model>();
  m->ctx = ctx;
  int st = parse_model_file(data, n, m->host);
  if (st != kOk) return st;
  for (int d : ctx->devices) {
    std::unique_ptr<DevModel> dm;
    if ((st = build_dev_model(m->host, d, dm)) != kOk) return st;
    m->dev.push_back(std::move(dm));
  }
  *out = m.release();
  return kOk;
}

int mc_model_free(mc_model* m) {
  DeviceRestore restore_device;  // the destructors switch to the shards' devices
  delete m;
  return kOk;
}

int mc_model_info(const mc_model* m, int32_t* out) {
  clear_error();
  DeviceRestore restore_device;
  if (!m || !out) return set_error(kInvalidArgument, "mc_model_info: null argument");
  const DevModel& d = *m->dev[0];
  out[0] = d.V;
  out[1] = d.D;
  out[2] = d.H;
  out[3] = (int32_t)d.blocks.size();
  out[4] = d.max_context;
  out[5] = d.heads;
  out[6] = d.window;
  out[7] = d.total_steps;
  out[8] = d.ring;
  out[9] = d.cache;
  return kOk;
}

int mc_batch_open(mc_model* m, int count, int context_size, int max_prompt, int top_k, mc_batch** out) {
  clear_error();
  DeviceRestore restore_device;
  return batch_open(m, count, context_size, max_prompt, top_k, true, out);
}

int mc_batch_close(mc_batch* b) {
  DeviceRestore restore_device;  // the destructors switch to the shards' devices
  delete b;
  return kOk;
}
int mc_prefill(mc_batch* b, const int32_t* tokens, const int32_t* lens, int stride, float* logits, int32_t* next,
               float* prob) {
  clear_error();
  DeviceRestore restore_device;
  if (!b || !tokens || !lens) return set_error(kInvalidArgument, "mc_prefill: null argument");
  int P = 1;
  int st = upload_prompts(b, tokens, lens, stride, &P);
  if (st != kOk) return st;
  for (auto& sh : b->shard) {
    if (sh->S == 0) continue;
    MC_CUDA(cudaSetDevice(sh->m->device));
    if ((st = ensure_step_outputs(*sh, logits != nullptr, 1)) != kOk) return st;
    MC_CUDA(cudaMemsetAsync(sh->step, 0, 4, sh->stream));
    // MC_TRACE=1: phase timestamps of CTA 0 of every block-kernel launch, printed to stderr.
    const bool trace = getenv("MC_TRACE") != nullptr;
    const int nb = (int)sh->m->blocks.size() + 1;
    if (trace) {
      MC_CUDA(cudaMalloc(&sh->trace, (size_t)64 * nb * 8));
      MC_CUDA(cudaMemsetAsync(sh->trace, 0, (size_t)64 * nb * 8, sh->stream));
    }
    if ((st = enqueue_forward(*sh, P, 0, 0.0, 0, logits != nullptr, true)) != kOk) return st;
    if (trace) {
      std::vector<unsigned long long> tr((size_t)64 * nb);
      MC_CUDA(cudaStreamSynchronize(sh->stream));
      MC_CUDA(cudaMemcpy(tr.data(), sh->trace, tr.size() * 8, cudaMemcpyDeviceToHost));
      cudaFree(sh->trace);
      sh->trace = nullptr;
      for (int b2 = 0; b2 < nb; ++b2) {
        fprintf(stderr, "prefill block launch %d phase ns:", b2);
        for (int i = 1; i < 64 && tr[(size_t)64 * b2 + i]; ++i)
          fprintf(stderr, " %llu", tr[(size_t)64 * b2 + i] - tr[(size_t)64 * b2 + i - 1]);
        fprintf(stderr, "\n");
      }
    }
  }
  return copy_step_outputs(b, logits, next, prob);
}

int mc_score(mc_batch* b, const int32_t* seqs, const int32_t* lens, int stride, double* out) {
  clear_error();
  DeviceRestore restore_device;
  if (!b || !seqs || !lens || !out) return set_error(kInvalidArgument, "mc_score: null argument");
  return score_impl(b, seqs, lens, stride, nullptr, out, "mc_score");
}

int mc_score_targets(mc_batch* b, const int32_t* seqs, const int32_t* lens, int stride, const int32_t* targets,
                     double* out) {
  clear_error();
  DeviceRestore restore_device;
  if (!b || !seqs || !lens || !targets || !out) return set_error(kInvalidArgument, "mc_score_targets: null argument");
  return score_impl(b, seqs, lens, stride, targets, out, "mc_score_targets");
}

// One append per session is the Go provider's Session.Append for a batch of one, so its fixed cost
// per call matters as much as the step: the tokens go up and the outputs come back through the
// shard's pinned staging, and one stream synchronization per shard ends the call.
int mc_append(mc_batch* b, const int32_t* tokens, float* logits, int32_t* next, float* prob) {
  clear_error();
  DeviceRestore restore_device;
  if (!b || !tokens) return set_error(kInvalidArgument, "mc_append: null argument");
  int st;
  for (size_t g = 0; g < b->shard.size(); ++g) {
    DevBatch& sh = *b->shard[g];
    if (sh.S == 0) continue;
    MC_CUDA(cudaSetDevice(sh.m->device));
    if ((st = ensure_step_outputs(sh, logits != nullptr, 1)) != kOk) return st;
    if ((st = ensure_h_step(sh, logits != nullptr)) != kOk) return st;
    memcpy(sh.h_step, tokens + b->first[g], (size_t)sh.S * 4);  // the tokens up through the pinned staging
    MC_CUDA(cudaMemcpyAsync(sh.next_tok, sh.h_step, (size_t)sh.S * 4, cudaMemcpyHostToDevice, sh.stream));
    MC_CUDA(cudaMemsetAsync(sh.step, 0, 4, sh.stream));
    if (tiny_job_ok(sh, 0, 0, false, false))  // small models without attention: one launch
      st = launch_tiny_job(sh, 1, 1, true, logits ? sh.logits : nullptr);
    else
      st = run_graph_step(sh, 0, 0.0, 0, logits != nullptr);
    if (st != kOk) return st;
  }
  return copy_step_outputs(b, logits, next, prob);
}

int mc_generate(mc_batch* b, const int32_t* prompts, const int32_t* lens, int stride, int n_new, double temperature,
                uint32_t session0, int32_t* out_tokens, float* out_probs) {
  clear_error();
  DeviceRestore restore_device;
  return generate_impl(b, prompts, lens, stride, n_new, temperature, session0, nullptr, 0, out_tokens, out_probs, nullptr);
}

int mc_generate_stops(mc_batch* b, const int32_t* prompts, const int32_t* lens, int stride, int n_new,
                      double temperature, uint32_t session0, const int32_t* stops, int n_stops, int32_t* out_tokens,
                      float* out_probs, int32_t* out_lens) {
  clear_error();
  DeviceRestore restore_device;
  if (n_stops < 0 || n_stops > kMaxStops || (n_stops > 0 && !stops))
    return set_error(kInvalidArgument, "mc_generate_stops: 0 to 8 stop tokens");
  return generate_impl(b, prompts, lens, stride, n_new, temperature, session0, stops, n_stops, out_tokens, out_probs,
                       out_lens);
}

int mc_generate_policy(mc_batch* b, const int32_t* prompts, const int32_t* lens, int stride, int n_new,
                       const mc_sampling* sp, int penalize_prompt, const int32_t* dfa, int n_states,
                       const int32_t* dfa_start, uint32_t session0, const int32_t* stops, int n_stops,
                       int32_t* out_tokens, float* out_probs, int32_t* out_lens) {
  clear_error();
  DeviceRestore restore_device;
  if (n_stops < 0 || n_stops > kMaxStops || (n_stops > 0 && !stops))
    return set_error(kInvalidArgument, "mc_generate_policy: 0 to 8 stop tokens");
  if (!sp) return set_error(kInvalidArgument, "mc_generate_policy: null sampling parameters");
  const PolicyIn pi{sp, penalize_prompt, dfa, n_states, dfa_start};
  return generate_impl(b, prompts, lens, stride, n_new, 0.0, session0, stops, n_stops, out_tokens, out_probs, out_lens,
                       &pi);
}

int mc_sample_rows(int device, const float* logits, int n, int vocab, const int32_t* recent, const int32_t* recent_lens,
                   int recent_stride, const int32_t* allowed, const mc_sampling* sp, const double* u, uint32_t session0,
                   uint32_t step, int32_t* out_tokens, float* out_probs) {
  clear_error();
  DeviceRestore restore_device;
  if (n < 0 || vocab < 1 || !logits || !out_tokens || (recent && (!recent_lens || recent_stride < 0)))
    return set_error(kInvalidArgument, "mc_sample_rows: bad arguments");
  int st = check_policy(sp, nullptr, vocab, n);
  if (st != kOk) return st;
  if (recent)
    for (int r = 0; r < n; ++r)
      if (recent_lens[r] < 0 || recent_lens[r] > recent_stride)
        return set_error(kInvalidArgument, "mc_sample_rows: recent length outside [0, recent_stride]");
  if (n == 0) return kOk;
  MC_CUDA(cudaSetDevice(device));
  if ((st = ensure_attrs(device)) != kOk) return st;
  // one allocation: logits | allowed | recent | recent lengths | states | draws | tokens | probs
  const size_t nl = (size_t)n * vocab, nr = recent ? (size_t)n * std::max(recent_stride, 1) : 0;
  const size_t bytes = nl * 4 + (allowed ? nl * 4 : 0) + nr * 4 + (size_t)n * (4 + 4 + 8 + 4 + 4) + 64;
  DevBuf buf;
  if (cudaMalloc(&buf.p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return set_error(kOutOfMemory, "mc_sample_rows: cudaMalloc failed");
  }
  char* q = static_cast<char*>(buf.p);
  auto take = [&](size_t nb) {
    char* r = q;
    q += (nb + 15) & ~(size_t)15;
    return r;
  };
  float* d_logits = reinterpret_cast<float*>(take(nl * 4));
  int32_t* d_allowed = allowed ? reinterpret_cast<int32_t*>(take(nl * 4)) : nullptr;
  int32_t* d_recent = recent ? reinterpret_cast<int32_t*>(take(nr * 4)) : nullptr;
  int32_t* d_rlen = reinterpret_cast<int32_t*>(take((size_t)n * 4));
  int32_t* d_state = reinterpret_cast<int32_t*>(take((size_t)n * 4));
  double* d_u = reinterpret_cast<double*>(take((size_t)n * 8));
  int32_t* d_tok = reinterpret_cast<int32_t*>(take((size_t)n * 4));
  float* d_prob = reinterpret_cast<float*>(take((size_t)n * 4));
  cudaStream_t s = 0;
  MC_CUDA(cudaMemcpyAsync(d_logits, logits, nl * 4, cudaMemcpyHostToDevice, s));
  if (allowed) {
    // row r's mask is state r of a one-step automaton
    std::vector<int32_t> iota(n);
    for (int r = 0; r < n; ++r) iota[r] = r;
    MC_CUDA(cudaMemcpyAsync(d_allowed, allowed, nl * 4, cudaMemcpyHostToDevice, s));
    MC_CUDA(cudaMemcpyAsync(d_state, iota.data(), (size_t)n * 4, cudaMemcpyHostToDevice, s));
  }
  if (recent) {
    MC_CUDA(cudaMemcpyAsync(d_recent, recent, nr * 4, cudaMemcpyHostToDevice, s));
    MC_CUDA(cudaMemcpyAsync(d_rlen, recent_lens, (size_t)n * 4, cudaMemcpyHostToDevice, s));
  }
  if (u) MC_CUDA(cudaMemcpyAsync(d_u, u, (size_t)n * 8, cudaMemcpyHostToDevice, s));
  PolicyArgs pa;
  memset(&pa, 0, sizeof(pa));
  pa.n_rows = n;
  pa.V = vocab;
  pa.logits = d_logits;
  pa.temperature = sp->temperature;
  pa.rep_penalty = sp->rep_penalty;
  pa.top_p = sp->top_p;
  pa.top_k = sp->top_k;
  pa.rep_window = sp->rep_window;
  pa.ban_trigrams = sp->ban_trigrams ? 1 : 0;
  pa.gen = d_recent;
  pa.gen_len = d_rlen;
  pa.gen_stride = recent ? std::max(recent_stride, 1) : 0;
  pa.dfa = d_allowed;
  pa.dfa_state = allowed ? d_state : nullptr;
  pa.u = u ? d_u : nullptr;
  pa.session0 = session0;
  pa.step0 = step;
  pa.out_stride = 1;
  pa.out_tok = d_tok;
  pa.out_prob = d_prob;
  if ((st = launch_policy(pa, s)) != kOk) return st;
  MC_CUDA(cudaMemcpyAsync(out_tokens, d_tok, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
  if (out_probs) MC_CUDA(cudaMemcpyAsync(out_probs, d_prob, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
  return check_device_error(s);
}

int mc_batch_stream(mc_batch* b, int shard, void** stream) {
  clear_error();
  DeviceRestore restore_device;
  if (!b || !stream || shard < 0 || shard >= (int)b->shard.size()) return set_error(kInvalidArgument, "mc_batch_stream: bad arguments");
  *stream = (void*)b->shard[shard]->stream;
  return kOk;
}

int mc_generate_dev(mc_batch* b, const int32_t* d_prompts, const int32_t* d_lens, int stride, int pmax, int n_new,
                    double temperature, uint32_t session0, int32_t* d_out_tokens, float* d_out_probs) {
  clear_error();
  DeviceRestore restore_device;
  return generate_dev_impl(b, d_prompts, d_lens, stride, pmax, nullptr, n_new, temperature, session0, d_out_tokens,
                           d_out_probs, "mc_generate_dev");
}

int mc_generate_limits(mc_batch* b, const int32_t* prompts, const int32_t* lens, int stride, const int32_t* max_tokens,
                       int n_max, double temperature, uint32_t session0, int32_t* out_tokens, float* out_probs,
                       int32_t* out_lens) {
  clear_error();
  DeviceRestore restore_device;
  if (!max_tokens) return set_error(kInvalidArgument, "mc_generate_limits: null max_tokens");
  return generate_impl(b, prompts, lens, stride, n_max, temperature, session0, nullptr, 0, out_tokens, out_probs,
                       out_lens, nullptr, max_tokens);
}

int mc_generate_limits_dev(mc_batch* b, const int32_t* d_prompts, const int32_t* d_lens, int stride, int pmax,
                           const int32_t* d_max_tokens, int n_max, double temperature, uint32_t session0,
                           int32_t* d_out_tokens, float* d_out_probs) {
  clear_error();
  DeviceRestore restore_device;
  if (!d_max_tokens) return set_error(kInvalidArgument, "mc_generate_limits_dev: null max_tokens");
  return generate_dev_impl(b, d_prompts, d_lens, stride, pmax, d_max_tokens, n_max, temperature, session0,
                           d_out_tokens, d_out_probs, "mc_generate_limits_dev");
}

int mc_batch_error(mc_batch* b) {
  clear_error();
  DeviceRestore restore_device;
  if (!b) return set_error(kInvalidArgument, "mc_batch_error: null batch");
  return sync_all(b);
}

int mc_profile_step(mc_batch* b, int max_launches, float* ms, int32_t* kinds, int* n_launches) {
  clear_error();
  DeviceRestore restore_device;
  if (!b || !ms || !kinds || !n_launches || b->shard.size() != 1)
    return set_error(kInvalidArgument, "mc_profile_step: bad arguments (single-device batches only)");
  DevBatch& sh = *b->shard[0];
  MC_CUDA(cudaSetDevice(sh.m->device));
  int st;
  if ((st = ensure_step_outputs(sh, false, 1)) != kOk) return st;
  MC_CUDA(cudaMemsetAsync(sh.step, 0, 4, sh.stream));
  LaunchLog log;
  // MC_TRACE=1: phase timestamps of CTA 0 of every block-kernel launch, printed to stderr.
  const bool trace = getenv("MC_TRACE") != nullptr;
  const int nb = (int)sh.m->blocks.size() + 1;
  if (trace) {
    MC_CUDA(cudaMalloc(&sh.trace, (size_t)64 * nb * 8));
    MC_CUDA(cudaMemsetAsync(sh.trace, 0, (size_t)64 * nb * 8, sh.stream));
  }
  if ((st = log.record(sh.stream, -1)) != kOk) return st;
  if ((st = enqueue_forward(sh, 1, 0, 0.0, 0, false, false, &log)) != kOk) return st;
  MC_CUDA(cudaStreamSynchronize(sh.stream));
  if (trace) {
    std::vector<unsigned long long> tr((size_t)64 * nb);
    MC_CUDA(cudaMemcpy(tr.data(), sh.trace, tr.size() * 8, cudaMemcpyDeviceToHost));
    cudaFree(sh.trace);
    sh.trace = nullptr;
    for (int b2 = 0; b2 < nb; ++b2) {
      fprintf(stderr, "block launch %d phase ns:", b2);
      for (int i = 1; i < 64 && tr[(size_t)64 * b2 + i]; ++i)
        fprintf(stderr, " %llu", tr[(size_t)64 * b2 + i] - tr[(size_t)64 * b2 + i - 1]);
      fprintf(stderr, "\n");
    }
  }
  if ((st = check_device_error(sh.stream)) != kOk) return st;
  const int n = std::min((int)log.ev.size() - 1, max_launches);
  for (int i = 0; i < n; ++i) {
    MC_CUDA(cudaEventElapsedTime(&ms[i], log.ev[i], log.ev[i + 1]));
    kinds[i] = log.kind[i + 1];
  }
  *n_launches = n;
  return kOk;
}

int mc_gemm_i8_dev(const int8_t* a, const int8_t* w, int m, int n, int k, const float* row_scale,
                   const float* col_scale, const float* bias, int32_t* c_i32, float* y, void* stream) {
  clear_error();
  DeviceRestore restore_device;
  if (!a || !w) return set_error(kInvalidArgument, "mc_gemm_i8_dev: null operand");
  return gemm_i8_launch(a, w, m, n, k, row_scale, col_scale, bias, c_i32, y, (cudaStream_t)stream);
}

int mc_gemm_f32a_dev(const float* x, const int8_t* w, int m, int n, int k, float w_scale, const float* bias,
                     float* y, int32_t* slices, float* row_max_scratch, void* stream) {
  clear_error();
  DeviceRestore restore_device;
  if (!x || !w || !y || !row_max_scratch) return set_error(kInvalidArgument, "mc_gemm_f32a_dev: null pointer");
  return gemm_f32a_launch(x, w, m, n, k, w_scale, bias, y, slices, row_max_scratch, (cudaStream_t)stream);
}

int mc_gemm_f32a_noalloc_dev(const float* x, const int8_t* w, int m, int n, int k, float w_scale, const float* bias,
                             float* y, void* stream) {
  clear_error();
  DeviceRestore restore_device;
  if (!x || !w || !y) return set_error(kInvalidArgument, "mc_gemm_f32a_noalloc_dev: null pointer");
  return gemm_f32a_noalloc_launch(x, w, m, n, k, w_scale, bias, y, (cudaStream_t)stream);
}

int mc_gemm_i8(int device, const int8_t* a, const int8_t* w, int m, int n, int k, const float* row_scale,
               const float* col_scale, const float* bias, int32_t* c_i32, float* y) {
  clear_error();
  DeviceRestore restore_device;
  if (!a || !w || m <= 0 || n <= 0 || k <= 0) return set_error(kInvalidArgument, "mc_gemm_i8: bad arguments");
  MC_CUDA(cudaSetDevice(device));
  DevBuf da, dw, drs, dcs, db, dc, dy;
  const size_t mk = (size_t)m * k, nk = (size_t)n * k, mn = (size_t)m * n;
  MC_CUDA(cudaMalloc(&da.p, mk));
  MC_CUDA(cudaMalloc(&dw.p, nk));
  MC_CUDA(cudaMemcpy(da.p, a, mk, cudaMemcpyHostToDevice));
  MC_CUDA(cudaMemcpy(dw.p, w, nk, cudaMemcpyHostToDevice));
  if (row_scale) {
    MC_CUDA(cudaMalloc(&drs.p, 4 * (size_t)m));
    MC_CUDA(cudaMemcpy(drs.p, row_scale, 4 * (size_t)m, cudaMemcpyHostToDevice));
  }
  if (col_scale) {
    MC_CUDA(cudaMalloc(&dcs.p, 4 * (size_t)n));
    MC_CUDA(cudaMemcpy(dcs.p, col_scale, 4 * (size_t)n, cudaMemcpyHostToDevice));
  }
  if (bias) {
    MC_CUDA(cudaMalloc(&db.p, 4 * (size_t)n));
    MC_CUDA(cudaMemcpy(db.p, bias, 4 * (size_t)n, cudaMemcpyHostToDevice));
  }
  if (c_i32) MC_CUDA(cudaMalloc(&dc.p, 4 * mn));
  if (y) MC_CUDA(cudaMalloc(&dy.p, 4 * mn));
  int st = gemm_i8_launch((const int8_t*)da.p, (const int8_t*)dw.p, m, n, k, (const float*)drs.p,
                          (const float*)dcs.p, (const float*)db.p, (int32_t*)dc.p, (float*)dy.p, 0);
  if (st != kOk) return st;
  st = check_device_error(0);
  if (st != kOk) return st;
  if (c_i32) MC_CUDA(cudaMemcpy(c_i32, dc.p, 4 * mn, cudaMemcpyDeviceToHost));
  if (y) MC_CUDA(cudaMemcpy(y, dy.p, 4 * mn, cudaMemcpyDeviceToHost));
  return kOk;
}

}  // extern "C"
