// Continuous batching over a fixed pool of session slots (mc_sched_*, include/mignon_cuda.h).
//
// Requests wait in a host queue. Whenever enough slots are free (or none is running), the queued
// requests are admitted into the free slots by one prefill pass in which the running slots sit
// out (seglen 0: the kernels leave their state alone); the running slots resume afterwards. All
// running slots then decode together, each slot writing its own output row: its tokens so far
// (gen_n) are its output column, its draw counter and its 3-gram history, and it ends at its own
// token limit or at a stop token. The host harvests finished slots every few steps. Every token
// is chosen by the decode-loop policy of sampleContinuation (generate/sample.go:196-247) with
// draws keyed by the request, so a request's tokens do not depend on which slot it ran in or
// what ran beside it; plain argmax (no penalty, no 3-gram block) runs on the greedy head fused
// into the final decode launch, as mc_generate does.
#include <algorithm>
#include <chrono>
#include <deque>

namespace mc {
namespace eng {

// Slots with adm[s] > 0 restart from a prompt of adm[s] tokens at position 0 with no tokens
// generated; every other slot sits the admission pass out.
__global__ void sched_admit_kernel(int S, int P, const int32_t* adm, const int32_t* tok, int32_t* seglen, int32_t* pos,
                                   int32_t* gen_n, int32_t* next_tok) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= S) return;
  const int n = adm[s];
  if (n > 0) {
    seglen[s] = n;
    pos[s] = 0;
    gen_n[s] = 0;
    if (P == 1) next_tok[s] = tok[s];  // a one-row pass runs through the decode kernels
  } else {
    seglen[s] = 0;
  }
}

// After the admission pass the slots that were decoding (adm[s] < 0) resume.
__global__ void sched_resume_kernel(int S, const int32_t* adm, int32_t* seglen) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s < S && adm[s] < 0) seglen[s] = 1;
}

}  // namespace eng
}  // namespace mc

namespace {

struct SchedReq {
  std::vector<int32_t> prompt;
  int n_new = 0;
  uint32_t key = 0;
  int state = 0;  // 0 queued, 1 running, 2 finished
  std::vector<int32_t> tokens;
  std::vector<float> probs;
};

struct SchedShard {
  std::vector<int64_t> slot_req;  // request in each slot, -1: free
  std::vector<int32_t> limit;     // host copies of the per-slot device arrays
  std::vector<uint32_t> key;
  std::vector<int32_t> prefix, prefix_len;
  int busy = 0;
  // pinned host buffers: the admission list's uploads [tok S*P | rowmap | adm | limit | key |
  // prefix S*cap | prefix_len | pass tiles | pass sessions], and the collection's reads
  // [seglen | gen_n] and output rows
  cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};  // round start, admission done, decode steps done
  bool timed = false;                                // this round recorded them
  int32_t* h_up = nullptr;
  int32_t* h_state = nullptr;
  int32_t* h_tok = nullptr;
  float* h_prob = nullptr;
};

}  // namespace

struct mc_sched {
  mc_batch* batch = nullptr;
  mc_sampling sp{};
  int penalize_prompt = 0, max_new = 0, admit_min = 1;
  int mode = 3;  // 0: plain greedy (argmax, no penalty, no 3-gram block) on the fused greedy head
  int n_stops = 0;
  int32_t stops[kMaxStops] = {0};
  std::deque<int64_t> queue;
  std::vector<SchedReq> req;
  std::vector<SchedShard> sh;
  int64_t n_prefill = 0, n_steps = 0, n_tokens = 0, n_done = 0, n_admitted = 0;
  double admit_us = 0, decode_us = 0, host_us = 0;  // device time of admission passes and decode steps;
                                                    // wall time inside mc_sched_step
  double admit_host_us = 0;                         // host time choosing and staging admissions
  ~mc_sched() {
    for (SchedShard& ss : sh) {
      for (void* p : {(void*)ss.h_up, (void*)ss.h_state, (void*)ss.h_tok, (void*)ss.h_prob})
        if (p) cudaFreeHost(p);
      for (cudaEvent_t e : ss.ev)
        if (e) cudaEventDestroy(e);
    }
    delete batch;
  }
};

namespace {

// Admits queued requests into the free slots of shard g with one prefill pass.
int sched_admit(mc_sched* q, size_t g) {
  const auto t_host = std::chrono::steady_clock::now();
  SchedShard& ss = q->sh[g];
  DevBatch& sh = *q->batch->shard[g];
  const int S = sh.S, window = q->batch->window, cap = sh.pol_prefix_cap;
  std::vector<int32_t> adm(S, 0);
  std::vector<int> free_slots;
  for (int s = 0; s < S; ++s) {
    if (ss.slot_req[s] >= 0) adm[s] = -1;
    else free_slots.push_back(s);
  }
  // the requests this pass admits, in queue order (an empty prompt finishes at once: Prefill of
  // nothing returns no logits, so nothing is generated)
  std::vector<int64_t> take;
  while (!q->queue.empty() && take.size() < free_slots.size()) {
    const int64_t c = q->queue.front();
    q->queue.pop_front();
    if (q->req[c].prompt.empty()) {
      q->req[c].state = 2;
      ++q->n_done;
      continue;
    }
    take.push_back(c);
  }
  // Requests with similar token limits go to neighbouring slots: they tend to finish together, so
  // later passes find whole prefill tiles free instead of one slot in each. A request's tokens do
  // not depend on its slot.
  std::stable_sort(take.begin(), take.end(),
                   [&](int64_t x, int64_t y) { return q->req[x].n_new < q->req[y].n_new; });
  int P = 0, n_adm = 0;
  for (size_t i = 0; i < take.size(); ++i) {
    const int s = free_slots[i];
    const int64_t id = take[i];
    SchedReq& r = q->req[id];
    const int n = std::min((int)r.prompt.size(), window);
    r.state = 1;
    ss.slot_req[s] = id;
    adm[s] = n;
    P = std::max(P, n);
    ++n_adm;
    ss.limit[s] = r.n_new;
    ss.key[s] = r.key;
    const int k = std::min(cap, (int)r.prompt.size());
    std::copy(r.prompt.end() - k, r.prompt.end(), ss.prefix.begin() + (size_t)s * cap);
    ss.prefix_len[s] = k;
  }
  if (n_adm == 0) return kOk;
  // staging (the previous admission's copies finished: every round ends with a synchronizing read)
  int32_t* tok = ss.h_up;
  int32_t* rowmap = tok + (size_t)S * P;
  int32_t* hadm = rowmap + S;
  int32_t* hlim = hadm + S;
  int32_t* hkey = hlim + S;
  int32_t* hpre = hkey + S;
  int32_t* hplen = hpre + (size_t)S * cap;
  int32_t* htiles = hplen + S;  // the pass's tiles and sessions: the kernels run only these
  int32_t* hsess = htiles + S;
  std::fill(tok, tok + (size_t)S * P, 0);
  const int spt = std::max(1, 128 / P);
  for (int s = 0; s < S; ++s) {
    const int n = std::max(adm[s], 0);
    if (n > 0) {
      const std::vector<int32_t>& pr = q->req[ss.slot_req[s]].prompt;
      std::copy(pr.end() - n, pr.end(), tok + (size_t)s * P);
    }
    rowmap[s] = (s / spt) * 128 + (s % spt) * P + std::max(n - 1, 0);
  }
  std::copy(adm.begin(), adm.end(), hadm);
  std::copy(ss.limit.begin(), ss.limit.end(), hlim);
  for (int s = 0; s < S; ++s) hkey[s] = (int32_t)ss.key[s];
  std::copy(ss.prefix.begin(), ss.prefix.end(), hpre);
  std::copy(ss.prefix_len.begin(), ss.prefix_len.end(), hplen);
  int n_tiles = 0, n_sess = 0;
  for (int s = 0; s < S; ++s) {
    if (adm[s] <= 0) continue;
    hsess[n_sess++] = s;
    const int t = s / spt;
    if (n_tiles == 0 || htiles[n_tiles - 1] != t) htiles[n_tiles++] = t;
  }
  cudaStream_t st = sh.stream;
  // the admission's device time starts here, after the host's part
  MC_CUDA(cudaEventRecord(ss.ev[0], st));
  q->admit_host_us += std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t_host).count();
  MC_CUDA(cudaMemcpyAsync(sh.tok, tok, (size_t)S * P * 4, cudaMemcpyHostToDevice, st));
  MC_CUDA(cudaMemcpyAsync(sh.rowmap, rowmap, (size_t)S * 4, cudaMemcpyHostToDevice, st));
  MC_CUDA(cudaMemcpyAsync(sh.sched_adm, hadm, (size_t)S * 4, cudaMemcpyHostToDevice, st));
  MC_CUDA(cudaMemcpyAsync(sh.limit, hlim, (size_t)S * 4, cudaMemcpyHostToDevice, st));
  MC_CUDA(cudaMemcpyAsync(sh.key, hkey, (size_t)S * 4, cudaMemcpyHostToDevice, st));
  if (cap > 0) MC_CUDA(cudaMemcpyAsync(sh.pol_prefix, hpre, (size_t)S * cap * 4, cudaMemcpyHostToDevice, st));
  MC_CUDA(cudaMemcpyAsync(sh.pol_prefix_len, hplen, (size_t)S * 4, cudaMemcpyHostToDevice, st));
  MC_CUDA(cudaMemcpyAsync(sh.pass_tiles, htiles, (size_t)n_tiles * 4, cudaMemcpyHostToDevice, st));
  MC_CUDA(cudaMemcpyAsync(sh.pass_sess, hsess, (size_t)n_sess * 4, cudaMemcpyHostToDevice, st));
  const int thr = 256, blocks = (S + thr - 1) / thr;
  sched_admit_kernel<<<blocks, thr, 0, st>>>(S, P, sh.sched_adm, sh.tok, sh.seglen, sh.pos, sh.gen_n, sh.next_tok);
  MC_CUDA(cudaGetLastError());
  sh.n_pass_tiles = n_tiles;
  sh.n_pass_sess = n_sess;
  int rc = enqueue_forward(sh, P, q->mode, 0.0, 0, false, true);
  sh.n_pass_tiles = sh.n_pass_sess = 0;
  if (rc != kOk) return rc;
  sched_resume_kernel<<<blocks, thr, 0, st>>>(S, sh.sched_adm, sh.seglen);
  MC_CUDA(cudaGetLastError());
  ss.busy += n_adm;
  ++q->n_prefill;
  q->n_admitted += n_adm;
  return kOk;
}

// Reads which slots of shard g have finished and moves their tokens to their requests.
int sched_harvest(mc_sched* q, size_t g) {
  SchedShard& ss = q->sh[g];
  DevBatch& sh = *q->batch->shard[g];
  const int S = sh.S;
  int32_t* seglen = ss.h_state;
  int32_t* gen_n = seglen + S;
  MC_CUDA(cudaMemcpyAsync(seglen, sh.seglen, (size_t)S * 4, cudaMemcpyDeviceToHost, sh.stream));
  MC_CUDA(cudaMemcpyAsync(gen_n, sh.gen_n, (size_t)S * 4, cudaMemcpyDeviceToHost, sh.stream));
  int st = check_device_error(sh.stream);  // synchronizes the stream
  if (st != kOk) return st;
  if (ss.timed) {
    float a = 0.f, d = 0.f;
    MC_CUDA(cudaEventElapsedTime(&a, ss.ev[0], ss.ev[1]));
    MC_CUDA(cudaEventElapsedTime(&d, ss.ev[1], ss.ev[2]));
    q->admit_us += 1e3 * a;
    q->decode_us += 1e3 * d;
    ss.timed = false;
  }
  std::vector<int> done;
  for (int s = 0; s < S; ++s)
    if (ss.slot_req[s] >= 0 && seglen[s] <= 0) done.push_back(s);
  if (done.empty()) return kOk;
  const int W = q->max_new;
  MC_CUDA(cudaMemcpy2DAsync(ss.h_tok, (size_t)W * 4, sh.out_tok, (size_t)sh.out_stride * 4, (size_t)W * 4, S,
                            cudaMemcpyDeviceToHost, sh.stream));
  MC_CUDA(cudaMemcpy2DAsync(ss.h_prob, (size_t)W * 4, sh.out_prob, (size_t)sh.out_stride * 4, (size_t)W * 4, S,
                            cudaMemcpyDeviceToHost, sh.stream));
  MC_CUDA(cudaStreamSynchronize(sh.stream));
  for (int s : done) {
    SchedReq& r = q->req[ss.slot_req[s]];
    const int n = std::min(std::max(gen_n[s], 0), r.n_new);
    r.tokens.assign(ss.h_tok + (size_t)s * W, ss.h_tok + (size_t)s * W + n);
    r.probs.assign(ss.h_prob + (size_t)s * W, ss.h_prob + (size_t)s * W + n);
    r.state = 2;
    ss.slot_req[s] = -1;
    --ss.busy;
    ++q->n_done;
    q->n_tokens += n;
  }
  return kOk;
}

int sched_in_flight(const mc_sched* q) {
  int n = (int)q->queue.size();
  for (const SchedShard& ss : q->sh) n += ss.busy;
  return n;
}

}  // namespace

extern "C" {

int mc_sched_open(mc_model* model, int slots, int context_size, int max_prompt, int max_new, const mc_sampling* sp,
                  int penalize_prompt, const int32_t* stops, int n_stops, mc_sched** out) {
  clear_error();
  DeviceRestore restore_device;
  if (!model || !out || slots <= 0 || max_new <= 0 || !sp) return set_error(kInvalidArgument, "mc_sched_open: bad arguments");
  if (n_stops < 0 || n_stops > kMaxStops || (n_stops > 0 && !stops))
    return set_error(kInvalidArgument, "mc_sched_open: 0 to 8 stop tokens");
  int st = check_policy(sp, nullptr, model->dev[0]->V, 0);
  if (st != kOk) return st;
  const bool penalize = penalize_prompt && sp->rep_penalty > 1.0;
  if (penalize && sp->rep_window <= 0)
    return set_error(kInvalidArgument, "mc_sched_open: a prompt penalty needs rep_window >= 1");
  auto q = std::make_unique<mc_sched>();
  // admission passes run over lists of tiles: the batch keeps a scratch row for every prefill row
  if ((st = batch_open(model, slots, context_size, max_prompt, 0, false, &q->batch)) != kOk) return st;
  q->sp = *sp;
  q->penalize_prompt = penalize ? 1 : 0;
  // argmax with nothing to change the logits is greedyLoop's selection: the decode steps then
  // run the greedy head fused into the final block launch
  q->mode = sp->temperature <= 0.001 && sp->rep_penalty <= 1.0 && !sp->ban_trigrams ? 0 : 3;
  q->max_new = max_new;
  q->admit_min = std::max(1, slots / 8);
  q->n_stops = n_stops;
  for (int k = 0; k < n_stops; ++k) q->stops[k] = stops[k];
  const int cap = penalize ? sp->rep_window : 0;
  for (size_t g = 0; g < q->batch->shard.size(); ++g) {
    DevBatch& sh = *q->batch->shard[g];
    SchedShard ss;
    ss.slot_req.assign(sh.S, -1);
    ss.limit.assign(sh.S, 0);
    ss.key.assign(sh.S, 0);
    ss.prefix.assign((size_t)sh.S * cap, 0);
    ss.prefix_len.assign(sh.S, 0);
    q->sh.push_back(std::move(ss));
    if (sh.S == 0) continue;
    MC_CUDA(cudaSetDevice(sh.m->device));
    SchedShard& sp_ = q->sh.back();
    const size_t up = (size_t)sh.S * (sh.pmax + cap + 8);
    MC_CUDA(cudaHostAlloc(&sp_.h_up, up * 4, cudaHostAllocDefault));
    for (cudaEvent_t& e : sp_.ev) MC_CUDA(cudaEventCreate(&e));
    MC_CUDA(cudaHostAlloc(&sp_.h_state, (size_t)sh.S * 2 * 4, cudaHostAllocDefault));
    MC_CUDA(cudaHostAlloc(&sp_.h_tok, (size_t)sh.S * max_new * 4, cudaHostAllocDefault));
    MC_CUDA(cudaHostAlloc(&sp_.h_prob, (size_t)sh.S * max_new * 4, cudaHostAllocDefault));
    if ((st = ensure_step_outputs(sh, q->mode == 3, max_new)) != kOk) return st;
    if ((st = sh.alloc(sh.gen_n, (size_t)sh.S * 4)) || (st = sh.alloc(sh.limit, (size_t)sh.S * 4)) ||
        (st = sh.alloc(sh.key, (size_t)sh.S * 4)) || (st = sh.alloc(sh.sched_adm, (size_t)sh.S * 4)) ||
        (st = sh.alloc(sh.pass_tiles, (size_t)sh.S * 4)) || (st = sh.alloc(sh.pass_sess, (size_t)sh.S * 4)) ||
        (st = sh.alloc(sh.pol_prefix_len, (size_t)sh.S * 4)) || (st = sh.alloc(sh.pol_state, (size_t)sh.S * 4)))
      return st;
    if (cap > 0 && (st = sh.alloc(sh.pol_prefix, (size_t)sh.S * cap * 4)) != kOk) return st;
    sh.pol_prefix_cap = cap;
    MC_CUDA(cudaMemsetAsync(sh.seglen, 0, (size_t)sh.S * 4, sh.stream));
    MC_CUDA(cudaMemsetAsync(sh.gen_n, 0, (size_t)sh.S * 4, sh.stream));
    MC_CUDA(cudaMemsetAsync(sh.pol_prefix_len, 0, (size_t)sh.S * 4, sh.stream));
    MC_CUDA(cudaMemsetAsync(sh.out_tok, 0xFF, (size_t)sh.S * sh.out_stride * 4, sh.stream));
    MC_CUDA(cudaMemsetAsync(sh.step, 0, 4, sh.stream));
    sh.pol = DevBatch::Policy();
    sh.pol.temperature = sp->temperature;
    sh.pol.rep_penalty = sp->rep_penalty;
    sh.pol.top_p = sp->top_p;
    sh.pol.top_k = sp->top_k;
    sh.pol.rep_window = sp->rep_window;
    sh.pol.ban_trigrams = sp->ban_trigrams ? 1 : 0;
    sh.per_session = true;
    sh.n_stops = n_stops;
    for (int k = 0; k < n_stops; ++k) sh.stops[k] = stops[k];
    if ((st = check_device_error(sh.stream)) != kOk) return st;
  }
  *out = q.release();
  return kOk;
}

int mc_sched_close(mc_sched* q) {
  DeviceRestore restore_device;  // the destructors switch to the shards' devices
  delete q;
  return kOk;
}

int mc_sched_submit(mc_sched* q, const int32_t* prompt, int len, int n_new, uint32_t draw_key, int64_t* id) {
  clear_error();
  DeviceRestore restore_device;
  if (!q || len < 0 || (len > 0 && !prompt) || n_new <= 0 || n_new > q->max_new)
    return set_error(kInvalidArgument, "mc_sched_submit: bad arguments (n_new in [1, max_new])");
  if (std::min(len, q->batch->window) > q->batch->pmax)
    return set_error(kInvalidArgument, "mc_sched_submit: prompt longer than the scheduler's max_prompt");
  SchedReq r;
  r.prompt.assign(prompt, prompt + len);
  r.n_new = n_new;
  r.key = draw_key;
  q->req.push_back(std::move(r));
  q->queue.push_back((int64_t)q->req.size() - 1);
  if (id) *id = (int64_t)q->req.size() - 1;
  return kOk;
}

int mc_sched_step(mc_sched* q, int steps, int* in_flight) {
  clear_error();
  DeviceRestore restore_device;
  if (!q || steps < 1) return set_error(kInvalidArgument, "mc_sched_step: bad arguments");
  int st;
  const auto t0 = std::chrono::steady_clock::now();
  for (size_t g = 0; g < q->sh.size(); ++g) {
    DevBatch& sh = *q->batch->shard[g];
    SchedShard& ss = q->sh[g];
    if (sh.S == 0) continue;
    MC_CUDA(cudaSetDevice(sh.m->device));
    MC_CUDA(cudaEventRecord(ss.ev[0], sh.stream));
    const int free_slots = sh.S - ss.busy;
    if (!q->queue.empty() && free_slots > 0 && (free_slots >= q->admit_min || ss.busy == 0))
      if ((st = sched_admit(q, g)) != kOk) return st;
    MC_CUDA(cudaEventRecord(ss.ev[1], sh.stream));
    if (ss.busy > 0) {
      for (int k = 0; k < steps; ++k)
        if ((st = run_graph_step(sh, q->mode, 0.0, 0, false)) != kOk) return st;
      q->n_steps += steps;
    }
    MC_CUDA(cudaEventRecord(ss.ev[2], sh.stream));
    ss.timed = true;
  }
  for (size_t g = 0; g < q->sh.size(); ++g) {
    DevBatch& sh = *q->batch->shard[g];
    if (sh.S == 0 || q->sh[g].busy == 0) continue;
    MC_CUDA(cudaSetDevice(sh.m->device));
    if ((st = sched_harvest(q, g)) != kOk) return st;
  }
  q->host_us += std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
  if (in_flight) *in_flight = sched_in_flight(q);
  return kOk;
}

int mc_sched_run(mc_sched* q, int steps_per_poll) {
  clear_error();
  DeviceRestore restore_device;
  if (!q) return set_error(kInvalidArgument, "mc_sched_run: null scheduler");
  int left = 1, st;
  while (left > 0)
    if ((st = mc_sched_step(q, std::max(1, steps_per_poll), &left)) != kOk) return st;
  return kOk;
}

int mc_sched_result(mc_sched* q, int64_t id, int32_t* tokens, float* probs, int capacity, int* n) {
  clear_error();
  DeviceRestore restore_device;
  if (!q || id < 0 || id >= (int64_t)q->req.size() || !n) return set_error(kInvalidArgument, "mc_sched_result: bad id");
  const SchedReq& r = q->req[id];
  if (r.state != 2) {
    *n = -1;  // still queued or running
    return kOk;
  }
  const int k = std::min(capacity, (int)r.tokens.size());
  if (tokens) std::copy(r.tokens.begin(), r.tokens.begin() + k, tokens);
  if (probs) std::copy(r.probs.begin(), r.probs.begin() + k, probs);
  *n = (int)r.tokens.size();
  return kOk;
}

int mc_sched_stats(const mc_sched* q, int64_t* out) {
  clear_error();
  DeviceRestore restore_device;
  if (!q || !out) return set_error(kInvalidArgument, "mc_sched_stats: bad arguments");
  out[0] = q->n_prefill;
  out[1] = q->n_steps;
  out[2] = q->n_tokens;
  out[3] = q->n_done;
  out[4] = sched_in_flight(q);
  out[5] = (int64_t)q->admit_us;
  out[6] = (int64_t)q->decode_us;
  out[7] = (int64_t)q->host_us;
  out[8] = (int64_t)q->admit_host_us;
  out[9] = q->n_admitted;
  return kOk;
}

int mc_sched_set_admit_min(mc_sched* q, int admit_min) {
  clear_error();
  DeviceRestore restore_device;
  if (!q || admit_min < 1) return set_error(kInvalidArgument, "mc_sched_set_admit_min: admit_min >= 1");
  q->admit_min = admit_min;
  return kOk;
}

}  // extern "C"
