// Host orchestration of the engine: the device replica of a model (pre-tiled weights), session
// batches (state in HBM), and the launch sequences of prefill and decode.
//
// Decode step (one token for every session of a batch), all on one stream and captured once in a
// CUDA graph:
//   for each block b: block_kernel(b) [+ attn_decode_kernel(b)]
//   block_kernel(final: last output projection + final RMSNorm)
//   head_kernel (vocabulary split across CTAs) -> select_kernel (also advances the step counter)
// Prefill runs the same kernels layer-major over whole prompt segments (attn_prefill_kernel).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

#include "mc_engine.cuh"
#include "mc_host.h"

namespace mc {

int parse_model_file(const uint8_t* data, size_t n, struct HostModel& m);

namespace eng {

// ------------------------------------------------------------------------------------------------
// Weight tiling
// ------------------------------------------------------------------------------------------------
// Builds the pre-tiled image of W [rows x K] (row-major int8): chunk c, K tile kt, row r of the
// tile = W row perm[c*128 + r] (-1: zero row), 128-byte swizzled.
static std::vector<uint8_t> tile_weights(const int8_t* W, int K, const std::vector<int>& perm, int nchunks, int ktiles) {
  std::vector<uint8_t> img((size_t)nchunks * ktiles * kTile, 0);
  for (int c = 0; c < nchunks; ++c)
    for (int kt = 0; kt < ktiles; ++kt) {
      uint8_t* t = img.data() + ((size_t)c * ktiles + kt) * kTile;
      for (int r = 0; r < 128; ++r) {
        const int src = perm[(size_t)c * 128 + r];
        if (src < 0) continue;
        for (int k = 0; k < 128; ++k) {
          const int kk = kt * 128 + k;
          if (kk >= K) break;
          const int chunk = k / 16;
          const size_t off = (size_t)(r >> 3) * 1024 + (r & 7) * 128 + (size_t)((chunk ^ (r & 7)) << 4) + (k & 15);
          t[off] = (uint8_t)W[(size_t)src * K + kk];
        }
      }
    }
  return img;
}

static std::vector<int> perm_identity(int rows, int nchunks) {
  std::vector<int> p((size_t)nchunks * 128, -1);
  for (int i = 0; i < rows; ++i) p[i] = i;
  return p;
}

// Paired chunks: chunk c holds units [64c, 64c+64) of the first half (rows u) followed by the same
// units of the second half (rows half + u): the GLU value/gate (W1) and highway delta/gate (W2)
// pairs then meet in one 128-column accumulator.
static std::vector<int> perm_paired(int half, int nchunks) {
  std::vector<int> p((size_t)nchunks * 128, -1);
  for (int c = 0; c < nchunks; ++c)
    for (int j = 0; j < kHalfChunk; ++j) {
      const int u = c * kHalfChunk + j;
      if (u < half) {
        p[(size_t)c * 128 + j] = u;
        p[(size_t)c * 128 + kHalfChunk + j] = half + u;
      }
    }
  return p;
}

// Split pairs (the decode kernel's layout): tile 2c holds units [128c, 128c+128) of the first half,
// tile 2c+1 the same units of the second half, so a TMEM lane sees a value and its gate in two
// consecutive accumulators.
static std::vector<int> perm_split(int half, int npairs) {
  std::vector<int> p((size_t)2 * npairs * 128, -1);
  for (int c = 0; c < npairs; ++c)
    for (int j = 0; j < 128; ++j) {
      const int u = c * 128 + j;
      if (u < half) {
        p[(size_t)(2 * c) * 128 + j] = u;
        p[(size_t)(2 * c + 1) * 128 + j] = half + u;
      }
    }
  return p;
}

struct DevGemm {
  uint8_t* tiles = nullptr;
  int K = 0, ktiles = 0, nchunks = 0;
  float scale = 0;
};

struct DevBlock {
  int steps = 0, attn_slot = -1;
  std::vector<int> dil;
  DevGemm w1, w2, wsel, qkv, out;
  DevGemm w1d, w2d;  // W1 and W2 in split-pair tiles (decode kernel)
  float *b1 = nullptr, *b2 = nullptr, *gamma = nullptr, *attn_norm = nullptr;
};

struct DevModel {
  int device = 0;
  int V = 0, D = 0, H = 0, max_context = 0, heads = 0, window = 0, cache = 0, ring = 0, total_steps = 0, n_attn = 0;
  int dec_kt = 0;         // decode kernel: K tiles of its activation planes
  int dec_r = 32;         // decode kernel: sessions per CTA (16 or 32)
  size_t dec_smem = 0;    // decode kernel: dynamic shared memory
  bool dec_ok = false;    // the decode kernel fits this model (else decode uses block_kernel)
  bool tied = true;
  int8_t* embed = nullptr;
  float embed_scale = 0;
  DevGemm head;
  float *head_b = nullptr, *final_gain = nullptr, *latch_base = nullptr;
  std::vector<DevBlock> blocks;
  // small models without attention: every block's int8 rows for tiny_generate_kernel
  bool tiny = false;
  uint32_t* tiny_w = nullptr;
  int tiny_blk_words = 0;
  size_t tiny_smem = 0;
  std::vector<void*> allocs;
  ~DevModel() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    for (void* p : allocs) cudaFree(p);
    cudaSetDevice(prev);
  }
  template <class T>
  int upload(T*& dst, const void* src, size_t bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, std::max<size_t>(bytes, 16)) != cudaSuccess)
      return set_error(kOutOfMemory, "cudaMalloc failed for model weights");
    allocs.push_back(p);
    if (bytes) MC_CUDA(cudaMemcpy(p, src, bytes, cudaMemcpyHostToDevice));
    dst = reinterpret_cast<T*>(p);
    return kOk;
  }
  int upload_gemm(DevGemm& g, const int8_t* W, int rows, int K, float scale, int paired_half, bool split = false) {
    g.K = K;
    g.ktiles = (K + 127) / 128;
    g.scale = scale;
    std::vector<int> perm;
    if (split) {
      g.nchunks = 2 * ((paired_half + 127) / 128);
      perm = perm_split(paired_half, g.nchunks / 2);
    } else if (paired_half > 0) {
      g.nchunks = (paired_half + kHalfChunk - 1) / kHalfChunk;
      perm = perm_paired(paired_half, g.nchunks);
    } else {
      g.nchunks = (rows + 127) / 128;
      perm = perm_identity(rows, g.nchunks);
    }
    auto img = tile_weights(W, K, perm, g.nchunks, g.ktiles);
    return upload(g.tiles, img.data(), img.size());
  }
};

// Latch base logits (ca/latch.go:11-25 over ca/layout.go:63-85).
static void latch_base_logits(int D, std::vector<float>& out) {
  out.resize(D);
  const double minT = 1.5, maxT = 64.0;
  for (int d = 0; d < D; ++d) {
    double td = minT;
    if (D > 1) td = minT * std::pow(std::pow(maxT / minT, 1.0 / (double)(D - 1)), (double)d);
    const double lam = (double)(float)std::pow(2.0, -1.0 / td);
    if (lam <= 0.0) out[d] = -15.0f;
    else if (lam >= 1.0) out[d] = 15.0f;
    else out[d] = (float)std::log(lam / (1.0 - lam));
  }
}

static int step_dilation(int initial, int base, int step) {
  int d = initial;
  for (int s = 0; s < step && d < 32; ++s) d *= base;
  return std::min(d, 32);
}

int build_dev_model(const HostModel& hm, int device, std::unique_ptr<DevModel>& out) {
  auto m = std::make_unique<DevModel>();
  m->device = device;
  MC_CUDA(cudaSetDevice(device));
  const int D = hm.state, H = hm.hidden, V = hm.vocab;
  m->V = V;
  m->D = D;
  m->H = H;
  m->tied = hm.tied;
  m->max_context = hm.context_size < 64 ? 128 : hm.context_size;
  m->heads = hm.attn_heads;
  m->window = hm.attn_window;
  m->cache = hm.attn_window > 0 ? hm.attn_window : m->max_context;
  if (D > 384) return set_error(kUnsupported, "state_size > 384 is not supported by this build");
  if (D % 4 != 0 || H % 4 != 0) return set_error(kUnsupported, "state_size and hidden_size must be multiples of 4");
  int st;
  if ((st = m->upload(m->embed, hm.embed.data.data(), hm.embed.data.size())) != kOk) return st;
  m->embed_scale = hm.embed.scale;
  const HostTensor& hw = hm.tied ? hm.embed : hm.head_w;
  if ((st = m->upload_gemm(m->head, hw.data.data(), V, D, hw.scale, 0)) != kOk) return st;
  if ((st = m->upload(m->head_b, hm.head_b.data(), hm.head_b.size() * 4)) != kOk) return st;
  if ((int)hm.final_norm.size() == D) {
    if ((st = m->upload(m->final_gain, hm.final_norm.data(), D * 4)) != kOk) return st;
  }
  std::vector<float> base;
  latch_base_logits(D, base);
  if ((st = m->upload(m->latch_base, base.data(), D * 4)) != kOk) return st;
  int total = 0, longest = 0, nattn = 0;
  for (const HostBlock& hb : hm.blocks) {
    DevBlock b;
    b.steps = hb.steps;
    if (hb.steps > kMaxSteps) return set_error(kUnsupported, "more than 8 rule steps per block");
    for (int s = 0; s < hb.steps; ++s) {
      b.dil.push_back(step_dilation(hb.initial_dilation, hb.dilation_base, s));
      longest = std::max(longest, b.dil.back());
    }
    total += hb.steps;
    if ((st = m->upload_gemm(b.w1, hb.w1.data.data(), 2 * H, 3 * D, hb.w1.scale, H)) != kOk) return st;
    if ((st = m->upload_gemm(b.w2, hb.w2.data.data(), 2 * D, H, hb.w2.scale, D)) != kOk) return st;
    if ((st = m->upload_gemm(b.w1d, hb.w1.data.data(), 2 * H, 3 * D, hb.w1.scale, H, true)) != kOk) return st;
    if ((st = m->upload_gemm(b.w2d, hb.w2.data.data(), 2 * D, H, hb.w2.scale, D, true)) != kOk) return st;
    if ((st = m->upload_gemm(b.wsel, hb.wsel.data.data(), D, D, hb.wsel.scale, 0)) != kOk) return st;
    if ((st = m->upload(b.b1, hb.b1.data(), hb.b1.size() * 4)) != kOk) return st;
    if ((st = m->upload(b.b2, hb.b2.data(), hb.b2.size() * 4)) != kOk) return st;
    if ((int)hb.gamma.size() == D && (st = m->upload(b.gamma, hb.gamma.data(), D * 4)) != kOk) return st;
    if (hb.has_attn) {
      if (m->heads <= 0 || D % m->heads != 0) return set_error(kBadModel, "attention blocks need attn_heads dividing state_size");
      if (D / m->heads > 64) return set_error(kUnsupported, "attention head width above 64");
      b.attn_slot = nattn++;
      if ((st = m->upload_gemm(b.qkv, hb.qkv.data.data(), 3 * D, D, hb.qkv.scale, 0)) != kOk) return st;
      if ((st = m->upload_gemm(b.out, hb.out.data.data(), D, D, hb.out.scale, 0)) != kOk) return st;
      if ((st = m->upload(b.attn_norm, hb.attn_norm.data(), D * 4)) != kOk) return st;
    }
    m->blocks.push_back(std::move(b));
  }
  m->total_steps = total;
  m->ring = longest + 1;
  m->n_attn = nattn;
  m->dec_kt = (std::max(3 * D, H) + 127) / 128;
  // Sessions per CTA: 16 with a 3-stage weight ring where two such CTAs share a multiprocessor
  // (state width <= 128: their latency chains interleave), else 32 with a 6-stage ring, else
  // (wide models) 16 with 3 stages, one CTA per multiprocessor. MC_DECODE_R=16 / 32 forces one.
  const size_t smem16 = decode_smem_bytes(D, H, m->dec_kt, 16, 3), smem32 = decode_smem_bytes(D, H, m->dec_kt, 32, 6);
  const bool pair16 = decode_ctas_per_sm((D + 127) / 128, 16) == 2 && 2 * (smem16 + 1024) <= kSmemPerSm;
  const char* rsel = getenv("MC_DECODE_R");
  const int want = rsel ? atoi(rsel) : 0;
  m->dec_r = (want == 16 || (want != 32 && pair16) || smem32 > kDecodeSmemMax) ? 16 : 32;
  m->dec_smem = m->dec_r == 16 ? smem16 : smem32;
  m->dec_ok = m->dec_smem <= kDecodeSmemMax;
  if (nattn > 0 && m->cache > 128) return set_error(kUnsupported, "attention caches above 128 positions");
  // Small models without attention also keep their blocks' int8 rows for tiny_generate_kernel:
  // per block W_select, W1 and W2 row-major, each row padded to an odd number of 16-byte quads.
  const int nb = (int)hm.blocks.size();
  if (nattn == 0 && m->tied && nb >= 1 && nb <= kTinyMaxBlocks && D <= kTinyMaxD && D % 16 == 0 && H % 16 == 0 &&
      tiny_smem_bytes(D, H, V, nb, total, m->ring) <= kTinySmemMax) {
    const int bw = tiny_block_words(D, H);
    std::vector<uint32_t> img((size_t)nb * bw, 0u);
    auto put_rows = [&](uint32_t* dst, const std::vector<int8_t>& w, int rows, int k) {
      const int kw = tiny_stride_words(k);
      for (int r = 0; r < rows; ++r) memcpy(dst + (size_t)r * kw, w.data() + (size_t)r * k, (size_t)k);
      return dst + (size_t)rows * kw;
    };
    for (int bi = 0; bi < nb; ++bi) {
      const HostBlock& hb = hm.blocks[bi];
      uint32_t* p = img.data() + (size_t)bi * bw;
      p = put_rows(p, hb.wsel.data, D, D);
      p = put_rows(p, hb.w1.data, 2 * H, 3 * D);
      put_rows(p, hb.w2.data, 2 * D, H);
    }
    if ((st = m->upload(m->tiny_w, img.data(), img.size() * 4)) != kOk) return st;
    m->tiny_blk_words = bw;
    m->tiny_smem = tiny_smem_bytes(D, H, V, nb, total, m->ring);
    m->tiny = true;
  }
  out = std::move(m);
  return kOk;
}

// ------------------------------------------------------------------------------------------------
// Session batches on one device
// ------------------------------------------------------------------------------------------------
// SM ids the block kernel's plane cache covers (ids above it slice every chunk instead).
constexpr int kACacheSms = 256;

struct DevBatch {
  DevModel* m = nullptr;
  int S = 0, window = 0, pmax = 0, nsplit = 1, topk = 0;
  bool decode_kernel = true;  // decode steps use block_decode_kernel, else block_kernel (see batch_create)
  int n_sm = 148;             // multiprocessors of the device (persistent grids)
  size_t rows = 0;  // scratch rows
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  int32_t* sel_done = nullptr;  // select_kernel's finished-block counter (zero between launches)
  int n_stops = 0;              // stop tokens of the generation being enqueued (0: none)
  int stops[kMaxStops] = {0};
  // The decode-loop policy of mc_generate_policy (mode 3): the sampling knobs, each session's
  // penalty prefix (its last pol_prefix_len[s] prompt tokens), and the token automaton with each
  // session's state.
  struct Policy {
    double temperature = 0, rep_penalty = 1, top_p = 1;
    int top_k = 0, rep_window = 0, ban_trigrams = 0;
    const int32_t* dfa = nullptr;
    bool operator==(const Policy& o) const {
      return temperature == o.temperature && rep_penalty == o.rep_penalty && top_p == o.top_p && top_k == o.top_k &&
             rep_window == o.rep_window && ban_trigrams == o.ban_trigrams && dfa == o.dfa;
    }
  } pol;
  int32_t *pol_prefix = nullptr, *pol_prefix_len = nullptr, *pol_state = nullptr, *pol_dfa = nullptr;
  int pol_prefix_cap = 0;  // tokens per session that pol_prefix holds
  size_t pol_dfa_n = 0;    // entries pol_dfa holds
  // Per-session generation (the scheduler's slots): tokens emitted, token limit and draw key of
  // each session, used by mode-3 launches when per_session is set; sched_adm is the scheduler's
  // admission list.
  bool per_session = false;
  int32_t *gen_n = nullptr, *limit = nullptr, *sched_adm = nullptr;
  // A prefill pass over some sessions only (the scheduler's admissions): the block kernel runs the
  // n_pass_tiles tiles of pass_tiles, the prefill attention the n_pass_sess sessions of pass_sess
  // (0: all). Set for one pass.
  int32_t *pass_tiles = nullptr, *pass_sess = nullptr;
  int n_pass_tiles = 0, n_pass_sess = 0;
  uint32_t* key = nullptr;
  uint8_t* a_cache = nullptr;    // block kernel: per-SM digit-plane cache of GEMMs wider than the A slots
  int a_cache_kt = 0;
  int32_t *pos = nullptr, *seglen = nullptr, *tok = nullptr, *next_tok = nullptr, *step = nullptr, *rowmap = nullptr,
          *rowmap_id = nullptr, *target = nullptr;
  float *norm_ring = nullptr, *latch = nullptr, *kv = nullptr;
  float *cur = nullptr, *blockin = nullptr, *xbuf = nullptr, *hbuf = nullptr, *qbuf = nullptr, *att = nullptr,
        *att_rowmax = nullptr, *fnorm = nullptr, *fnorm_rowmax = nullptr, *kvlin = nullptr, *logits = nullptr;
  float4* part = nullptr;
  float* gmax = nullptr;  // sampling: [S][128] the head's 32-column group maxima of each row
  float* topv = nullptr;
  int32_t* topi = nullptr;
  unsigned long long* trace = nullptr;  // phase timestamps of CTA 0 per block-kernel launch (debug)
  int32_t* out_tok = nullptr;
  float* out_prob = nullptr;
  double* out_logprob = nullptr;
  // scoring (every row of a segment through the head): per-row scratch, grown on demand
  size_t sc_rows = 0;
  int sc_nsplit = 1;
  int32_t *sc_rowmap = nullptr, *sc_target = nullptr, *sc_valid = nullptr, *sc_next = nullptr;
  float4* sc_part = nullptr;
  double* sc_logprob = nullptr;
  int out_stride = 0;
  cudaGraphExec_t graph = nullptr;
  // pinned host staging of uploaded prompt segments (tokens, lengths, zero positions, row map),
  // and an event recorded after the copies out of it: the next upload waits for it
  int32_t* h_stage = nullptr;
  size_t h_stage_n = 0;
  cudaEvent_t h_stage_done = nullptr;
  // pinned host staging of one append: [tokens S | next S | prob S | device error word, padding 4 |
  // logits S x V], so its copies are asynchronous and one stream synchronization ends the call
  int32_t* h_step = nullptr;
  size_t h_step_n = 0;
  // Everything the captured decode step bakes in; a change forces a new capture.
  struct GraphKey {
    int mode = -1, logits = -1, stride = -1;
    double inv_t = 0;
    uint32_t session0 = 0;
    const void* out_tok = nullptr;
    const void* logits_buf = nullptr;
    int n_stops = 0;
    int stops[kMaxStops] = {0};
    Policy pol;
    bool per_session = false;
    bool operator==(const GraphKey& o) const {
      if (n_stops != o.n_stops || !(pol == o.pol) || per_session != o.per_session) return false;
      for (int k = 0; k < n_stops; ++k)
        if (stops[k] != o.stops[k]) return false;
      return mode == o.mode && logits == o.logits && stride == o.stride && inv_t == o.inv_t && session0 == o.session0 &&
             out_tok == o.out_tok && logits_buf == o.logits_buf;
    }
  } graph_key;
  ~DevBatch() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(m ? m->device : prev);
    if (graph) cudaGraphExecDestroy(graph);
    if (h_stage_done) cudaEventSynchronize(h_stage_done), cudaEventDestroy(h_stage_done);
    if (h_stage) cudaFreeHost(h_stage);
    if (h_step) cudaFreeHost(h_step);
    for (void* p : allocs) cudaFree(p);
    if (stream) cudaStreamDestroy(stream);
    cudaSetDevice(prev);
  }
  template <class T>
  int alloc(T*& p, size_t bytes) {
    void* q = nullptr;
    if (cudaMalloc(&q, std::max<size_t>(bytes, 16)) != cudaSuccess) {
      cudaGetLastError();
      return set_error(kOutOfMemory, "cudaMalloc of " + std::to_string(bytes) + " bytes failed");
    }
    allocs.push_back(q);
    p = reinterpret_cast<T*>(q);
    return kOk;
  }
};

static bool g_attr_done[64];
static std::mutex g_attr_mu;

static int ensure_attrs(int device) {
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (device < 64 && g_attr_done[device]) return kOk;
  MC_CUDA(cudaFuncSetAttribute(block_kernel<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBlockSmem));
  MC_CUDA(cudaFuncSetAttribute(block_kernel<1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBlockSmem));
  MC_CUDA(cudaFuncSetAttribute(block_kernel<2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBlockSmem));
  MC_CUDA(cudaFuncSetAttribute(block_kernel<2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBlockSmem));
  MC_CUDA(cudaFuncSetAttribute(block_kernel<3, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBlockSmem));
  MC_CUDA(cudaFuncSetAttribute(block_kernel<3, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBlockSmem));
  MC_CUDA(cudaFuncSetAttribute(block_decode_kernel<1, 32, 6>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDecodeSmemMax));
  MC_CUDA(cudaFuncSetAttribute(block_decode_kernel<2, 32, 6>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDecodeSmemMax));
  MC_CUDA(cudaFuncSetAttribute(block_decode_kernel<3, 32, 6>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDecodeSmemMax));
  MC_CUDA(cudaFuncSetAttribute(block_decode_kernel<1, 16, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDecodeSmemMax));
  // two CTAs of this instance share a multiprocessor: ask for the largest shared-memory carveout
  MC_CUDA(cudaFuncSetAttribute(block_decode_kernel<1, 16, 3>, cudaFuncAttributePreferredSharedMemoryCarveout,
                               (int)cudaSharedmemCarveoutMaxShared));
  MC_CUDA(cudaFuncSetAttribute(block_decode_kernel<2, 16, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDecodeSmemMax));
  MC_CUDA(cudaFuncSetAttribute(block_decode_kernel<3, 16, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDecodeSmemMax));
  MC_CUDA(cudaFuncSetAttribute(head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kHeadSmem));
  MC_CUDA(cudaFuncSetAttribute(tiny_generate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTinySmemMax));
  MC_CUDA(cudaFuncSetAttribute(policy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)policy_smem(kPolicyMaxVocab)));
  MC_CUDA(cudaFuncSetAttribute(attn_decode_staged_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAsSmemMax));
  MC_CUDA(cudaFuncSetAttribute(attn_decode_staged_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAsSmemMax));
  MC_CUDA(cudaFuncSetAttribute(attn_decode_staged_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAsSmemMax));
  MC_CUDA(cudaFuncSetAttribute(attn_decode_staged_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAsSmemMax));
  MC_CUDA(cudaFuncSetAttribute(attn_decode_staged_kernel<48>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAsSmemMax));
  MC_CUDA(cudaFuncSetAttribute(attn_decode_staged_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAsSmemMax));
  MC_CUDA(cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
  MC_CUDA(cudaFuncSetAttribute(attn_prefill_fast_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
  MC_CUDA(cudaFuncSetAttribute(attn_prefill_fast_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
  MC_CUDA(cudaFuncSetAttribute(attn_prefill_fast_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
  MC_CUDA(cudaFuncSetAttribute(attn_prefill_fast_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
  MC_CUDA(cudaFuncSetAttribute(attn_prefill_fast_kernel<48>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
  MC_CUDA(cudaFuncSetAttribute(attn_prefill_fast_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
  // several prefill CTAs (a few tens of KB each) share a multiprocessor
  MC_CUDA(cudaFuncSetAttribute(attn_prefill_fast_kernel<32>, cudaFuncAttributePreferredSharedMemoryCarveout,
                               (int)cudaSharedmemCarveoutMaxShared));
  if (device < 64) g_attr_done[device] = true;
  return kOk;
}

// Scratch bytes a batch may hold for prefill rows (MC_PREFILL_SCRATCH_MB, default 8 GiB). A prefill
// whose rows need more runs as several passes over contiguous ranges of sessions.
static size_t prefill_scratch_budget() {
  const char* e = getenv("MC_PREFILL_SCRATCH_MB");
  const long long mb = e ? atoll(e) : 8192;
  return (size_t)std::max(mb, 1LL) << 20;
}

int batch_create(DevModel* m, int S, int window, int pmax, int topk, bool allow_passes, std::unique_ptr<DevBatch>& out) {
  MC_CUDA(cudaSetDevice(m->device));
  int st = ensure_attrs(m->device);
  if (st != kOk) return st;
  auto b = std::make_unique<DevBatch>();
  b->m = m;
  b->S = S;
  b->window = window;
  b->pmax = std::max(1, std::min(pmax, 128));
  b->topk = topk;
  MC_CUDA(cudaDeviceGetAttribute(&b->n_sm, cudaDevAttrMultiProcessorCount, m->device));
  {
    // Decode steps run on block_decode_kernel (weights on the MMA's M side, 16 sessions per CTA)
    // unless the batch is large and the model wide: from three waves of 128-session tiles on, at
    // state widths above 128, block_kernel (128 sessions on M, each weight tile read once per 128
    // sessions instead of once per 16) takes the decode steps too (config 3 at 65,536 sessions:
    // 2.64 against 3.19 ms per block launch). MC_DECODE_KERNEL=block / decode forces one.
    const char* k = getenv("MC_DECODE_KERNEL");
    const bool big_wide = m->D > 128 && (long long)(S + 127) / 128 >= 3LL * b->n_sm;
    const bool want_block = k ? strcmp(k, "block") == 0 : big_wide;
    b->decode_kernel = m->dec_ok && !want_block;
  }
  const int D = m->D, H = m->H;
  const int spt_min = std::max(1, 128 / b->pmax);
  const size_t full_tiles = std::max((size_t)(S + 127) / 128, (size_t)(S + spt_min - 1) / spt_min);
  // per scratch row: cur, blockin, the 3D neighbourhood, hidden, q, attention output, final norm
  // (8D + H floats), two row maxima and a prefill row's key and value (2D floats)
  const size_t row_bytes = (size_t)(10 * D + H + 2) * 4;
  size_t tiles = full_tiles;
  if (allow_passes) {
    // decode needs one row per session; a prefill may run in passes of fewer rows
    const size_t fit = std::max<size_t>(prefill_scratch_budget() / (row_bytes * 128), 1);
    tiles = std::max((size_t)(S + 127) / 128, std::min(full_tiles, fit));
  }
  b->rows = tiles * 128;
  // vocabulary splits: enough CTAs to cover the SMs
  const int mtiles = (S + 127) / 128;
  // at most 16 chunks per CTA (the head kernel stages their biases in shared memory), at most 16 splits
  const int want = std::max((m->head.nchunks + 15) / 16, std::min({16, m->head.nchunks, (296 + mtiles - 1) / mtiles}));
  const int cps = (m->head.nchunks + want - 1) / want;
  b->nsplit = (m->head.nchunks + cps - 1) / cps;  // every split gets at least one chunk
  MC_CUDA(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking));
  const size_t R = b->rows;
  if ((st = b->alloc(b->pos, S * 4)) || (st = b->alloc(b->seglen, S * 4)) || (st = b->alloc(b->tok, (size_t)S * b->pmax * 4)) ||
      (st = b->alloc(b->next_tok, S * 4)) || (st = b->alloc(b->step, 4)) || (st = b->alloc(b->sel_done, 4)) || (st = b->alloc(b->rowmap, S * 4)) ||
      (st = b->alloc(b->rowmap_id, S * 4)) || (st = b->alloc(b->target, S * 4)))
    return st;
  if ((st = b->alloc(b->norm_ring, (size_t)S * m->total_steps * m->ring * D * 4)) ||
      (st = b->alloc(b->latch, (size_t)S * m->total_steps * D * 4)) ||
      (st = b->alloc(b->kv, (size_t)S * std::max(m->n_attn, 0) * 2 * m->cache * D * 4)))
    return st;
  if ((st = b->alloc(b->cur, R * D * 4)) || (st = b->alloc(b->blockin, R * D * 4)) || (st = b->alloc(b->xbuf, R * 3 * D * 4)) ||
      (st = b->alloc(b->hbuf, R * H * 4)) || (st = b->alloc(b->qbuf, R * D * 4)) || (st = b->alloc(b->att, R * D * 4)) ||
      (st = b->alloc(b->att_rowmax, R * 4)) || (st = b->alloc(b->fnorm, R * D * 4)) || (st = b->alloc(b->fnorm_rowmax, R * 4)))
    return st;
  // a prefill row's key and value: session i's row t of a pass is row (i - first session) * P + t,
  // below the pass's tiles x 128 scratch rows
  if (m->n_attn > 0 && (st = b->alloc(b->kvlin, R * 2 * D * 4))) return st;
  {
    // K tiles of the widest GEMM (K = 3D for W1, H for W2): beyond the A slots, the block kernel
    // slices its first chunk once and reads the planes back from this per-SM cache
    const int kt = std::max((3 * D + 127) / 128, (H + 127) / 128);
    if (kt > kASlots) {
      b->a_cache_kt = kt;
      if ((st = b->alloc(b->a_cache, (size_t)kACacheSms * kt * kASlot))) return st;
    }
  }
  if ((st = b->alloc(b->part, (size_t)S * b->nsplit * 4 * sizeof(float4)))) return st;
  if (topk > 0 && ((st = b->alloc(b->topv, (size_t)S * b->nsplit * 4 * topk * 4)) ||
                   (st = b->alloc(b->topi, (size_t)S * b->nsplit * 4 * topk * 4))))
    return st;
  MC_CUDA(cudaMemsetAsync(b->pos, 0, S * 4, b->stream));
  MC_CUDA(cudaMemsetAsync(b->seglen, 0, S * 4, b->stream));
  MC_CUDA(cudaMemsetAsync(b->step, 0, 4, b->stream));
  MC_CUDA(cudaMemsetAsync(b->sel_done, 0, 4, b->stream));
  MC_CUDA(cudaMemsetAsync(b->latch, 0, (size_t)S * m->total_steps * D * 4, b->stream));
  std::vector<int32_t> id(S);
  for (int i = 0; i < S; ++i) id[i] = i;
  MC_CUDA(cudaMemcpyAsync(b->rowmap_id, id.data(), S * 4, cudaMemcpyHostToDevice, b->stream));
  MC_CUDA(cudaStreamSynchronize(b->stream));
  out = std::move(b);
  return kOk;
}

static void fill_common(const DevBatch& b, BlockArgs& a, int P) {
  const DevModel& m = *b.m;
  memset(&a, 0, sizeof(a));
  a.P = P;
  a.spt = std::max(1, 128 / P);
  a.n_sess = b.S;
  a.n_tiles = (b.S + a.spt - 1) / a.spt;
  a.pos0 = b.pos;
  a.seglen = b.seglen;
  a.tokens = P == 1 ? b.next_tok : b.tok;
  a.D = m.D;
  a.H = m.H;
  a.V = m.V;
  a.ring = m.ring;
  a.total_steps = m.total_steps;
  a.n_attn = m.n_attn;
  a.cache = m.cache;
  a.window = m.window;
  a.dh = m.heads > 0 ? m.D / m.heads : 0;
  a.embed = m.embed;
  a.embed_scale = m.embed_scale;
  a.latch_base = m.latch_base;
  a.final_gain = m.final_gain;
  a.norm_ring = b.norm_ring;
  a.latch = b.latch;
  a.kv = b.kv;
  a.cur = b.cur;
  a.blockin = b.blockin;
  a.xbuf = b.xbuf;
  a.hbuf = b.hbuf;
  a.qbuf = b.qbuf;
  a.att = b.att;
  a.att_rowmax = b.att_rowmax;
  a.fnorm = b.fnorm;
  a.fnorm_rowmax = b.fnorm_rowmax;
  a.kvlin = P > 1 ? b.kvlin : nullptr;
  a.a_cache = b.a_cache;
  a.a_cache_kt = b.a_cache_kt;
  a.a_cache_sms = kACacheSms;
}

static GemmSpec spec(const DevGemm& g, int type, int step) {
  GemmSpec s;
  s.tiles = g.tiles;
  s.K = g.K;
  s.ktiles = g.ktiles;
  s.nchunks = g.nchunks;
  s.type = type;
  s.step = step;
  s.scale = g.scale;
  return s;
}


// Launch profiler: when set, an event is recorded after every launch with the launch's kind
// (0 block, 1 attention, 2 final block, 3 head, 4 select, 5 step counter).
struct LaunchLog {
  std::vector<cudaEvent_t> ev;
  std::vector<int> kind;
  int record(cudaStream_t s, int k) {
    cudaEvent_t e;
    MC_CUDA(cudaEventCreate(&e));
    MC_CUDA(cudaEventRecord(e, s));
    ev.push_back(e);
    kind.push_back(k);
    return kOk;
  }
  ~LaunchLog() {
    for (auto e : ev) cudaEventDestroy(e);
  }
};

// Prepares a prefill from device-resident prompts: trims each prompt to the window, lays the
// segment out [S][P], resets positions and computes the head's row map. A one-row segment runs
// through the decode kernels, which read the token of each session from next_tok: P == 1 also
// writes it there.
__global__ void prepare_prompts_kernel(const int32_t* prompts, const int32_t* lens, int stride, int S, int P, int window,
                                       int32_t* tok, int32_t* seglen, int32_t* pos, int32_t* rowmap, int32_t* step,
                                       int32_t* next_tok) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s == 0) *step = 0;
  if (s >= S) return;
  const int L = max(0, min(lens[s], stride));
  const int n = min(min(L, window), P);
  const int32_t* src = prompts + (size_t)s * stride + (L - n);
  for (int i = 0; i < P; ++i) tok[(size_t)s * P + i] = i < n ? src[i] : 0;
  if (P == 1) next_tok[s] = n > 0 ? src[0] : 0;
  seglen[s] = n;
  pos[s] = 0;
  const int spt = max(1, 128 / P);
  rowmap[s] = (s / spt) * 128 + (s % spt) * P + max(n - 1, 0);
}

// The arguments of launch bi of one forward (the CA blocks, then bi = blocks: the final one) for
// P rows per session; *bs: rule steps of the blocks before bi (advanced past block bi).
static void build_block_args(const DevBatch& b, int P, int bi, bool fuse_head, int* bs, BlockArgs& a,
                             bool head_logits = false) {
  const DevModel& m = *b.m;
  const int nb = (int)m.blocks.size();
  fill_common(b, a, P);
  const bool final_k = bi == nb;
  int g = 0;
  if (bi > 0 && m.blocks[bi - 1].attn_slot >= 0) {
    a.has_out = 1;
    a.gemms[g++] = spec(m.blocks[bi - 1].out, kGOut, 0);
  }
  if (!final_k) {
    const DevBlock& blk = m.blocks[bi];
    a.block = bi;
    a.embed_first = bi == 0;
    a.residual = bi > 0;
    a.nsteps = blk.steps;
    a.bs0 = *bs;
    for (int st = 0; st < blk.steps; ++st) {
      a.dil[st] = blk.dil[st];
      a.gemms[g++] = spec(blk.wsel, kGWsel, st);
      a.gemms[g++] = spec(blk.w1, kGW1, st);
      a.gemms[g++] = spec(blk.w2, kGW2, st);
    }
    a.gamma = blk.gamma;
    a.b1 = blk.b1;
    a.b2 = blk.b2;
    if (blk.attn_slot >= 0) {
      a.has_attn = 1;
      a.attn_slot = blk.attn_slot;
      a.attn_norm = blk.attn_norm;
      a.gemms[g++] = spec(blk.qkv, kGQkv, 0);
    }
    *bs += blk.steps;
  } else {
    a.block = nb;
    a.embed_first = nb == 0;
    a.final_norm = 1;
    if (fuse_head && head_logits) {
      // the head runs inside the final decode launch and writes the logits (the policy selects)
      a.fuse_head = 1;
      a.gemms[g++] = spec(m.head, kGHead, 0);
      a.head_b = m.head_b;
      a.head_logits = b.logits;
    } else if (fuse_head) {
      // the greedy head and selection run inside the final decode launch
      a.fuse_head = 1;
      a.gemms[g++] = spec(m.head, kGHead, 0);
      a.head_b = m.head_b;
      a.next_tok = b.next_tok;
      a.out_tok = b.out_tok;
      a.out_prob = b.out_prob;
      a.out_stride = b.out_stride;
      a.pos_w = b.pos;
      a.step = b.step;
      a.done = b.sel_done;
      a.n_stops = b.n_stops;
      for (int k = 0; k < b.n_stops; ++k) a.stops[k] = b.stops[k];
      a.seglen_w = b.seglen;
      if (b.per_session) {
        a.gen_n = b.gen_n;
        a.limit = b.limit;
      }
    }
  }
  a.ngemms = g;
  a.trace = b.trace ? b.trace + 64 * bi : nullptr;
  a.trace_fine = getenv("MC_TRACE_FINE") != nullptr;
  if (P == 1 && b.decode_kernel) {
    // the decode kernel reads W1 and W2 in split-pair tiles
    for (int i = 0; i < a.ngemms; ++i) {
      if (a.gemms[i].type == kGW1) a.gemms[i] = spec(m.blocks[bi].w1d, kGW1, a.gemms[i].step);
      if (a.gemms[i].type == kGW2) a.gemms[i] = spec(m.blocks[bi].w2d, kGW2, a.gemms[i].step);
    }
    a.dec_kt = m.dec_kt;
  }
}

// A prefill pass over the contiguous tiles [t0, t0 + nt) (sessions [s0, s0 + ns)) of a batch
// whose scratch holds fewer rows than a whole prefill needs. The kernels index scratch rows by
// the global row (tile * 128 + r) and a segment's keys/values by the session: the pass hands
// them those bases moved back by its first row and first session, so the rows it touches are
// the first nt * 128 of the buffers.
struct PassRange {
  int t0 = 0, nt = 0, s0 = 0, ns = 0;
};

template <class T>
static T* rows_back(T* p, size_t n) {
  return p ? reinterpret_cast<T*>(reinterpret_cast<uintptr_t>(p) - n * sizeof(T)) : p;
}

// Tiles of 128 rows a segment of P rows per session takes for the batch's sessions.
static int segment_tiles(const DevBatch& b, int P) {
  const int spt = std::max(1, 128 / P);
  return (b.S + spt - 1) / spt;
}

// Enqueues the blocks (and attention sublayers) of one segment: P rows per session, P = 1 a decode
// step; ends with the final RMSNorm of every row. pr: a prefill pass over some tiles (null: all).
// last_only: the caller reads each session's last row only (its head); the last block's attention
// then runs only the last query of each prompt segment when that block is the model's last (every
// other position's output would only feed rows nothing reads).
static int enqueue_layers(DevBatch& b, int P, LaunchLog* log, bool fuse_head = false, const PassRange* pr = nullptr,
                          bool head_logits = false, bool last_only = false) {
  const DevModel& m = *b.m;
  cudaStream_t s = b.stream;
  const int nb = (int)m.blocks.size();
  if (P > 1 && !pr && (size_t)segment_tiles(b, P) * 128 > b.rows)
    return set_error(kUnsupported, "prefill rows exceed the batch's scratch (a pass over a tile list needs them all)");
  const size_t row0 = pr ? (size_t)pr->t0 * 128 : 0, kv0 = pr ? (size_t)pr->s0 * P : 0;
  int bs = 0;
  for (int bi = 0; bi <= nb; ++bi) {
    BlockArgs a;
    build_block_args(b, P, bi, fuse_head, &bs, a, head_logits);
    if (pr) {
      a.tile0 = pr->t0;
      a.cur = rows_back(a.cur, row0 * m.D);
      a.blockin = rows_back(a.blockin, row0 * m.D);
      a.xbuf = rows_back(a.xbuf, row0 * 3 * m.D);
      a.hbuf = rows_back(a.hbuf, row0 * m.H);
      a.qbuf = rows_back(a.qbuf, row0 * m.D);
      a.att = rows_back(a.att, row0 * m.D);
      a.att_rowmax = rows_back(a.att_rowmax, row0);
      a.fnorm = rows_back(a.fnorm, row0 * m.D);
      a.fnorm_rowmax = rows_back(a.fnorm_rowmax, row0);
      a.kvlin = rows_back(a.kvlin, kv0 * 2 * m.D);
    }
    const bool final_k = bi == nb;
    if (P == 1 && b.decode_kernel) {
      const int grid = (b.S + m.dec_r - 1) / m.dec_r;
      const int kf = (m.D + 127) / 128;
      void (*kern)(BlockArgs);
      if (m.dec_r == 32) kern = kf == 1 ? block_decode_kernel<1, 32, 6> : kf == 2 ? block_decode_kernel<2, 32, 6> : block_decode_kernel<3, 32, 6>;
      else kern = kf == 1 ? block_decode_kernel<1, 16, 3> : kf == 2 ? block_decode_kernel<2, 16, 3> : block_decode_kernel<3, 16, 3>;
      kern<<<grid, kDThreads, m.dec_smem, s>>>(a);
    } else {
      int grid = pr ? pr->nt : a.n_tiles;
      if (b.n_pass_tiles > 0) {
        a.tile_list = b.pass_tiles;
        grid = b.n_pass_tiles;
      }
      switch ((m.D + 127) / 128) {
        case 1: (a.a_cache ? block_kernel<1, true> : block_kernel<1, false>)<<<grid, kBlockThreads, kBlockSmem, s>>>(a); break;
        case 2: (a.a_cache ? block_kernel<2, true> : block_kernel<2, false>)<<<grid, kBlockThreads, kBlockSmem, s>>>(a); break;
        default: (a.a_cache ? block_kernel<3, true> : block_kernel<3, false>)<<<grid, kBlockThreads, kBlockSmem, s>>>(a); break;
      }
    }
    MC_CUDA(cudaGetLastError());
    if (log) log->record(s, final_k ? 2 : 0);
    if (!final_k && m.blocks[bi].attn_slot >= 0) {
      AttnArgs aa;
      memset(&aa, 0, sizeof(aa));
      aa.n_sess = b.S;
      aa.D = m.D;
      aa.heads = m.heads;
      aa.dh = m.D / m.heads;
      aa.cache = m.cache;
      aa.window = m.window;
      aa.n_attn = m.n_attn;
      aa.attn_slot = m.blocks[bi].attn_slot;
      aa.P = P;
      aa.spt = a.spt;
      aa.pos0 = b.pos;
      aa.seglen = b.seglen;
      aa.qbuf = b.qbuf;
      aa.kv = b.kv;
      aa.kvlin = b.kvlin;
      aa.att = b.att;
      aa.att_rowmax = b.att_rowmax;
      aa.scale = (float)(1.0 / std::sqrt((double)aa.dh));
      const AttnStaging stg = attn_staging(m.cache, aa.dh);
      if (P == 1 && stg.warps > 0 && stg.smem <= kAsSmemMax && (long long)b.S * m.heads < (1LL << 31)) {
        const long long items = (long long)b.S * m.heads;
        const int grid = (int)std::min<long long>((items + stg.warps - 1) / stg.warps, b.n_sm);
        const int threads = stg.warps * 32;
        void (*kern)(AttnArgs);
        switch (aa.dh) {
          case 4: kern = attn_decode_staged_kernel<4>; break;
          case 8: kern = attn_decode_staged_kernel<8>; break;
          case 16: kern = attn_decode_staged_kernel<16>; break;
          case 32: kern = attn_decode_staged_kernel<32>; break;
          case 48: kern = attn_decode_staged_kernel<48>; break;
          default: kern = attn_decode_staged_kernel<64>; break;
        }
        kern<<<grid, threads, stg.smem, s>>>(aa);
      } else if (P == 1) {
        const long long warps = (long long)b.S * m.heads;
        const int grid = (int)((warps * 32 + kAttnThreads - 1) / kAttnThreads);
        switch (aa.dh) {
          case 32: attn_decode_kernel<32><<<grid, kAttnThreads, 0, s>>>(aa); break;
          case 48: attn_decode_kernel<48><<<grid, kAttnThreads, 0, s>>>(aa); break;
          case 64: attn_decode_kernel<64><<<grid, kAttnThreads, 0, s>>>(aa); break;
          default: attn_decode_kernel<0><<<grid, kAttnThreads, 0, s>>>(aa); break;
        }
      } else {
        int grid = b.S;
        if (pr) {
          aa.sess0 = pr->s0;
          grid = pr->ns;
          aa.qbuf = rows_back(aa.qbuf, row0 * m.D);
          aa.att = rows_back(aa.att, row0 * m.D);
          aa.att_rowmax = rows_back(aa.att_rowmax, row0);
          aa.kvlin = rows_back(aa.kvlin, kv0 * 2 * m.D);
        }
        if (b.n_pass_sess > 0) {
          aa.sess_list = b.pass_sess;
          grid = b.n_pass_sess;
        }
        if (attn_prefill_fast_ok(aa.dh) && attn_prefill_fast_smem(P, m.D) <= 220 * 1024) {
          const size_t smem = attn_prefill_fast_smem(P, m.D);
          aa.last_only = last_only && bi == nb - 1 && !getenv("MC_PREFILL_ALL_QUERIES") ? 1 : 0;
          switch (aa.dh) {
            case 4: attn_prefill_fast_kernel<4><<<grid, kAttnThreads, smem, s>>>(aa); break;
            case 8: attn_prefill_fast_kernel<8><<<grid, kAttnThreads, smem, s>>>(aa); break;
            case 16: attn_prefill_fast_kernel<16><<<grid, kAttnThreads, smem, s>>>(aa); break;
            case 32: attn_prefill_fast_kernel<32><<<grid, kAttnThreads, smem, s>>>(aa); break;
            case 48: attn_prefill_fast_kernel<48><<<grid, kAttnThreads, smem, s>>>(aa); break;
            default: attn_prefill_fast_kernel<64><<<grid, kAttnThreads, smem, s>>>(aa); break;
          }
        } else {
          const size_t smem = (size_t)P * 2 * m.D * 4 + 32 * 4 + 16 + 128;
          if (smem > 220 * 1024) return set_error(kUnsupported, "prefill segment too long for the attention kernel");
          attn_prefill_kernel<<<grid, kAttnThreads, smem, s>>>(aa);
        }
      }
      MC_CUDA(cudaGetLastError());
      if (log) log->record(s, 1);
    }
  }
  return kOk;
}

// The head over the final-normed rows of sessions [s0, s0 + ns) of one pass (its scratch rows
// start at row0), with the selection partials of those sessions.
// Sampling (mode 1) takes its top-k candidates from the materialised logits, selected per row
// by select_kernel, when the batch holds a logits buffer and the vocabulary fits the select's
// shared memory (else from the head's per-partial top-k lists).
static bool select_from_logits(const DevBatch& b, int mode) {
  return mode == 1 && b.topk > 1 && b.logits != nullptr;
}

// The head's 32-column group maxima serve the select's bound when there are enough groups for
// the top-k (4 per 128-column chunk, at most kSelSamples): their count, or 0.
static int head_groups(const DevBatch& b) {
  const int g = 4 * b.m->head.nchunks;
  return b.gmax && g <= kSelSamples && (b.m->V + 31) / 32 > b.topk ? g : 0;
}

static int enqueue_head(DevBatch& b, int P, int mode, bool want_logits, int s0, int ns, size_t row0, LaunchLog* log) {
  const DevModel& m = *b.m;
  const bool sel_logits = select_from_logits(b, mode);
  HeadArgs h;
  memset(&h, 0, sizeof(h));
  h.n_sess = ns;
  h.D = m.D;
  h.V = m.V;
  h.nsplit = b.nsplit;
  h.nchunks = m.head.nchunks;
  h.cps = (m.head.nchunks + b.nsplit - 1) / b.nsplit;
  h.ktiles = m.head.ktiles;
  h.rowmap = (P == 1 ? b.rowmap_id : b.rowmap) + s0;
  h.fnorm = rows_back(b.fnorm, row0 * m.D);
  h.fnorm_rowmax = rows_back(b.fnorm_rowmax, row0);
  h.tiles = m.head.tiles;
  h.scale = m.head.scale;
  h.head_b = m.head_b;
  h.topk = mode == 1 && !sel_logits ? b.topk : 0;
  h.target = mode == 2 ? b.target + s0 : nullptr;
  h.logits_out = want_logits || mode == 3 || sel_logits ? b.logits + (size_t)s0 * m.V : nullptr;
  h.logits_only = mode == 3 ? 1 : 0;  // the policy kernel reads the logits, not the partials
  if (sel_logits && head_groups(b) > 0) {
    h.ngroups = head_groups(b);
    h.gmax_out = b.gmax + (size_t)s0 * h.ngroups;
  }
  const size_t np = (size_t)b.nsplit * 4;  // partials per session: splits x column quarters
  h.part = b.part + (size_t)s0 * np;
  h.topv = b.topv ? b.topv + (size_t)s0 * np * b.topk : nullptr;
  h.topi = b.topi ? b.topi + (size_t)s0 * np * b.topk : nullptr;
  dim3 hg((ns + 127) / 128, b.nsplit);
  head_kernel<<<hg, kHeadThreads, kHeadSmem, b.stream>>>(h);
  MC_CUDA(cudaGetLastError());
  if (log) log->record(b.stream, 3);
  return kOk;
}

// The selection of sessions [s0, s0 + ns); bump: this launch advances the step counter (the last
// selection of a step).
static int enqueue_select(DevBatch& b, int mode, double inv_temp, uint32_t session0, bool advance_from_len, int s0,
                          int ns, bool bump, LaunchLog* log) {
  const size_t np = (size_t)b.nsplit * 4;
  SelectArgs sa;
  memset(&sa, 0, sizeof(sa));
  sa.n_sess = ns;
  sa.nsplit = (int)np;
  sa.topk = b.topk;
  sa.mode = mode;
  sa.inv_temp = inv_temp;
  sa.session0 = session0 + (uint32_t)s0;
  sa.part = b.part + (size_t)s0 * np;
  sa.topv = b.topv ? b.topv + (size_t)s0 * np * b.topk : nullptr;
  sa.topi = b.topi ? b.topi + (size_t)s0 * np * b.topk : nullptr;
  sa.step = b.step;
  sa.out_stride = b.out_stride;
  sa.next_tok = b.next_tok + s0;
  sa.out_tok = b.out_tok ? b.out_tok + (size_t)s0 * b.out_stride : nullptr;
  sa.out_prob = b.out_prob ? b.out_prob + (size_t)s0 * b.out_stride : nullptr;
  sa.out_logprob = b.out_logprob ? b.out_logprob + (size_t)s0 * b.out_stride : nullptr;
  sa.pos = b.pos + s0;
  sa.seglen = b.seglen + s0;
  sa.advance_from_len = advance_from_len ? 1 : 0;
  sa.done = bump ? b.sel_done : nullptr;  // the last block of that launch advances the step counter
  sa.n_stops = b.n_stops;
  if (b.per_session) {
    sa.gen_n = b.gen_n + s0;
    sa.limit = b.limit ? b.limit + s0 : nullptr;
  }
  for (int k = 0; k < b.n_stops; ++k) sa.stops[k] = b.stops[k];
  if (select_from_logits(b, mode)) {
    sa.logits = b.logits + (size_t)s0 * b.m->V;
    sa.V = b.m->V;
    if (head_groups(b) > 0) {
      sa.ngroups = head_groups(b);
      sa.gmax = b.gmax + (size_t)s0 * sa.ngroups;
    }
  }
  select_kernel<<<(ns + kSelectWarps - 1) / kSelectWarps, kSelectWarps * 32, 0, b.stream>>>(sa);
  MC_CUDA(cudaGetLastError());
  if (log) log->record(b.stream, 4);
  return kOk;
}

// A greedy job (the prompts of upload_prompts / prepare_prompts_kernel, then n_new tokens) on
// tiny_generate_kernel, when the batch's model has its tiny weights and the job is plain greedy
// decoding of a batch of at most two CTAs per multiprocessor (MC_TINY_OFF=1: the batched kernels).
bool tiny_job_ok(const DevBatch& b, int mode, int n_stops, bool limits, bool policy) {
  return b.m->tiny && mode == 0 && n_stops == 0 && !limits && !policy && b.S <= 2 * b.n_sm && !getenv("MC_TINY_OFF");
}

// The whole job (P-token prompt segments, n_new tokens) or, with append, one pending token per
// session (next_tok at pos, the batched step's state convention) and optionally the logits rows.
int launch_tiny_job(DevBatch& b, int P, int n_new, bool append = false, float* logits = nullptr) {
  const DevModel& m = *b.m;
  TinyArgs a;
  memset(&a, 0, sizeof(a));
  a.S = b.S;
  a.D = m.D;
  a.H = m.H;
  a.V = m.V;
  a.nblocks = (int)m.blocks.size();
  a.total_steps = m.total_steps;
  a.ring = m.ring;
  a.P = P;
  a.n_new = n_new;
  a.out_stride = b.out_stride;
  a.kw_sel = tiny_stride_words(m.D);
  a.kw1 = tiny_stride_words(3 * m.D);
  a.kw2 = tiny_stride_words(m.H);
  a.blk_words = m.tiny_blk_words;
  a.embed = m.embed;
  a.embed_scale = m.embed_scale;
  a.head_scale = m.head.scale;
  a.head_b = m.head_b;
  a.final_gain = m.final_gain;
  a.latch_base = m.latch_base;
  a.tok = b.tok;
  a.seglen = b.seglen;
  a.pos = b.pos;
  a.next_tok = b.next_tok;
  a.step = b.step;
  a.latch = b.latch;
  a.norm_ring = b.norm_ring;
  a.out_tok = b.out_tok;
  a.out_prob = b.out_prob;
  a.append = append ? 1 : 0;
  a.logits = logits;
  int bs = 0;
  for (int bi = 0; bi < a.nblocks; ++bi) {
    const DevBlock& blk = m.blocks[bi];
    TinyBlock& t = a.blk[bi];
    t.w = m.tiny_w + (size_t)bi * m.tiny_blk_words;
    t.s_sel = blk.wsel.scale;
    t.s1 = blk.w1.scale;
    t.s2 = blk.w2.scale;
    t.b1 = blk.b1;
    t.b2 = blk.b2;
    t.gamma = blk.gamma;
    t.steps = blk.steps;
    t.bs0 = bs;
    for (int st = 0; st < blk.steps; ++st) t.dil[st] = blk.dil[st];
    bs += blk.steps;
  }
  tiny_generate_kernel<<<b.S, kTinyThreads, m.tiny_smem, b.stream>>>(a);
  MC_CUDA(cudaGetLastError());
  return kOk;
}

int enqueue_forward(DevBatch& b, int P, int mode, double inv_temp, uint32_t session0, bool want_logits,
                    bool advance_from_len, LaunchLog* log = nullptr) {
  const DevModel& m = *b.m;
  cudaStream_t s = b.stream;
  // greedy decode steps without logits: the head and the selection are fused into the final
  // decode launch
  const bool fuse = P == 1 && b.decode_kernel && mode == 0 && !want_logits && !getenv("MC_NO_FUSED_HEAD");
  // decode steps under the policy: the head fused into the final decode launch writes the logits
  const bool fuse_logits = P == 1 && b.decode_kernel && mode == 3 && !getenv("MC_NO_FUSED_HEAD");
  int st;
  const int total = segment_tiles(b, P);
  const int per = (int)(b.rows / 128);
  if (P > 1 && b.n_pass_tiles == 0 && total > per) {
    // a prefill larger than the scratch: passes over contiguous tiles, each through the head and
    // the selection of its sessions (the policy runs once, over the logits of all of them)
    const int spt = std::max(1, 128 / P);
    for (int t0 = 0; t0 < total; t0 += per) {
      PassRange pr;
      pr.t0 = t0;
      pr.nt = std::min(per, total - t0);
      pr.s0 = t0 * spt;
      pr.ns = std::min(b.S, (t0 + pr.nt) * spt) - pr.s0;
      if ((st = enqueue_layers(b, P, log, false, &pr, false, true)) != kOk) return st;
      if ((st = enqueue_head(b, P, mode, want_logits, pr.s0, pr.ns, (size_t)t0 * 128, log)) != kOk) return st;
      if (mode != 3 && (st = enqueue_select(b, mode, inv_temp, session0, advance_from_len, pr.s0, pr.ns,
                                            t0 + pr.nt >= total, log)) != kOk)
        return st;
    }
  } else {
    if ((st = enqueue_layers(b, P, log, fuse || fuse_logits, nullptr, fuse_logits, true)) != kOk) return st;
    if (fuse) return kOk;
    if (!fuse_logits && (st = enqueue_head(b, P, mode, want_logits, 0, b.S, 0, log)) != kOk) return st;
    if (mode != 3) return enqueue_select(b, mode, inv_temp, session0, advance_from_len, 0, b.S, true, log);
  }
  if (mode != 3) return kOk;
  // the whole decode-loop policy over the materialised logits; the generated tokens so far are
  // the first *step columns of out_tok
  PolicyArgs pa;
  memset(&pa, 0, sizeof(pa));
  pa.n_rows = b.S;
  pa.V = m.V;
  pa.logits = b.logits;
  pa.temperature = b.pol.temperature;
  pa.rep_penalty = b.pol.rep_penalty;
  pa.top_p = b.pol.top_p;
  pa.top_k = b.pol.top_k;
  pa.rep_window = b.pol.rep_window;
  pa.ban_trigrams = b.pol.ban_trigrams;
  pa.prefix = b.pol_prefix;
  pa.prefix_len = b.pol_prefix_len;
  pa.prefix_stride = b.pol_prefix_cap;
  pa.gen = b.out_tok;
  pa.gen_stride = b.out_stride;
  pa.dfa = b.pol.dfa;
  pa.dfa_state = b.pol.dfa ? b.pol_state : nullptr;
  pa.session0 = session0;
  pa.step = b.step;
  if (b.per_session) {
    pa.gen_n = b.gen_n;
    pa.limit = b.limit;
    pa.key = b.key;
  }
  pa.out_stride = b.out_stride;
  pa.next_tok = b.next_tok;
  pa.out_tok = b.out_tok;
  pa.out_prob = b.out_prob;
  pa.pos = b.pos;
  pa.seglen = b.seglen;
  pa.advance_from_len = advance_from_len ? 1 : 0;
  pa.done = b.sel_done;
  pa.n_stops = b.n_stops;
  for (int k = 0; k < b.n_stops; ++k) pa.stops[k] = b.stops[k];
  if ((st = launch_policy(pa, s)) != kOk) return st;
  if (log) log->record(s, 4);
  return kOk;
}

// Scoring rows: every row of the last segment goes through the head with the next token of its
// sequence as target; select_kernel writes logProb (internal/eval/suite.go:201-209) per row.
int ensure_score_rows(DevBatch& b, size_t rows) {
  if (rows <= b.sc_rows) return kOk;
  const DevModel& m = *b.m;
  // at most 16 chunks per CTA (the head kernel stages their biases in shared memory)
  b.sc_nsplit = std::max(1, (m.head.nchunks + 15) / 16);
  int st;
  if ((st = b.alloc(b.sc_rowmap, rows * 4)) || (st = b.alloc(b.sc_target, rows * 4)) ||
      (st = b.alloc(b.sc_valid, rows * 4)) || (st = b.alloc(b.sc_next, rows * 4)) ||
      (st = b.alloc(b.sc_part, rows * b.sc_nsplit * 4 * sizeof(float4))) || (st = b.alloc(b.sc_logprob, rows * 8)))
    return st;
  b.sc_rows = rows;
  return kOk;
}

// The forward pass of a prompt segment (P rows per session) and the log-probability of every
// row's target: sc_logprob[r] for the rows r with sc_valid[r] != 0 (r = session * P + t). A segment
// larger than the batch's scratch runs in passes over contiguous sessions, each scored at once.
int enqueue_score(DevBatch& b, int P, size_t rows) {
  const DevModel& m = *b.m;
  cudaStream_t s = b.stream;
  const int total = segment_tiles(b, P), per = (int)(b.rows / 128);
  const int spt = std::max(1, 128 / P);
  for (int t0 = 0; t0 < total; t0 += per) {
    PassRange pr;
    pr.t0 = t0;
    pr.nt = std::min(per, total - t0);
    pr.s0 = t0 * spt;
    pr.ns = std::min(b.S, (t0 + pr.nt) * spt) - pr.s0;
    const bool whole = pr.nt == total;
    int st = enqueue_layers(b, P, nullptr, false, whole ? nullptr : &pr);
    if (st != kOk) return st;
    const size_t r0 = (size_t)pr.s0 * P, nr = std::min(rows, (size_t)(pr.s0 + pr.ns) * P) - r0;
    const size_t row0 = whole ? 0 : (size_t)t0 * 128;
    HeadArgs h;
    memset(&h, 0, sizeof(h));
    h.n_sess = (int)nr;
    h.D = m.D;
    h.V = m.V;
    h.nsplit = b.sc_nsplit;
    h.nchunks = m.head.nchunks;
    h.cps = (m.head.nchunks + b.sc_nsplit - 1) / b.sc_nsplit;
    h.ktiles = m.head.ktiles;
    h.rowmap = b.sc_rowmap + r0;
    h.fnorm = rows_back(b.fnorm, row0 * m.D);
    h.fnorm_rowmax = rows_back(b.fnorm_rowmax, row0);
    h.tiles = m.head.tiles;
    h.scale = m.head.scale;
    h.head_b = m.head_b;
    h.target = b.sc_target + r0;
    h.part = b.sc_part + r0 * b.sc_nsplit * 4;
    dim3 hg((unsigned)((nr + 127) / 128), b.sc_nsplit);
    head_kernel<<<hg, kHeadThreads, kHeadSmem, s>>>(h);
    MC_CUDA(cudaGetLastError());
    SelectArgs sa;
    memset(&sa, 0, sizeof(sa));
    sa.n_sess = (int)nr;
    sa.nsplit = b.sc_nsplit * 4;
    sa.mode = 2;
    sa.part = b.sc_part + r0 * b.sc_nsplit * 4;
    sa.out_stride = 1;
    sa.next_tok = b.sc_next + r0;
    sa.out_logprob = b.sc_logprob + r0;
    sa.seglen = b.sc_valid + r0;  // rows without a target are skipped
    select_kernel<<<(unsigned)((nr + kSelectWarps - 1) / kSelectWarps), kSelectWarps * 32, 0, s>>>(sa);
    MC_CUDA(cudaGetLastError());
  }
  return kOk;
}

}  // namespace eng
}  // namespace mc
