// Output head and token selection.
//
// head_kernel: logits = E c s_e + head_b for the final-normed state c of each session
// (headLogits, internal/quant/stream.go:233-248; tied head = the embedding, convert.go:77-83),
// on the tensor core with the vocabulary split across CTAs. The epilogue never materialises the
// logits unless asked: it keeps, per row and split, the running max, its first index, the sum of
// exp(l - max), the logit of a scoring target and (for sampling) the split's top-k logits.
//
// select_kernel merges the splits of each row:
//   greedy  argmaxProb (internal/generate/greedy.go:90-102): first index of the max,
//           probability 1 / sum exp(l - max);
//   sample  the truncated branch of SampleRawLogitsAdvanced (generate/sample.go:91-172) with
//           sampleFromCDF (:174-191): top-k of l/T, weights exp(l/T - max), a draw u from
//           Philox4x32-10 keyed by the session (the reference draws from Go's math/rand);
//   score   logProb (internal/eval/suite.go:201-209): l[target] - max - log(sum exp(l - max)).
#include "mc_engine.cuh"

namespace mc {
namespace eng {

constexpr int kMaxTopK = 64;

struct HeadArgs {
  int n_sess, D, V, nsplit, cps, ktiles, nchunks;
  const int32_t* rowmap;   // [S] scratch row of each session's final state
  const float* fnorm;
  const float* fnorm_rowmax;
  const uint8_t* tiles;
  float scale;
  const float* head_b;
  int topk;                // 0: no top-k lists
  const int32_t* target;   // [S] or null
  float* logits_out;       // [S][V] or null
  int logits_only;         // with logits_out: no partials (the policy kernel reads the logits only)
  float* gmax_out;         // [S][ngroups] or null: the row's maximum over each 32-column piece
  int ngroups;             // (column quarter h of chunk c is group 4c + h)
  float4* part;            // [S][nsplit]: max, sum, first argmax (bits), target logit
  float* topv;             // [S][nsplit][topk]
  int32_t* topi;
};

constexpr int kHeadRowThreads = 512;  // four threads per row, each a quarter of every chunk's columns
constexpr int kHeadRowWarps = kHeadRowThreads / 32;
constexpr int kHeadThreads = kHeadRowThreads + 64;
constexpr int kHeadMmaWarp = kHeadRowWarps, kHeadProducerWarp = kHeadRowWarps + 1;
constexpr int kHeadSmemA = kASlots * kASlot;
constexpr int kHeadSmemB = kBStages * kTile;
constexpr int kHeadMaxBias = 16 * 128;  // biases of at most 16 chunks per CTA
constexpr int kHeadSmem = kHeadSmemA + kHeadSmemB + 1024 + 12288;

struct HeadBars {
  uint64_t a_full, b_full[kBStages], b_empty[kBStages], acc_full, acc_empty;
  uint32_t tmem;
  int rrow[kRows];
  int rvalid[kRows];
  float rmax[kRows];
  float bias[kHeadMaxBias];
};
static_assert(sizeof(HeadBars) <= 12288, "head barrier block");

// Partials: per session, nsplit x 4 entries (split, column quarter), each (max, sum exp(l - max),
// first argmax as int bits, target logit or 0); top-k lists likewise per (split, quarter).
__global__ void __launch_bounds__(kHeadThreads, 1) head_kernel(const __grid_constant__ HeadArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kHeadSmemA;
  HeadBars* bars = reinterpret_cast<HeadBars*>(sB + kHeadSmemB);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int mtile = blockIdx.x, split = blockIdx.y;
  const int c0 = split * a.cps, c1 = min(c0 + a.cps, a.nchunks);

  if (threadIdx.x == 0) {
    mbar_init(&bars->a_full, kHeadRowThreads);
    for (int i = 0; i < kBStages; ++i) {
      mbar_init(&bars->b_full[i], 1);
      mbar_init(&bars->b_empty[i], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, kHeadRowThreads);
    fence_barrier_init();
  }
  if (warp == kHeadMmaWarp) tmem_alloc(&bars->tmem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;

  if (warp == kHeadProducerWarp) {
    if (lane == 0) {
      uint32_t bidx = 0;
      for (int c = c0; c < c1; ++c)
        for (int kt = 0; kt < a.ktiles; ++kt, ++bidx) {
          const int st = bidx % kBStages;
          if (bidx >= kBStages && !mbar_wait_or_abort(&bars->b_empty[st], ((bidx / kBStages) - 1) & 1, kErrWaitEmpty))
            goto producer_done;
          mbar_arrive_expect_tx(&bars->b_full[st], kTile);
          bulk_load(sB + st * kTile, a.tiles + ((size_t)c * a.ktiles + kt) * kTile, kTile, &bars->b_full[st]);
        }
    producer_done:;
    }
  } else if (warp == kHeadMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(kRows, kNC);
      uint32_t bidx = 0;
      bool ok = mbar_wait_or_abort(&bars->a_full, 0, kErrWaitFull);
      for (int c = c0; c < c1 && ok; ++c) {
        const int ci = c - c0;
        if (ci > 0 && !mbar_wait_or_abort(&bars->acc_empty, (ci - 1) & 1, kErrWaitAccFree)) break;
        tc_fence_after();
        for (int kt = 0; kt < a.ktiles; ++kt, ++bidx) {
          const int st = bidx % kBStages;
          if (!mbar_wait_or_abort(&bars->b_full[st], (bidx / kBStages) & 1, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t db = smem_desc_sw128(sB + st * kTile);
          const int ksteps = min(4, (a.D - kt * 128 + 31) / 32);
#pragma unroll
          for (int p = 0; p < 3; ++p) {
            const uint64_t da = smem_desc_sw128(sA + kt * kASlot + p * kTile);
            for (int kk = 0; kk < ksteps; ++kk)
              mma_i8(tmem + p * kNC, da + 2 * kk, db + 2 * kk, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&bars->b_empty[st]);
        }
        if (!ok) break;
        mma_commit(&bars->acc_full);
      }
    }
  } else {
    const int t = threadIdx.x;
    const int r = t & (kRows - 1), h = t >> 7;
    const int s = mtile * kRows + r;
    const bool valid = s < a.n_sess;
    if (h == 0) {
      const int gr = valid ? a.rowmap[s] : 0;
      bars->rrow[r] = gr;
      bars->rvalid[r] = valid ? 1 : 0;
      bars->rmax[r] = valid ? a.fnorm_rowmax[gr] : 0.f;
    }
    for (int i = t; i < (c1 - c0) * kNC && i < kHeadMaxBias; i += kHeadRowThreads) {
      const int v = c0 * kNC + i;
      bars->bias[i] = v < a.V ? a.head_b[v] : 0.f;
    }
    asm volatile("bar.sync 1, 512;" ::: "memory");
    // operand: the final-normed rows, sliced warp-per-row (all rows of a warp in flight together)
    for (int kt = 0; kt < a.ktiles; ++kt) {
      float4 v[kRows / kHeadRowWarps];
      const int e = kt * 128 + 4 * lane;
#pragma unroll
      for (int u = 0; u < kRows / kHeadRowWarps; ++u) {
        const int rr = warp + kHeadRowWarps * u;
        v[u] = ld4_or0(a.fnorm + (size_t)bars->rrow[rr] * a.D, e, a.D, bars->rvalid[rr] != 0);
      }
#pragma unroll
      for (int u = 0; u < kRows / kHeadRowWarps; ++u) {
        const int rr = warp + kHeadRowWarps * u;
        put4(sA, rr, e, v[u], row_inv_step(bars->rmax[rr]));
      }
    }
    fence_proxy_async_smem();
    mbar_arrive(&bars->a_full);

    const float step = row_step(bars->rmax[r]);
    float m = -INFINITY, sum = 0.f, lt = 0.f;
    int idx = 0;
    const int tgt = (valid && a.target) ? a.target[s] : -1;
    const int pi = split * 4 + h;  // this thread's partial
    const int npart = a.nsplit * 4;
    float* tv = nullptr;
    int32_t* ti = nullptr;
    float thresh = -INFINITY;
    if (valid && a.topk > 0) {
      tv = a.topv + ((size_t)s * npart + pi) * a.topk;
      ti = a.topi + ((size_t)s * npart + pi) * a.topk;
      for (int i = 0; i < a.topk; ++i) {
        tv[i] = -INFINITY;
        ti[i] = 0x7fffffff;
      }
    }
    bool ok = true;
    for (int c = c0; c < c1; ++c) {
      const int ci = c - c0;
      const bool got = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&bars->acc_full, ci & 1, kErrWaitAcc));
      if (!got) ok = false;
      if (ok) {
        tc_fence_after();
        float qm = -INFINITY;  // this thread's 32 columns of the chunk: one group maximum
        for (int j0 = h * 32; j0 < h * 32 + 32; j0 += 16) {
          uint32_t a1[16], a2[16], a3[16];
          load_acc16(tmem, warp, j0, a1, a2, a3);
          if (!valid) continue;
          float l16[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            l16[j] = __fadd_rn(dequant(a1[j], a2[j], a3[j], step, a.scale), bars->bias[ci * kNC + j0 + j]);
          const int v0 = c * kNC + j0;
          if (a.logits_out) st16(a.logits_out + (size_t)s * a.V, v0, a.V, l16);
          if (a.logits_only) continue;
          // chunk-local max first, then one rescale of the running sum
          float cm = -INFINITY;
          int ci2 = 0;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (v0 + j < a.V && l16[j] > cm) {
              cm = l16[j];
              ci2 = v0 + j;
            }
          qm = fmaxf(qm, cm);
          if (cm > m) {
            sum = __fmul_rn(sum, expf(m - cm));
            m = cm;
            idx = ci2;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (v0 + j < a.V) sum = __fadd_rn(sum, expf(l16[j] - m));
          if (tgt >= v0 && tgt < v0 + 16) lt = l16[tgt - v0];
          if (tv) {
            for (int j = 0; j < 16; ++j) {
              const float l = l16[j];
              if (v0 + j >= a.V || !(l > thresh)) continue;
              int i = a.topk - 1;
              while (i > 0 && tv[i - 1] < l) {
                tv[i] = tv[i - 1];
                ti[i] = ti[i - 1];
                --i;
              }
              tv[i] = l;
              ti[i] = v0 + j;
              thresh = tv[a.topk - 1];
            }
          }
        }
        if (valid && a.gmax_out) a.gmax_out[(size_t)s * a.ngroups + 4 * c + h] = qm;
      }
      tc_fence_before();
      mbar_arrive(&bars->acc_empty);
    }
    if (valid && !a.logits_only) a.part[(size_t)s * npart + pi] = make_float4(m, sum, __int_as_float(idx), lt);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kHeadMmaWarp) tmem_dealloc(tmem, 512);
}

struct SelectArgs {
  int n_sess, nsplit, topk, mode;  // mode: 0 greedy, 1 sample, 2 score
  double inv_temp;
  uint32_t session0;               // global index of session 0 (Philox key)
  const float4* part;
  const float* topv;
  const int32_t* topi;
  int32_t* step;                   // device step counter (output column, Philox counter)
  int out_stride;                  // columns of the output arrays
  int32_t* next_tok;               // [S] input of the next decode step
  int32_t* out_tok;                // [S][out_stride] or null
  float* out_prob;                 // [S][out_stride] or null
  double* out_logprob;             // [S][out_stride] or null (score mode)
  int32_t* pos;                    // [S] positions, advanced by `advance` (0 = no change)
  int32_t* seglen;                 // [S] set to 1 for the next decode step when advancing
  int advance_from_len;            // 1: pos = pos0 + seglen (after a prefill); 0: pos += 1
  int32_t* done;                   // finished-block counter (zero between launches); null: no step bump
  int n_stops;                     // a chosen token among stops[0..n_stops) ends the session: no output,
  int stops[kMaxStops];            // seglen = 0 (greedyLoop's stop tokens, generate/greedy.go:75-77)
  int32_t* gen_n;                  // [S] tokens each session has emitted (its output column), or null: step
  const int32_t* limit;            // [S] tokens a session may emit (it ends after the last), with gen_n
  const float* logits;             // [S][V] sampling: the top-k candidates come from the row's logits
  int V;                           // (null: from the head's per-partial top-k lists)
  const float* gmax;               // [S][ngroups] the head's 32-column group maxima, or null
  int ngroups;
};

// Sampling candidates from materialised logits, one warp per row (no per-row array in shared
// memory): the k-th largest of up to 128 group maxima bounds the top k from below, the entries at
// or above it (at most kSelCand; else an exact radix select over the whole row) are ranked exactly.
constexpr int kSelCand = 128;
constexpr int kSelSamples = 128;

// Order-preserving key of a float: unsigned comparison of keys = float comparison of values.
__device__ __forceinline__ unsigned int float_key(float v) {
  const unsigned int u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Warp-level radix select, 8 bits per pass from the top of BITS-bit keys key(0..n-1) (an
// order-preserving unsigned view of the values): the key of the k-th largest entry, and in *r_out
// how many entries equal to it rank among the first k. hist: 256 ints of this warp.
template <typename K, int BITS, class KeyFn>
__device__ __forceinline__ K warp_radix_select(KeyFn key, int n, int k, int* hist, int* r_out) {
  const int lane = threadIdx.x & 31;
  K prefix = 0, mask = 0;
  int r = k;
#pragma unroll 1
  for (int shift = BITS - 8; shift >= 0; shift -= 8) {
    for (int b = lane; b < 256; b += 32) hist[b] = 0;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
      const K kb = key(i);
      if ((kb & mask) == prefix) atomicAdd(&hist[(int)(kb >> shift) & 255], 1);
    }
    __syncwarp();
    // lane l holds the bins 255 - 8l down to 248 - 8l: counts above a bin come from lower lanes
    int c[8], tot = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = hist[255 - 8 * lane - j];
      tot += c[j];
    }
    int incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int acc = incl - tot, bin = -1, above = 0;
    if (acc < r && r <= incl) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (bin < 0 && acc < r && r <= acc + c[j]) {
          bin = 255 - 8 * lane - j;
          above = acc;
        }
        acc += c[j];
      }
    }
    const unsigned int who = __ballot_sync(0xffffffffu, bin >= 0);
    const int src = __ffs(who) - 1;
    bin = __shfl_sync(0xffffffffu, bin, src);
    above = __shfl_sync(0xffffffffu, above, src);
    prefix |= (K)bin << shift;
    mask |= (K)255 << shift;
    r -= above;
    __syncwarp();
  }
  *r_out = r;
  return prefix;
}

__device__ __forceinline__ void philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                              uint32_t k1, uint32_t out[4]) {
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
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

// The uniform draw of (session, step): 53 bits from Philox4x32-10, key (session, "SAMP").
__device__ __forceinline__ double sample_uniform(uint32_t session, uint32_t step) {
  uint32_t o[4];
  philox4x32_10(step, 0, 0, 0, session, 0x53414D50u, o);
  const unsigned long long a = o[0] >> 5, b = o[1] >> 6;
  return (double)(a * 67108864ull + b) * (1.0 / 9007199254740992.0);
}

// One warp per session; lane k holds partials k and k + 32 (at most 64 partials). The step
// counter (output column and Philox counter) is read by every block before any work and advanced
// by the last block to finish (a.done counts finished blocks), so no separate launch bumps it.
constexpr int kSelectWarps = 4;

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

__global__ void __launch_bounds__(kSelectWarps * 32) select_kernel(const SelectArgs a) {
  __shared__ float cand_v[kSelectWarps][kSelCand];
  __shared__ int cand_i[kSelectWarps][kSelCand];
  __shared__ int sel_hist[kSelectWarps][256];
  __shared__ unsigned int sel_samp[kSelectWarps][kSelSamples];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = blockIdx.x * kSelectWarps + warp;
  const int step = a.step ? *a.step : 0;
  const int np = a.nsplit;  // partials per session (<= 64)
  if (s < a.n_sess && a.seglen[s] > 0) {
    const float4 none = make_float4(-INFINITY, 0.f, __int_as_float(0x7fffffff), 0.f);
    const float4 p0 = lane < np ? a.part[(size_t)s * np + lane] : none;
    const float4 p1 = lane + 32 < np ? a.part[(size_t)s * np + lane + 32] : none;
    // max and its first index (argmaxProb, greedy.go:90-102: the lowest index among equal maxima)
    float M = fmaxf(p0.x, p1.x);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    int idx = 0x7fffffff;
    if (p0.x == M) idx = __float_as_int(p0.z);
    if (p1.x == M) idx = min(idx, __float_as_int(p1.z));
#pragma unroll
    for (int o = 16; o; o >>= 1) idx = min(idx, __shfl_xor_sync(0xffffffffu, idx, o));
    // sum exp(l - max) over the vocabulary (in double, like the reference) and the target logit
    double S = 0.0;
    if (p0.x > -INFINITY) S += (double)p0.y * exp((double)p0.x - (double)M);
    if (p1.x > -INFINITY) S += (double)p1.y * exp((double)p1.x - (double)M);
    float lt = p0.w + p1.w;  // only the partial holding the target has a non-zero entry
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      S += __shfl_xor_sync(0xffffffffu, S, o);
      lt += __shfl_xor_sync(0xffffffffu, lt, o);
    }
    int tok = idx;
    if (a.mode == 1 && a.topk > 1 && a.logits) {
      // The top-k of the row's logits in (value descending, index ascending) order, compared as
      // order-preserving keys. The bound: the k-th largest of the group maxima (the head's, or
      // those of the groups (lane, g) = entries 32j + lane with j % 4 == g); at least k entries
      // reach it, and an entry below it ranks behind them all.
      const float* lg = a.logits + (size_t)s * a.V;
      const int V = a.V;
      const int K = min(a.topk, V);
      unsigned int* samp = sel_samp[warp];
      int ns = kSelSamples;
      if (a.gmax) {
        ns = a.ngroups;
        for (int i = lane; i < ns; i += 32) samp[i] = float_key(a.gmax[(size_t)s * a.ngroups + i]);
      } else {
        float gm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        for (int j0 = 0; j0 * 32 < V; j0 += 4) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int t = (j0 + g) * 32 + lane;
            if (t < V) gm[g] = fmaxf(gm[g], lg[t]);
          }
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) samp[lane * 4 + g] = float_key(gm[g]);
      }
      __syncwarp();
      int r_eq = 0;
      unsigned int tk = 0u;  // K >= V: every entry is a candidate
      if (K < V) tk = warp_radix_select<unsigned int, 32>([&](int i) { return samp[i]; }, ns, K, sel_hist[warp], &r_eq);
      int C = 0;
      for (int b0 = 0; b0 < V; b0 += 256) {
        float lv[8];  // eight loads in flight before any is used
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = b0 + 32 * u + lane;
          lv[u] = i < V ? lg[i] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = b0 + 32 * u + lane;
          const bool take = i < V && float_key(lv[u]) >= tk;
          const unsigned int tm = __ballot_sync(0xffffffffu, take);
          if (take) {
            const int at = C + __popc(tm & ((1u << lane) - 1u));
            if (at < kSelCand) {
              cand_v[warp][at] = lv[u];
              cand_i[warp][at] = i;
            }
          }
          C += __popc(tm);
        }
      }
      if (C > kSelCand) {
        // keys tied at the bound past the room: exactly the top k by a radix select over the row
        const unsigned int tau = warp_radix_select<unsigned int, 32>([&](int i) { return float_key(lg[i]); }, V, K,
                                                                     sel_hist[warp], &r_eq);
        int have = 0, eq_seen = 0;
        for (int base = 0; base < V; base += 32) {
          const int i = base + lane;
          const float l = i < V ? lg[i] : 0.f;
          const unsigned int kb = i < V ? float_key(l) : 0u;
          const bool eq = i < V && kb == tau;
          const unsigned int eqm = __ballot_sync(0xffffffffu, eq);
          const bool take = (i < V && kb > tau) || (eq && eq_seen + __popc(eqm & ((1u << lane) - 1u)) < r_eq);
          const unsigned int tm = __ballot_sync(0xffffffffu, take);
          if (take) {
            const int at = have + __popc(tm & ((1u << lane) - 1u));
            cand_v[warp][at] = l;
            cand_i[warp][at] = i;
          }
          have += __popc(tm);
          eq_seen += __popc(eqm);
        }
        C = K;
      }
      __syncwarp();
      // rank of each candidate: those before it in (value descending, index ascending) order
      float rv[kSelCand / 32];
      int ri[kSelCand / 32], rk[kSelCand / 32];
#pragma unroll
      for (int q = 0; q < kSelCand / 32; ++q) {
        const int c = lane + 32 * q;
        rv[q] = c < C ? cand_v[warp][c] : 0.f;
        ri[q] = c < C ? cand_i[warp][c] : 0;
        rk[q] = 0;
        if (c < C)
          for (int j = 0; j < C; ++j) rk[q] += better(cand_v[warp][j], cand_i[warp][j], rv[q], ri[q]) ? 1 : 0;
      }
      __syncwarp();
#pragma unroll
      for (int q = 0; q < kSelCand / 32; ++q)
        if (lane + 32 * q < C && rk[q] < K) {
          cand_v[warp][rk[q]] = rv[q];
          cand_i[warp][rk[q]] = ri[q];
        }
      for (int c = K + lane; c < a.topk; c += 32) {  // fewer tokens than k: the rest never drawn
        cand_v[warp][c] = -INFINITY;
        cand_i[warp][c] = 0x7fffffff;
      }
      __syncwarp();
    } else if (a.mode == 1 && a.topk > 1) {
      // Merge the partials' top-k lists: repeatedly take the largest remaining value (lowest
      // index on ties); lane k walks lists k and k + 32.
      int h0 = 0, h1 = 0;
      const size_t b0 = ((size_t)s * np + lane) * a.topk, b1 = ((size_t)s * np + lane + 32) * a.topk;
      for (int n = 0; n < a.topk; ++n) {
        float v0 = -INFINITY, v1 = -INFINITY;
        int i0 = 0x7fffffff, i1 = 0x7fffffff;
        if (lane < np && h0 < a.topk) {
          v0 = a.topv[b0 + h0];
          i0 = a.topi[b0 + h0];
        }
        if (lane + 32 < np && h1 < a.topk) {
          v1 = a.topv[b1 + h1];
          i1 = a.topi[b1 + h1];
        }
        const bool take1 = better(v1, i1, v0, i0);
        float bv = take1 ? v1 : v0;
        int bi = take1 ? i1 : i0;
        int bl = lane * 2 + (take1 ? 1 : 0);  // which list of which lane
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
          if (better(ov, oi, bv, bi) || (ov == bv && oi == bi && ol < bl)) {
            bv = ov;
            bi = oi;
            bl = ol;
          }
        }
        if (lane == 0) {
          cand_v[warp][n] = bv;
          cand_i[warp][n] = bi;
        }
        if (bl == lane * 2) ++h0;
        if (bl == lane * 2 + 1) ++h1;
      }
      __syncwarp();
    }
    if (a.mode == 1 && a.topk > 1) {
      // the draw over the k candidates (sampleFromCDF over the truncated distribution)
      if (lane == 0) {
        const double mx = (double)cand_v[warp][0] * a.inv_temp;
        double sp = 0.0;
        for (int n = 0; n < a.topk; ++n)
          sp += (cand_v[warp][n] == -INFINITY) ? 0.0 : exp((double)cand_v[warp][n] * a.inv_temp - mx);
        const double r = sample_uniform(a.session0 + (uint32_t)s, (uint32_t)step) * sp;
        double cum = 0.0;
        tok = cand_i[warp][a.topk - 1];
        for (int n = 0; n < a.topk; ++n) {
          cum += (cand_v[warp][n] == -INFINITY) ? 0.0 : exp((double)cand_v[warp][n] * a.inv_temp - mx);
          if (r <= cum) {
            tok = cand_i[warp][n];
            break;
          }
        }
      }
    }
    bool stop = false;
    for (int k = 0; k < a.n_stops; ++k) stop |= tok == a.stops[k];
    if (lane == 0 && stop) a.seglen[s] = 0;  // the session ends before the stop token
    if (lane == 0 && !stop) {
      const int col = a.gen_n ? a.gen_n[s] : step;
      a.next_tok[s] = tok;
      if (a.out_tok) a.out_tok[(size_t)s * a.out_stride + col] = tok;
      if (a.out_prob) a.out_prob[(size_t)s * a.out_stride + col] = (float)(1.0 / S);
      if (a.out_logprob) a.out_logprob[(size_t)s * a.out_stride + col] = (double)lt - (double)M - log(S);
      if (a.pos) {
        if (a.advance_from_len) a.pos[s] = a.pos[s] + a.seglen[s];
        else a.pos[s] = a.pos[s] + 1;
        a.seglen[s] = 1;
      }
      if (a.gen_n) {  // per-session generation: the session ends after its last token
        a.gen_n[s] = col + 1;
        if (a.limit && col + 1 >= a.limit[s]) a.seglen[s] = 0;
      }
    }
  }
  if (a.done) {
    // the last block to finish advances the step counter (every block has read it by then)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(a.done, 1) == (int)gridDim.x - 1) {
        *a.step += 1;
        *a.done = 0;
        __threadfence();
      }
    }
  }
}

}  // namespace eng
}  // namespace mc
