// Token selection with the whole decode-loop policy of sampleContinuation
// (internal/generate/sample.go:196-247) over materialised logits, one CTA per row:
//   1. the 3-gram repetition block (:213-227): a token that followed the trailing pair of the
//      generated tokens earlier gets -MaxFloat64;
//   2. Constraint.Mask (:229-231) as a token automaton: dfa[state][token] is the next state, -1
//      for a token that is not allowed (it gets -1e300, like constrain/grammar.go:259);
//   3. SampleRawLogitsAdvanced (:33-172): repetition penalty over the distinct tokens of the
//      trailing window of prefix ++ generated, argmax at T <= 0.001, else temperature, softmax and
//      either the draw in index order (no truncation) or the sort, top-k, top-p and
//      sampleFromCDF (:174-191);
//   4. stop tokens end the session before they are emitted (:233-237); Constraint.Advance (:238).
// Arithmetic in double like the reference. The running sums are taken in per-thread chunks whose
// totals are scanned across the block, so they differ from Go's left-to-right sums by rounding
// only; a draw can change only when it lies within that rounding of a bucket edge.
#include <cfloat>
#include <cstdlib>

#include "mc_engine.cuh"

namespace mc {
namespace eng {

constexpr int kPolicyThreads = 128;
constexpr int kPolicyWarps = kPolicyThreads / 32;
constexpr int kPolicyMaxVocab = 16384;  // the sort keys and indices of a row fill 192 KB of shared memory
constexpr int kPolicyMaxK = 1024;       // top-k up to this selects its candidates instead of sorting all

struct PolicyArgs {
  int n_rows, V, vp;                  // vp: V rounded up to a power of two (the sort's size)
  int kp;                             // top_k rounded up to a power of two (the candidates' sort)
  int kcap;                           // candidates the shared memory holds (a power of two >= kp)
  const float* logits;                // [n_rows][V]
  double temperature, rep_penalty, top_p;
  int top_k, rep_window, ban_trigrams;
  const int32_t* prefix;              // [n_rows][prefix_stride]: penalty prefix, prefix_len[row] tokens (or null)
  const int32_t* prefix_len;
  int prefix_stride;
  const int32_t* gen;                 // [n_rows][gen_stride]: generated tokens, gen_len[row] of them, or
  const int32_t* gen_len;             // *step of them when gen_len is null; null: none
  int gen_stride;
  const int32_t* dfa;                 // [states][V]: next state, -1 = not allowed; null: no constraint
  int32_t* dfa_state;                 // [n_rows] state of each row (< 0: unconstrained)
  const double* u;                    // [n_rows] uniform draws, or null: Philox (key, token index)
  uint32_t session0;                  // key of row r when key is null: session0 + r
  const uint32_t* key;                // [n_rows] Philox key of each row's draws, or null
  int32_t* gen_n;                     // [n_rows] tokens each row has emitted: its output column, draw counter
                                      // and 3-gram history length, advanced per emitted token; null: *step
  const int32_t* limit;               // [n_rows] tokens a row may emit (it ends after the last), with gen_n
  int32_t* step;                      // device step counter (output column and draw counter), or null:
  uint32_t step0;                     // column 0 and draw counter step0
  int out_stride;
  int32_t* next_tok;                  // [n_rows] or null
  int32_t* out_tok;                   // [n_rows][out_stride]
  float* out_prob;                    // [n_rows][out_stride] or null
  int32_t* pos;                       // positions advanced like SelectArgs (null: no change)
  int32_t* seglen;                    // [n_rows]: rows with seglen <= 0 have finished; null: all run
  int advance_from_len;
  int32_t* done;                      // finished-block counter; null: no step bump
  int n_stops;
  int stops[kMaxStops];
};

// Token k of the concatenation prefix ++ generated.
__device__ __forceinline__ int32_t pol_hist(const int32_t* pre, int np, const int32_t* gen, int k) {
  return k < np ? pre[k] : gen[k - np];
}

__device__ __forceinline__ bool pol_better(double v, int i, double bv, int bi) { return v > bv || (v == bv && i < bi); }

// Block reductions (every thread gets the result); red_d / red_i hold one entry per warp.
__device__ __forceinline__ double pol_block_sum(double v, double* red_d) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) red_d[warp] = v;
  __syncthreads();
  double s = 0.0;
#pragma unroll
  for (int w = 0; w < kPolicyWarps; ++w) s += red_d[w];
  __syncthreads();
  return s;
}

__device__ __forceinline__ double pol_block_max(double v, double* red_d) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) red_d[warp] = v;
  __syncthreads();
  double m = red_d[0];
#pragma unroll
  for (int w = 1; w < kPolicyWarps; ++w) m = fmax(m, red_d[w]);
  __syncthreads();
  return m;
}

__device__ __forceinline__ int pol_block_min(int v, int* red_i) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) red_i[warp] = v;
  __syncthreads();
  int m = red_i[0];
#pragma unroll
  for (int w = 1; w < kPolicyWarps; ++w) m = min(m, red_i[w]);
  __syncthreads();
  return m;
}

// First index of the largest value (argmax with the lowest index among equal maxima).
__device__ __forceinline__ void pol_block_argmax(double& bv, int& bi, double* red_d, int* red_i) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (pol_better(ov, oi, bv, bi)) bv = ov, bi = oi;
  }
  if (lane == 0) red_d[warp] = bv, red_i[warp] = bi;
  __syncthreads();
  bv = red_d[0];
  bi = red_i[0];
#pragma unroll
  for (int w = 1; w < kPolicyWarps; ++w)
    if (pol_better(red_d[w], red_i[w], bv, bi)) bv = red_d[w], bi = red_i[w];
  __syncthreads();
}

// Running sums of x[0..n): thread t owns the chunk [t*c, min(n, (t+1)*c)), c = ceil(n / threads);
// returns the sum of the chunks before its own (an exclusive scan of the chunk totals).
__device__ __forceinline__ double pol_chunk_base(const double* x, int n, int c, double* red_d) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int lo = min(n, (int)threadIdx.x * c), hi = min(n, lo + c);
  double s = 0.0;
  for (int i = lo; i < hi; ++i) s += x[i];
  double v = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += y;
  }
  if (lane == 31) red_d[warp] = v;
  __syncthreads();
  double base = 0.0;
  for (int w = 0; w < warp; ++w) base += red_d[w];
  __syncthreads();
  return base + v - s;
}

// Walks this thread's chunk with the running sum from base: the block-wide first index whose
// running sum is >= t (INT_MAX if none), and the running sum at index k into *at_k (shared).
__device__ __forceinline__ int pol_first_at_least(const double* x, int n, int c, double base, double t, int k,
                                                  double* at_k, int* red_i) {
  const int lo = min(n, (int)threadIdx.x * c), hi = min(n, lo + c);
  double cum = base;
  int first = 0x7fffffff;
  for (int i = lo; i < hi; ++i) {
    cum += x[i];
    if (first == 0x7fffffff && cum >= t) first = i;
    if (i == k) *at_k = cum;
  }
  return pol_block_min(first, red_i);
}

// Exclusive scan of one int per thread in thread order (every thread gets its own prefix).
__device__ __forceinline__ int pol_block_excl_scan(int v, int* red_i) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) red_i[warp] = x;
  __syncthreads();
  int base = 0;
  for (int w = 0; w < warp; ++w) base += red_i[w];
  __syncthreads();
  return base + x - v;
}

// Bitonic sort of n (a power of two) entries into (value descending, index ascending).
__device__ __forceinline__ void pol_sort(double* key, int32_t* idx, int n) {
  for (int kk = 2; kk <= n; kk <<= 1) {
    for (int j = kk >> 1; j > 0; j >>= 1) {
      for (int p = threadIdx.x; p < (n >> 1); p += kPolicyThreads) {
        const int lo = ((p & ~(j - 1)) << 1) | (p & (j - 1)), hi = lo | j;
        const bool up = (lo & kk) == 0;
        const double kl = key[lo], kh = key[hi];
        const int il = idx[lo], ih = idx[hi];
        if (pol_better(kh, ih, kl, il) == up) {
          key[lo] = kh;
          key[hi] = kl;
          idx[lo] = ih;
          idx[hi] = il;
        }
      }
      __syncthreads();
    }
  }
}

// Radix select over the bit patterns of p[0..n) (non-negative doubles, whose bits order like their
// values), 8 bits per pass from the top: *tau = the value bits of the k-th entry in (value
// descending, index ascending) order, *r = how many entries equal to it rank among the first k.
__device__ __forceinline__ void pol_radix_select(const double* p, int n, int k, unsigned long long* tau, int* r_out,
                                                 int* hist, int* pick) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned long long prefix = 0ull, mask = 0ull;
  int r = k;
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += kPolicyThreads) hist[b] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += kPolicyThreads) {
      const unsigned long long kb = (unsigned long long)__double_as_longlong(p[i]);
      if ((kb & mask) == prefix) atomicAdd(&hist[(int)(kb >> shift) & 255], 1);
    }
    __syncthreads();
    if (warp == 0) {
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
      int acc = incl - tot;
      if (acc < r && r <= incl) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (acc < r && r <= acc + c[j]) {
            pick[0] = 255 - 8 * lane - j;
            pick[1] = acc;
          }
          acc += c[j];
        }
      }
    }
    __syncthreads();
    prefix |= (unsigned long long)pick[0] << shift;
    mask |= 255ull << shift;
    r -= pick[1];
    __syncthreads();
  }
  *tau = prefix;
  *r_out = r;
}

// The k-th largest of the float keys fk[i] = bits of rz(p[i]) (p rounded toward zero to float32,
// whose bit patterns order like the values), by the same radix select over 32 bits: four passes.
__device__ __forceinline__ unsigned int pol_radix_select32(const unsigned int* fk, int n, int k, int* hist, int* pick) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned int prefix = 0u, mask = 0u;
  int r = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += kPolicyThreads) hist[b] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += kPolicyThreads) {
      const unsigned int kb = fk[i];
      if ((kb & mask) == prefix) atomicAdd(&hist[(kb >> shift) & 255], 1);
    }
    __syncthreads();
    if (warp == 0) {
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
      int acc = incl - tot;
      if (acc < r && r <= incl) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (acc < r && r <= acc + c[j]) {
            pick[0] = 255 - 8 * lane - j;
            pick[1] = acc;
          }
          acc += c[j];
        }
      }
    }
    __syncthreads();
    prefix |= (unsigned int)pick[0] << shift;
    mask |= 255u << shift;
    r -= pick[1];
    __syncthreads();
  }
  return prefix;
}

__global__ void __launch_bounds__(kPolicyThreads) policy_kernel(const __grid_constant__ PolicyArgs a) {
  extern __shared__ __align__(16) unsigned char pol_smem[];
  double* key = reinterpret_cast<double*>(pol_smem);
  // after the row's keys: its indices when the whole row is sorted, or the top-k candidates
  int32_t* idx = reinterpret_cast<int32_t*>(key + a.vp);
  double* ckey = key + a.vp;
  int32_t* cidx = reinterpret_cast<int32_t*>(ckey + a.kcap);
  unsigned int* fkey = reinterpret_cast<unsigned int*>(cidx + a.kcap);  // the candidates' float keys
  __shared__ double red_d[kPolicyWarps];
  __shared__ int red_i[kPolicyWarps];
  __shared__ int hist[256];
  __shared__ int pick[2];
  __shared__ double at_k;
  const int row = blockIdx.x, tid = threadIdx.x;
  const int V = a.V;
  const int step = a.step ? *a.step : (int)a.step0;
  const bool live = !a.seglen || a.seglen[row] > 0;
  if (live) {
    // tokens this row has emitted so far: its output column and the counter of its draw
    const int cnt = a.gen_n ? a.gen_n[row] : step;
    const uint32_t dkey = a.key ? a.key[row] : a.session0 + (uint32_t)row;
    const float* lg = a.logits + (size_t)row * V;
    for (int i = tid; i < V; i += kPolicyThreads) key[i] = (double)lg[i];
    const int ng = a.gen ? (a.gen_len ? a.gen_len[row] : cnt) : 0;
    const int32_t* gen = a.gen ? a.gen + (size_t)row * a.gen_stride : nullptr;
    const int np = a.prefix ? a.prefix_len[row] : 0;
    const int32_t* pre = a.prefix ? a.prefix + (size_t)row * a.prefix_stride : nullptr;
    __syncthreads();
    // 1. 3-gram block
    if (a.ban_trigrams && ng >= 2) {
      const int32_t w1 = gen[ng - 2], w2 = gen[ng - 1];
      for (int i = tid; i <= ng - 3; i += kPolicyThreads)
        if (gen[i] == w1 && gen[i + 1] == w2 && gen[i + 2] >= 0 && gen[i + 2] < V) key[gen[i + 2]] = -DBL_MAX;
    }
    __syncthreads();
    // 2. constraint mask
    const int state = a.dfa && a.dfa_state ? a.dfa_state[row] : -1;
    if (state >= 0) {
      const int32_t* tr = a.dfa + (size_t)state * V;
      for (int i = tid; i < V; i += kPolicyThreads)
        if (tr[i] < 0) key[i] = -1e300;
    }
    __syncthreads();
    // 3a. repetition penalty: each distinct in-range token of the window once
    const int total = np + ng;
    const int w = a.rep_window > 0 && a.rep_window < total ? a.rep_window : total;
    if (a.rep_penalty > 1.0 && w > 0) {
      for (int j = tid; j < w; j += kPolicyThreads) {
        const int32_t tok = pol_hist(pre, np, gen, total - w + j);
        if (tok < 0 || tok >= V) continue;
        bool seen = false;
        for (int k = 0; k < j && !seen; ++k) seen = pol_hist(pre, np, gen, total - w + k) == tok;
        if (seen) continue;
        const double v = key[tok];
        key[tok] = v > 0 ? v / a.rep_penalty : v * a.rep_penalty;
      }
    }
    __syncthreads();
    int tok = 0;
    double prob = 0.0;
    if (a.temperature <= 0.001) {
      // 3b. argmax; prob = 1 / sum exp(l - max)
      double bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int i = tid; i < V; i += kPolicyThreads)
        if (pol_better(key[i], i, bv, bi)) bv = key[i], bi = i;
      pol_block_argmax(bv, bi, red_d, red_i);
      double s = 0.0;
      for (int i = tid; i < V; i += kPolicyThreads) s += exp(key[i] - bv);
      s = pol_block_sum(s, red_d);
      tok = bi;
      prob = 1.0 / s;
    } else {
      // 3c. temperature and the shifted exponentials
      const double inv_t = 1.0 / a.temperature;
      double m = -DBL_MAX;
      for (int i = tid; i < V; i += kPolicyThreads) {
        const double v = key[i] * inv_t;
        key[i] = v;
        m = v > m ? v : m;
      }
      m = pol_block_max(m, red_d);
      for (int i = tid; i < V; i += kPolicyThreads) key[i] = exp(key[i] - m);
      __syncthreads();
      if (a.top_k <= 0 && a.top_p >= 0.9999) {
        // 3d. the draw in index order over every token
        const int c = (V + kPolicyThreads - 1) / kPolicyThreads;
        const double base = pol_chunk_base(key, V, c, red_d);
        pol_first_at_least(key, V, c, base, INFINITY, V - 1, &at_k, red_i);
        const double s = at_k;
        const double u = a.u ? a.u[row] : sample_uniform(dkey, (uint32_t)cnt);
        const int k = pol_first_at_least(key, V, c, base, u * s, -1, &at_k, red_i);
        tok = k == 0x7fffffff ? 0 : k;
        prob = key[tok] / s;
      } else {
        // 3e. probabilities in (value descending, index ascending) order: with top-k up to
        //     kPolicyMaxK, a radix select finds the k-th entry and only the k candidates are
        //     sorted; otherwise the whole row is sorted
        double s = 0.0;
        for (int i = tid; i < V; i += kPolicyThreads) s += key[i];
        s = pol_block_sum(s, red_d);
        const double inv = 1.0 / s;
        for (int i = tid; i < V; i += kPolicyThreads) key[i] *= inv;
        __syncthreads();
        const double* sk;
        const int32_t* si;
        int active;
        if (a.top_k > 0 && a.top_k < V && a.top_k <= kPolicyMaxK) {
          const int K = a.top_k;
          const int c = (V + kPolicyThreads - 1) / kPolicyThreads;
          const int lo = min(V, tid * c), hi = min(V, lo + c);
          // (i) the entries whose float key reaches the k-th largest float key F hold the top k:
          // an entry below F ranks behind the >= k entries at or above it. Their number C is k
          // unless float keys tie at F; up to the candidate capacity they are sorted exactly.
          for (int i = tid; i < V; i += kPolicyThreads) fkey[i] = __float_as_uint(__double2float_rz(key[i]));
          __syncthreads();
          const unsigned int F = pol_radix_select32(fkey, V, K, hist, pick);
          int cnt = 0;
          for (int i = lo; i < hi; ++i) cnt += fkey[i] >= F;
          int base = pol_block_excl_scan(cnt, red_i);
          if (tid == kPolicyThreads - 1) pick[0] = base + cnt;
          __syncthreads();
          const int C = pick[0];
          __syncthreads();
          int kp;
          if (C <= a.kcap) {
            for (int i = lo; i < hi; ++i)
              if (fkey[i] >= F) {
                ckey[base] = key[i];
                cidx[base++] = i;
              }
            kp = 1;
            while (kp < C) kp <<= 1;
            for (int j = C + tid; j < kp; j += kPolicyThreads) {
              ckey[j] = -1.0;
              cidx[j] = 0x7fffffff;
            }
          } else {
            // (ii) too many float ties: the exact select over the 64-bit patterns, then the
            // entries above its value tau and the first r entries equal to it by index
            unsigned long long tau;
            int r;
            pol_radix_select(key, V, K, &tau, &r, hist, pick);
            int eq = 0;
            for (int i = lo; i < hi; ++i) eq += (unsigned long long)__double_as_longlong(key[i]) == tau;
            int rank = pol_block_excl_scan(eq, red_i);
            if (tid == 0) pick[0] = 0;
            __syncthreads();
            for (int i = lo; i < hi; ++i) {
              const unsigned long long kb = (unsigned long long)__double_as_longlong(key[i]);
              const bool take = kb > tau || (kb == tau && rank++ < r);
              if (take) {
                const int at = atomicAdd(&pick[0], 1);
                ckey[at] = key[i];
                cidx[at] = i;
              }
            }
            kp = a.kp;
            for (int j = K + tid; j < kp; j += kPolicyThreads) {
              ckey[j] = -1.0;
              cidx[j] = 0x7fffffff;
            }
          }
          __syncthreads();
          pol_sort(ckey, cidx, kp);
          sk = ckey;
          si = cidx;
          active = K;
        } else {
          for (int i = tid; i < a.vp; i += kPolicyThreads) {
            idx[i] = i < V ? i : 0x7fffffff;
            if (i >= V) key[i] = -1.0;
          }
          __syncthreads();
          pol_sort(key, idx, a.vp);
          sk = key;
          si = idx;
          active = a.top_k > 0 && a.top_k < V ? a.top_k : V;
        }
        // 3f. the shortest prefix whose mass reaches top-p, then the draw
        const int c = (active + kPolicyThreads - 1) / kPolicyThreads;
        const double base = pol_chunk_base(sk, active, c, red_d);
        int cut = active;
        if (a.top_p > 0.0 && a.top_p < 1.0) {
          const int k = pol_first_at_least(sk, active, c, base, a.top_p, -1, &at_k, red_i);
          if (k != 0x7fffffff) cut = k + 1;
        }
        if (cut == 1) {
          tok = si[0];
          prob = 1.0;
        } else {
          pol_first_at_least(sk, active, c, base, INFINITY, cut - 1, &at_k, red_i);
          const double sp = at_k;
          const double u = a.u ? a.u[row] : sample_uniform(dkey, (uint32_t)cnt);
          int k = pol_first_at_least(sk, active, c, base, u * sp, -1, &at_k, red_i);
          if (k >= cut) k = cut - 1;
          tok = si[k];
          prob = sk[k] / sp;
        }
      }
    }
    // 4. stop tokens, outputs, position, constraint advance
    if (tid == 0) {
      bool stop = false;
      for (int k = 0; k < a.n_stops; ++k) stop |= a.stops[k] >= 0 && tok == a.stops[k];
      if (stop) {
        if (a.seglen) a.seglen[row] = 0;
      } else {
        const int col = a.gen_n || a.step ? cnt : 0;
        if (a.next_tok) a.next_tok[row] = tok;
        a.out_tok[(size_t)row * a.out_stride + col] = tok;
        if (a.out_prob) a.out_prob[(size_t)row * a.out_stride + col] = (float)prob;
        if (a.pos) {
          if (a.advance_from_len) a.pos[row] = a.pos[row] + a.seglen[row];
          else a.pos[row] = a.pos[row] + 1;
          a.seglen[row] = 1;
        }
        if (state >= 0) a.dfa_state[row] = a.dfa[(size_t)state * V + tok];
        if (a.gen_n) {
          a.gen_n[row] = cnt + 1;
          if (a.limit && a.seglen && cnt + 1 >= a.limit[row]) a.seglen[row] = 0;  // its last token
        }
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

// ---------------------------------------------------------------------------------------------
// The same policy with one warp per row and no per-row array in shared memory, for the knobs
// whose work needs no whole-row sort: argmax, the draw in index order, and top-k up to
// kPolRowMaxK. The warp streams its row's logits from global memory (L2-resident after the
// head) once per pass and recomputes each value the same way every time:
//   v(t) = logit, then -MaxFloat64 if the 3-gram block bans t, -1e300 if the automaton masks t,
//   then the repetition penalty if t is in the window (sample.go:48-69, 213-231), with the bans,
//   the penalty window and their union as bitmaps of the vocabulary in shared memory.
// Top-k, exactly: the probabilities p = exp(x - max) / sum are non-decreasing in x = v / T. Pass A
// takes the max and 128 group maxima of x; the k-th largest group maximum rounded down to float,
// tau, bounds the k-th largest x from below, so the entries with x >= tau (pass B, which also sums
// the exponentials) hold the top k unless an entry below tau has a probability equal to the k-th
// (rounding or underflow ties). Their exact probabilities are ranked by (p descending, index
// ascending); if the largest probability below tau is not clearly smaller than the k-th, or more
// than kPolRowCand entries reach tau, a 64-bit radix select over the probabilities' bit patterns
// (recomputed per pass) takes exactly the top k instead. Top-p and the draw then run over the k
// sorted candidates in sequence, like sample.go:152-191.
constexpr int kPolRowWarps = 4;
constexpr int kPolRowMaxK = 64;
constexpr int kPolRowCand = 128;
constexpr int kPolRowSamples = 128;  // group maxima: 4 per lane

__device__ __forceinline__ double pol_warp_sum(double v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// 2^z for z <= 0 to within 2e-6 relative, for the softmax denominator only. z is rounded to
// float: |z| 2^-24 absolute, so at most 30 * 2^-24 * ln 2 < 1.3e-6 relative for every term above
// 2^-30 (the largest term is 2^0 = 1, and the terms below 2^-30 weigh under 2048 * 2^-30 of the
// sum); exp2f adds at most 2 ulp (2.4e-7). Terms below 2^-126 are dropped.
constexpr double kPolSumRelErr = 2e-6;
__device__ __forceinline__ double pol_exp2_term(double z) {
  return z > -126.0 ? (double)exp2f((float)z) : 0.0;
}

__device__ __forceinline__ double pol_warp_max(double v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

struct PolRowValue {
  const float* lg;
  const uint32_t* ban;  // bitmap: the 3-gram block bans the token
  const uint32_t* pen;  // bitmap: the token is in the repetition window
  const uint32_t* mod;  // bitmap: ban | pen
  const int32_t* tr;    // the automaton's transitions from the row's state, or null
  double rep_penalty;
  // the token's value differs from its logit (banned, penalised or masked)
  __device__ __forceinline__ bool modified(int t) const {
    return ((mod[t >> 5] >> (t & 31)) & 1u) || (tr && tr[t] < 0);
  }
  // (not inlined: a predicated copy of the penalty's double division would run for every token)
  __device__ __noinline__ double full(float f, int t) const {
    double v = (double)f;
    const uint32_t bit = 1u << (t & 31);
    if (ban[t >> 5] & bit) v = -DBL_MAX;
    if (tr && tr[t] < 0) v = -1e300;
    if (pen[t >> 5] & bit) v = v > 0 ? v / rep_penalty : v * rep_penalty;
    return v;
  }
  __device__ __forceinline__ double operator()(int t) const {
    const float f = lg[t];
    return modified(t) ? full(f, t) : (double)f;
  }
  // The values of tokens 32 (j0 + g) + lane, g < 4 (0 past V), every lane of the warp calling:
  // the four loads are issued before any is used, and the rare modified tokens take the full
  // path under a warp-uniform branch.
  __device__ __forceinline__ void warp_values4(int j0, int V, double (&v)[4]) const {
    const int lane = threadIdx.x & 31;
    const int nwords = (V + 31) >> 5;
    float f[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int t = (j0 + g) * 32 + lane;
      f[g] = t < V ? lg[t] : 0.f;
    }
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int t = (j0 + g) * 32 + lane;
      v[g] = (double)f[g];
      if (tr) {
        const bool m = t < V && modified(t);
        if (__any_sync(0xffffffffu, m)) {
          if (m) v[g] = full(f[g], t);
        }
      } else if (j0 + g < nwords) {
        // the warp's 32 tokens share one bitmap word (bits past V are clear)
        const uint32_t wd = mod[j0 + g];
        if (wd != 0u && ((wd >> lane) & 1u)) v[g] = full(f[g], t);
      }
    }
  }
};

__global__ void __launch_bounds__(kPolRowWarps * 32, 7) policy_row_kernel(const __grid_constant__ PolicyArgs a) {
  extern __shared__ __align__(16) unsigned char pol_smem[];  // per warp: ban, penalty and ban|penalty bitmaps
  __shared__ double cand_p[kPolRowWarps][kPolRowCand];
  __shared__ int cand_i[kPolRowWarps][kPolRowCand];
  __shared__ int whist[kPolRowWarps][256];
  __shared__ unsigned int wsamp[kPolRowWarps][kPolRowSamples];
  __shared__ double csum[kPolRowWarps][kPolRowMaxK];  // running sums of the sorted candidates
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kPolRowWarps + warp;
  const int V = a.V;
  const int nw = (V + 31) / 32;  // bitmap words
  uint32_t* ban = reinterpret_cast<uint32_t*>(pol_smem) + (size_t)warp * 3 * nw;
  uint32_t* pen = ban + nw;
  uint32_t* mod = pen + nw;
  const int step = a.step ? *a.step : (int)a.step0;
  const bool live = row < a.n_rows && (!a.seglen || a.seglen[row] > 0);
  if (live) {
    const int cnt = a.gen_n ? a.gen_n[row] : step;
    const uint32_t dkey = a.key ? a.key[row] : a.session0 + (uint32_t)row;
    const int ng = a.gen ? (a.gen_len ? a.gen_len[row] : cnt) : 0;
    const int32_t* gen = a.gen ? a.gen + (size_t)row * a.gen_stride : nullptr;
    const int np = a.prefix ? a.prefix_len[row] : 0;
    const int32_t* pre = a.prefix ? a.prefix + (size_t)row * a.prefix_stride : nullptr;
    const int state = a.dfa && a.dfa_state ? a.dfa_state[row] : -1;
    for (int w = lane; w < 3 * nw; w += 32) ban[w] = 0u;
    __syncwarp();
    // 1. 3-gram block
    if (a.ban_trigrams && ng >= 2) {
      const int32_t w1 = gen[ng - 2], w2 = gen[ng - 1];
      for (int i = lane; i <= ng - 3; i += 32) {
        const int32_t t = gen[i + 2];
        if (gen[i] == w1 && gen[i + 1] == w2 && t >= 0 && t < V) {
          atomicOr(&ban[t >> 5], 1u << (t & 31));
          atomicOr(&mod[t >> 5], 1u << (t & 31));
        }
      }
    }
    // 3a. repetition penalty: each distinct in-range token of the window (the bitmap makes it once)
    const int total = np + ng;
    const int w = a.rep_window > 0 && a.rep_window < total ? a.rep_window : total;
    if (a.rep_penalty > 1.0 && w > 0) {
      for (int j = lane; j < w; j += 32) {
        const int32_t t = pol_hist(pre, np, gen, total - w + j);
        if (t >= 0 && t < V) {
          atomicOr(&pen[t >> 5], 1u << (t & 31));
          atomicOr(&mod[t >> 5], 1u << (t & 31));
        }
      }
    }
    __syncwarp();
    // 2. the constraint mask is read from the automaton's row in each pass
    const PolRowValue val{a.logits + (size_t)row * V, ban, pen, mod,
                          state >= 0 ? a.dfa + (size_t)state * V : nullptr, a.rep_penalty};
    int tok = 0;
    double prob = 0.0;
    if (a.temperature <= 0.001) {
      // 3b. argmax; prob = 1 / sum exp(v - max)
      double bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int j0 = 0; j0 * 32 < V; j0 += 4) {
        double v[4];
        val.warp_values4(j0, V, v);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int t = (j0 + g) * 32 + lane;
          if (t < V && pol_better(v[g], t, bv, bi)) bv = v[g], bi = t;
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (pol_better(ov, oi, bv, bi)) bv = ov, bi = oi;
      }
      double s = 0.0;
      for (int j0 = 0; j0 * 32 < V; j0 += 4) {
        double v[4];
        val.warp_values4(j0, V, v);
#pragma unroll
        for (int g = 0; g < 4; ++g)
          if ((j0 + g) * 32 + lane < V) s += exp(v[g] - bv);
      }
      s = pol_warp_sum(s);
      tok = bi;
      prob = 1.0 / s;
    } else {
      const double inv_t = 1.0 / a.temperature;
      const double u = a.u ? a.u[row] : sample_uniform(dkey, (uint32_t)cnt);
      if (a.top_k <= 0 && a.top_p >= 0.9999) {
        // 3d. the draw in index order: lane l owns the chunk [l*c, (l+1)*c); running sums from
        // the exclusive scan of the chunk totals
        double m = -DBL_MAX;
        for (int j0 = 0; j0 * 32 < V; j0 += 4) {
          double v[4];
          val.warp_values4(j0, V, v);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const double x = v[g] * inv_t;
            if ((j0 + g) * 32 + lane < V) m = x > m ? x : m;
          }
        }
        m = pol_warp_max(m);
        const int c = (V + 31) / 32;
        const int lo = min(V, lane * c), hi = min(V, lo + c);
        double cs = 0.0;
        for (int t = lo; t < hi; ++t) cs += exp(val(t) * inv_t - m);
        double incl = cs;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const double y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const double base = incl - cs;
        // the running sum at V - 1 (its owner walks its chunk from the base)
        double cum = base;
        for (int t = lo; t < hi; ++t) cum += exp(val(t) * inv_t - m);
        const double s = __shfl_sync(0xffffffffu, cum, (V - 1) / c);
        const double thr = u * s;
        int first = 0x7fffffff;
        double efirst = 0.0;
        cum = base;
        for (int t = lo; t < hi; ++t) {
          const double e = exp(val(t) * inv_t - m);
          cum += e;
          if (cum >= thr) {
            first = t;
            efirst = e;
            break;
          }
        }
        int f = first;
#pragma unroll
        for (int o = 16; o; o >>= 1) f = min(f, __shfl_xor_sync(0xffffffffu, f, o));
        tok = f == 0x7fffffff ? 0 : f;
        const double e_tok = f == 0x7fffffff ? exp(val(0) * inv_t - m)
                                             : __shfl_sync(0xffffffffu, efirst, __ffs(__ballot_sync(0xffffffffu, first == f)) - 1);
        prob = e_tok / s;
      } else {
        // 3e. top-k (0 < k < V, k <= kPolRowMaxK)
        const int K = a.top_k;
        double* cp = cand_p[warp];
        int* ci = cand_i[warp];
        // pass A: the max and the group maxima of x (lane l, group g: the lane's entries with j % 4 == g)
        // (the maxima of x = v / T are the maxima of v times 1/T, since rounding keeps the order;
        // unmodified values are their float logits, so those maxima are taken in float)
        // 16 loads in flight per lane (the pass waits on L2, not on arithmetic); entry j of the
        // lane belongs to group j % 4
        float fm = -INFINITY, fg[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        double dm = -INFINITY, dg[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        for (int j0 = 0; j0 * 32 < V; j0 += 16) {
          float f[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int t = (j0 + q) * 32 + lane;
            f[q] = t < V ? val.lg[t] : 0.f;
          }
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int g = q & 3;
            const int t = (j0 + q) * 32 + lane;
            const bool in = t < V;
            bool md;
            if (val.tr) {
              md = in && val.modified(t);
            } else {
              // the warp's 32 tokens share one bitmap word (bits past V are clear)
              md = (j0 + q) * 32 < V && ((val.mod[j0 + q] >> lane) & 1u);
            }
            if (__any_sync(0xffffffffu, md)) {
              if (md) {
                const double v = val.full(f[q], t);
                dm = fmax(dm, v);
                dg[g] = fmax(dg[g], v);
              }
            }
            if (in && !md) {
              fm = fmaxf(fm, f[q]);
              fg[g] = fmaxf(fg[g], f[q]);
            }
          }
        }
        double m = pol_warp_max(fmax((double)fm, dm)) * inv_t;
        if (!(m > -DBL_MAX)) m = -DBL_MAX;  // the running maximum starts at -MaxFloat64
        double gm[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) gm[g] = fmax((double)fg[g], dg[g]) * inv_t;
        // the bound: the k-th largest of the group maxima rounded down to float (32-bit keys, four
        // radix passes). At least k entries reach it (each such maximum is an entry >= its
        // rounded-down value), which is all the candidate set needs.
#pragma unroll
        for (int g = 0; g < 4; ++g) wsamp[warp][lane * 4 + g] = float_key(__double2float_rd(gm[g]));
        __syncwarp();
        int r_unused;
        const unsigned int tk = warp_radix_select<unsigned int, 32>([&](int i) { return wsamp[warp][i]; },
                                                                     kPolRowSamples, K, whist[warp], &r_unused);
        const double tau = (double)__uint_as_float((tk & 0x80000000u) ? (tk & 0x7fffffffu) : ~tk);
        // pass B: the sum of the exponentials; the entries with x >= tau in index order, and the
        // largest x below tau
        double s = 0.0, xo = -INFINITY;
        int C = 0;
        // the exponent of 2 of entry x is (x - m) log2(e) = x log2(e) + zm (one rounding fewer than
        // the subtraction first; m = -DBL_MAX only when every x is -inf, whose terms stay 0)
        const double zm = -m * 1.4426950408889634;
        for (int j0 = 0; j0 * 32 < V; j0 += 4) {
          double v[4];
          val.warp_values4(j0, V, v);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int t = (j0 + g) * 32 + lane;
            const bool in = t < V;
            const double x = v[g] * inv_t;
            if (in) s += pol_exp2_term(fma(x, 1.4426950408889634, zm));  // (x - m) log2(e)
            const bool take = in && x >= tau;
            if (in && !take) xo = fmax(xo, x);
            const unsigned int tm = __ballot_sync(0xffffffffu, take);
            if (take) {
              const int at = C + __popc(tm & ((1u << lane) - 1u));
              if (at < kPolRowCand) {
                cp[at] = x;
                ci[at] = t;
              }
            }
            C += __popc(tm);
          }
        }
        s = pol_warp_sum(s);
        xo = pol_warp_max(xo);
        const double inv = 1.0 / s;
        bool exact = C <= kPolRowCand;
        if (exact) {
          __syncwarp();
          for (int c = lane; c < C; c += 32) cp[c] = exp(cp[c] - m) * inv;
          __syncwarp();
        }
        // rank the candidates: those before each in (p descending, index ascending) order
        auto rank_in_place = [&](int n) {
          double rv[kPolRowCand / 32];
          int ri[kPolRowCand / 32], rk[kPolRowCand / 32];
#pragma unroll
          for (int q = 0; q < kPolRowCand / 32; ++q) {
            const int c = lane + 32 * q;
            rv[q] = c < n ? cp[c] : 0.0;
            ri[q] = c < n ? ci[c] : 0;
            rk[q] = 0;
            if (c < n) {
#pragma unroll 4
              for (int j = 0; j < n; ++j) rk[q] += pol_better(cp[j], ci[j], rv[q], ri[q]) ? 1 : 0;
            }
          }
          __syncwarp();
#pragma unroll
          for (int q = 0; q < kPolRowCand / 32; ++q)
            if (lane + 32 * q < n && rk[q] < K) {
              cp[rk[q]] = rv[q];
              ci[rk[q]] = ri[q];
            }
          __syncwarp();
        };
        if (exact) {
          rank_in_place(C);
          // no entry below tau may reach the k-th probability (a margin covers the last bits of exp)
          const double p_out = xo == -INFINITY ? 0.0 : exp(xo - m) * inv;
          exact = p_out * (1.0 + 0x1p-40) < cp[K - 1];
        }
        if (!exact) {
          // exactly the top k by the 64-bit patterns of p (>= 0, so they order like p): the entries
          // above the k-th pattern, then the first r_eq equal to it in index order
          auto pbits = [&](int t) {
            return (unsigned long long)__double_as_longlong(exp(val(t) * inv_t - m) * inv);
          };
          int r_eq = 0;
          const unsigned long long kth = warp_radix_select<unsigned long long, 64>(pbits, V, K, whist[warp], &r_eq);
          int have = 0, eq_seen = 0;
          for (int j = 0; j * 32 < V; ++j) {
            const int t = j * 32 + lane;
            const unsigned long long kb = t < V ? pbits(t) : 0ull;
            const bool eq = t < V && kb == kth;
            const unsigned int eqm = __ballot_sync(0xffffffffu, eq);
            const bool take = (t < V && kb > kth) || (eq && eq_seen + __popc(eqm & ((1u << lane) - 1u)) < r_eq);
            const unsigned int tm = __ballot_sync(0xffffffffu, take);
            if (take) {
              const int at = have + __popc(tm & ((1u << lane) - 1u));
              cp[at] = __longlong_as_double((long long)kb);
              ci[at] = t;
            }
            have += __popc(tm);
            eq_seen += __popc(eqm);
          }
          __syncwarp();
          rank_in_place(K);
        }
        // 3f. the shortest prefix whose mass reaches top-p, then the draw, over the running sums of
        // the sorted candidates in the reference's order (sample.go:141-152, 174-191). Lane 0 forms
        // them once: the top-p cut is the first that reaches top-p, the draw's total sp is the one
        // at the cut (the same additions in the same order), and the draw takes the first running
        // sum at or above u * sp. The candidates' probabilities scale with 1/s, which pass B summed
        // to within kPolSumRelErr: a top-p comparison closer than that to its threshold is decided
        // again with the sum of double-precision exponentials (the draw and the reported
        // probability are ratios of candidate probabilities, so the scale of s cancels in them).
        const bool use_top_p = a.top_p > 0.0 && a.top_p < 1.0;
        double* cs = csum[warp];
        auto running_sums = [&](bool check) {
          int cut = K;
          bool near = false;
          if (lane == 0) {
            double cum = 0.0;
            for (int i = 0; i < K; ++i) {
              cum += cp[i];
              cs[i] = cum;
              if (use_top_p) {
                near |= check && fabs(cum - a.top_p) <= 4.0 * kPolSumRelErr * fmax(cum, a.top_p);
                if (cum >= a.top_p) {
                  cut = i + 1;
                  break;
                }
              }
            }
          }
          __syncwarp();
          return make_int2(__shfl_sync(0xffffffffu, cut, 0), __shfl_sync(0xffffffffu, near ? 1 : 0, 0));
        };
        int2 cn = running_sums(true);
        if (cn.y) {
          double sd = 0.0;
          for (int j0 = 0; j0 * 32 < V; j0 += 4) {
            double v[4];
            val.warp_values4(j0, V, v);
#pragma unroll
            for (int g = 0; g < 4; ++g)
              if ((j0 + g) * 32 + lane < V) sd += exp(v[g] * inv_t - m);
          }
          sd = pol_warp_sum(sd);
          const double f = s / sd;  // the candidates' probabilities with the exact sum
          for (int c = lane; c < K; c += 32) cp[c] *= f;
          __syncwarp();
          cn = running_sums(false);
        }
        const int active = cn.x;
        if (active == 1) {
          tok = ci[0];
          prob = 1.0;
        } else {
          const double sp = cs[active - 1];
          const double r = u * sp;
          int k = active - 1;
          for (int i0 = 0; i0 < active; i0 += 32) {
            const int i = i0 + lane;
            const unsigned int hit = __ballot_sync(0xffffffffu, i < active && r <= cs[i]);
            if (hit) {
              k = i0 + __ffs(hit) - 1;
              break;
            }
          }
          tok = ci[k];
          prob = cp[k] / sp;
        }
      }
    }
    // 4. stop tokens, outputs, position, constraint advance
    if (lane == 0) {
      bool stop = false;
      for (int k = 0; k < a.n_stops; ++k) stop |= a.stops[k] >= 0 && tok == a.stops[k];
      if (stop) {
        if (a.seglen) a.seglen[row] = 0;
      } else {
        const int col = a.gen_n || a.step ? cnt : 0;
        if (a.next_tok) a.next_tok[row] = tok;
        a.out_tok[(size_t)row * a.out_stride + col] = tok;
        if (a.out_prob) a.out_prob[(size_t)row * a.out_stride + col] = (float)prob;
        if (a.pos) {
          if (a.advance_from_len) a.pos[row] = a.pos[row] + a.seglen[row];
          else a.pos[row] = a.pos[row] + 1;
          a.seglen[row] = 1;
        }
        if (state >= 0) a.dfa_state[row] = a.dfa[(size_t)state * V + tok];
        if (a.gen_n) {
          a.gen_n[row] = cnt + 1;
          if (a.limit && a.seglen && cnt + 1 >= a.limit[row]) a.seglen[row] = 0;  // its last token
        }
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

inline int policy_vp(int V) {
  int vp = 2;  // even, so the candidate arrays after the row's keys and indices stay 8-byte aligned
  while (vp < V) vp <<= 1;
  return vp;
}

// The largest launch's shared memory: the top-k branch at the largest vocabulary and top-k (row
// keys, 2048 candidates, float keys), above a whole-row sort's.
inline size_t policy_smem(int V) {
  const size_t vp = (size_t)policy_vp(V);
  return vp * (sizeof(double) + sizeof(uint32_t)) + 2 * (size_t)kPolicyMaxK * (sizeof(double) + sizeof(int32_t));
}

// Shared memory of one launch: the row's keys, then the indices of a whole-row sort or the top-k
// candidates (keys and indices), by the branch the kernel takes for these knobs.
inline size_t policy_smem_for(const PolicyArgs& a) {
  const bool draw = a.temperature > 0.001;
  const bool truncated = draw && !(a.top_k <= 0 && a.top_p >= 0.9999);
  const bool select = truncated && a.top_k > 0 && a.top_k < a.V && a.top_k <= kPolicyMaxK;
  size_t b = (size_t)a.vp * sizeof(double);
  if (select) b += (size_t)a.kcap * (sizeof(double) + sizeof(int32_t)) + (size_t)a.vp * sizeof(uint32_t);
  else if (truncated) b += (size_t)a.vp * sizeof(int32_t);
  return b;
}

int launch_policy(PolicyArgs& a, cudaStream_t s) {
  if (a.V < 1 || a.V > kPolicyMaxVocab) return set_error(kUnsupported, "sampling policy: vocabulary above 16384");
  a.vp = policy_vp(a.V);
  a.kp = 1;
  while (a.kp < a.top_k && a.kp < kPolicyMaxK) a.kp <<= 1;
  a.kcap = 2 * a.kp;  // room for float-key ties beyond the top k
  const bool draw = a.temperature > 0.001;
  const bool index_draw = draw && a.top_k <= 0 && a.top_p >= 0.9999;
  const bool small_k = draw && !index_draw && a.top_k > 0 && a.top_k < a.V && a.top_k <= kPolRowMaxK;
  const bool force_block = getenv("MC_POLICY_BLOCK") != nullptr;  // the CTA-per-row kernel for every knob
  if (!force_block && (!draw || index_draw || small_k)) {
    const size_t smem = (size_t)kPolRowWarps * 3 * ((a.V + 31) / 32) * sizeof(uint32_t);  // <= 24 KB
    if (a.n_rows > 0) policy_row_kernel<<<(a.n_rows + kPolRowWarps - 1) / kPolRowWarps, kPolRowWarps * 32, smem, s>>>(a);
    MC_CUDA(cudaGetLastError());
    return kOk;
  }
  const size_t smem = policy_smem_for(a);  // within the limit raised once per device (policy_smem)
  if (a.n_rows > 0) policy_kernel<<<a.n_rows, kPolicyThreads, smem, s>>>(a);
  MC_CUDA(cudaGetLastError());
  return kOk;
}

}  // namespace eng
}  // namespace mc
