// Windowed causal attention over the per-session key/value rings (attendPosition,
// internal/quant/attention.go:71-104):
//   lo = max(WindowStart(pos, W), pos - cache + 1)        (attention.go:83, nn/attention.go:55-60)
//   s_j = (q_h . k_j,h) * float32(1/sqrt(dh))            (:85-90)
//   p = softmax(s) with the reference's exp polynomial    (nn/head.go:93-111)
//   o_h = sum_j p_j v_j,h                                 (:93-97)
// The output o (and max |o| of each row, the scale of its digit slicing) feeds the block kernel
// that applies the output projection.
//
// Decode is bound by reading the rings from HBM: each CTA walks its sessions, staging the
// session's key and value rings into shared memory with TMA bulk copies (one per ring, the
// slots [0, min(pos+1, cache)) are contiguous) while it computes on the previous session.
#include "mc_engine.cuh"

namespace mc {
namespace eng {

struct AttnArgs {
  int n_sess, D, heads, dh, cache, window, n_attn, attn_slot;
  int P, spt;
  const int32_t* pos0;
  const int32_t* seglen;
  const float* qbuf;
  const float* kv;
  const float* kvlin;
  float* att;
  float* att_rowmax;
  float scale;
};

constexpr int kAttnThreads = 256;

__device__ __forceinline__ int grow_of(const AttnArgs& a, int s, int t) {
  return (s / a.spt) * kRows + (s % a.spt) * a.P + t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
  return m;
}

// Decode: one row per session (P == 1). Dynamic smem: nbuf x (2 rings) + q + scores.
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const __grid_constant__ AttnArgs a, int nbuf) {
  extern __shared__ uint8_t smem_raw[];
  float* sm = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int D = a.D, cache = a.cache;
  const size_t ring_f = (size_t)cache * D;
  float* kvbuf = sm;                          // nbuf x [2][cache][D]
  float* sq = kvbuf + nbuf * 2 * ring_f;      // [D]
  float* sc = sq + D;                         // [heads][cache]
  float* red = sc + a.heads * cache;          // [32]
  uint64_t* bar = reinterpret_cast<uint64_t*>(red + 32);  // [2]

  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_barrier_init();
  }
  __syncthreads();

  auto issue = [&](int s, int buf) {
    const int pos = a.pos0[s];
    const int nslots = min(pos + 1, cache);
    const uint32_t bytes = (uint32_t)(nslots * D * 4);
    const float* src = a.kv + ((size_t)s * a.n_attn + a.attn_slot) * 2 * ring_f;
    float* dst = kvbuf + (size_t)buf * 2 * ring_f;
    mbar_arrive_expect_tx(&bar[buf], 2 * bytes);
    bulk_load(dst, src, bytes, &bar[buf]);
    bulk_load(dst + ring_f, src + ring_f, bytes, &bar[buf]);
  };

  uint32_t phase[2] = {0, 0};
  int it = 0;
  int s = blockIdx.x;
  if (threadIdx.x == 0 && s < a.n_sess && a.seglen[s] > 0) issue(s, 0);
  for (; s < a.n_sess; s += gridDim.x, ++it) {
    const int buf = nbuf == 2 ? (it & 1) : 0;
    const int next = s + gridDim.x;
    const bool active = a.seglen[s] > 0;
    // Single buffer: load this session now (the previous one is finished: the loop ends with a
    // block-wide barrier). Double buffer: prefetch the next session into the other buffer.
    if (nbuf == 1 && it > 0 && threadIdx.x == 0 && active) issue(s, 0);
    if (nbuf == 2 && threadIdx.x == 0 && next < a.n_sess && a.seglen[next] > 0) issue(next, buf ^ 1);
    if (!active) continue;
    bool ok = mbar_wait_or_abort(&bar[buf], phase[buf], kErrWaitFull);
    phase[buf] ^= 1;
    const int pos = a.pos0[s];
    int ws = 0;
    if (a.window > 0 && pos - a.window + 1 > 0) ws = pos - a.window + 1;
    const int lo = max(ws, pos - cache + 1);
    const int span = pos - lo + 1;
    const int grow = grow_of(a, s, 0);
    const float* K = kvbuf + (size_t)buf * 2 * ring_f;
    const float* V = K + ring_f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) sq[d] = a.qbuf[(size_t)grow * D + d];
    __syncthreads();
    const int dh = a.dh;
    if (ok) {
      for (int item = threadIdx.x; item < a.heads * span; item += blockDim.x) {
        const int h = item / span, i = item % span;
        const int slot = (lo + i) % cache;
        const float* k = K + (size_t)slot * D + h * dh;
        const float* q = sq + h * dh;
        float acc = 0.f;
        for (int e = 0; e < dh; ++e) {
          const int ee = (e + i) % dh;  // rotated start: lanes hit different banks
          acc = __fmaf_rn(q[ee], k[ee], acc);
        }
        sc[h * cache + i] = __fmul_rn(acc, a.scale);
      }
    }
    __syncthreads();
    // softmax per head: one warp per head
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int h = warp; h < a.heads; h += blockDim.x >> 5) {
      float* row = sc + h * cache;
      float m = -3.402823466e38f;
      for (int i = lane; i < span; i += 32) m = fmaxf(m, row[i]);
#pragma unroll
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float sum = 0.f;
      for (int i = lane; i < span; i += 32) {
        const float e = ref_vec_exp(__fsub_rn(row[i], m));
        row[i] = e;
        sum = __fadd_rn(sum, e);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
      const float inv = __fdiv_rn(1.0f, sum);
      for (int i = lane; i < span; i += 32) row[i] = __fmul_rn(row[i], inv);
    }
    __syncthreads();
    float omax = 0.f;
    for (int e = threadIdx.x; e < D; e += blockDim.x) {
      const int h = e / dh;
      const float* p = sc + h * cache;
      float o = 0.f;
      for (int i = 0; i < span; ++i) o = __fmaf_rn(p[i], V[(size_t)((lo + i) % cache) * D + e], o);
      a.att[(size_t)grow * D + e] = o;
      omax = fmaxf(omax, fabsf(o));
    }
    omax = block_max(omax, red);
    if (threadIdx.x == 0) a.att_rowmax[grow] = omax;
    __syncthreads();
  }
  // Drain a prefetch that was issued for a session this CTA does not compute (none by design:
  // prefetches target sessions of this CTA's own walk). Nothing to wait for here.
}

// Prefill: one CTA per session; the segment's keys and values (written by the block kernel to
// kvlin) are staged into shared memory; one warp per (query, head) item.
__global__ void __launch_bounds__(kAttnThreads) attn_prefill_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  float* sm = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int s = blockIdx.x;
  const int len = a.seglen[s];
  if (len <= 0) return;
  const int D = a.D, dh = a.dh;
  float* kvs = sm;                      // [len][2][D]
  float* red = kvs + (size_t)len * 2 * D;
  uint64_t* bar = reinterpret_cast<uint64_t*>(red + 32);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t bytes = (uint32_t)(len * 2 * D * 4);
    mbar_arrive_expect_tx(bar, bytes);
    bulk_load(kvs, a.kvlin + (size_t)s * a.P * 2 * D, bytes, bar);
  }
  const bool ok = mbar_wait_or_abort(bar, 0, kErrWaitFull);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int p0 = a.pos0[s];
  if (ok) {
    for (int item = warp; item < len * a.heads; item += nw) {
      const int t = item / a.heads, h = item % a.heads;
      const int pos = p0 + t;
      int ws = 0;
      if (a.window > 0 && pos - a.window + 1 > 0) ws = pos - a.window + 1;
      const int lo = max(max(ws, pos - a.cache + 1), p0) - p0;  // in-segment index of the first key
      const int span = t - lo + 1;
      const float* q = a.qbuf + (size_t)grow_of(a, s, t) * D + h * dh;
      // scores: lane i handles keys lo + i, lo + i + 32, ... (at most 4 per lane: span <= 128)
      float sv[4];
      float m = -3.402823466e38f;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = lane + 32 * u;
        sv[u] = -3.402823466e38f;
        if (i < span) {
          const float* k = kvs + (size_t)(lo + i) * 2 * D + h * dh;
          float acc = 0.f;
          for (int e = 0; e < dh; ++e) {
            const int ee = (e + i) % dh;
            acc = __fmaf_rn(q[ee], k[ee], acc);
          }
          sv[u] = __fmul_rn(acc, a.scale);
          m = fmaxf(m, sv[u]);
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float sum = 0.f;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = lane + 32 * u;
        if (i < span) {
          sv[u] = ref_vec_exp(__fsub_rn(sv[u], m));
          sum = __fadd_rn(sum, sv[u]);
        } else {
          sv[u] = 0.f;
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
      const float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
      for (int u = 0; u < 4; ++u) sv[u] = __fmul_rn(sv[u], inv);
      // o[e] for e = lane, lane + 32 (dh <= 64)
      float o0 = 0.f, o1 = 0.f;
      for (int i = 0; i < span; ++i) {
        const float p = __shfl_sync(0xffffffffu, sv[i >> 5], i & 31);
        const float* v = kvs + (size_t)(lo + i) * 2 * D + D + h * dh;
        if (lane < dh) o0 = __fmaf_rn(p, v[lane], o0);
        if (lane + 32 < dh) o1 = __fmaf_rn(p, v[lane + 32], o1);
      }
      float* out = a.att + (size_t)grow_of(a, s, t) * D + h * dh;
      if (lane < dh) out[lane] = o0;
      if (lane + 32 < dh) out[lane + 32] = o1;
    }
  }
  __syncthreads();
  // max |o| of each row
  for (int t = warp; t < len; t += nw) {
    const float* o = a.att + (size_t)grow_of(a, s, t) * D;
    float m = 0.f;
    for (int e = lane; e < D; e += 32) m = fmaxf(m, fabsf(o[e]));
#pragma unroll
    for (int k = 16; k; k >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, k));
    if (lane == 0) a.att_rowmax[grow_of(a, s, t)] = m;
  }
}

}  // namespace eng
}  // namespace mc
