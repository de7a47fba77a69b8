// Windowed causal attention over the per-session key/value rings (attendPosition,
// internal/quant/attention.go:71-104):
//   lo = max(WindowStart(pos, W), pos - cache + 1)        (attention.go:83, nn/attention.go:55-60)
//   s_j = (q_h . k_j,h) * float32(1/sqrt(dh))            (:85-90)
//   p = softmax(s) with the reference's exp polynomial    (nn/head.go:93-111)
//   o_h = sum_j p_j v_j,h                                 (:93-97)
// The output o (and max |o| of each row, the scale of its digit slicing) feeds the block kernel
// that applies the output projection.
//
// Decode is bound by reading the rings from HBM; each (session, head) warp streams its head's
// contiguous key and value windows with many loads in flight.
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
  const int32_t* sess_list;  // prefill: CTA i runs session sess_list[i] (some sessions only), or null: sess0 + i
  int sess0;                 // prefill: first session of a pass over a contiguous range of sessions
  int last_only;             // prefill: only each segment's last query (its other outputs are unused)
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

// Decode: one warp per (session, head), P == 1. The rings are head-major ([K|V][head][slot][dh]),
// so the warp streams two contiguous regions. Lane i computes the scores of window positions
// lo+i, lo+i+32, ... (its key rows, 16-byte loads, all issued before the dot products); the
// softmax runs on warp shuffles; then the lanes own head dimensions and walk the window's value
// rows sixteen at a time (loads issued before the multiply-adds). max |o| of the row is
// max-accumulated into att_rowmax (zeroed by the block kernel).
template <int DH>  // head width known at compile time (0: taken from the arguments)
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
  const int gw = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  const int s = gw / a.heads, h = gw - (gw / a.heads) * a.heads;
  if (s >= a.n_sess || a.seglen[s] <= 0) return;
  const int D = a.D, dh = DH > 0 ? DH : a.dh, cache = a.cache;
  const int pos = a.pos0[s];
  int ws = 0;
  if (a.window > 0 && pos - a.window + 1 > 0) ws = pos - a.window + 1;
  const int lo = max(ws, pos - cache + 1);
  const int span = pos - lo + 1;  // <= cache <= 128
  const int lo_slot = lo % cache;
  const int grow = grow_of(a, s, 0);
  const float* K = a.kv + ((size_t)a.attn_slot * a.n_sess + s) * 2 * (size_t)cache * D + (size_t)h * cache * dh;
  const float* V = K + (size_t)cache * D;
  const float* q = a.qbuf + (size_t)grow * D + h * dh;

  float sc[4];
  int slot[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    int sl = lo_slot + lane + 32 * k;
    if (sl >= cache) sl -= cache;
    if (sl >= cache) sl -= cache;
    slot[k] = sl;
    sc[k] = 0.f;
  }
  if constexpr (DH > 0) {
    float4 q4[DH / 4];
#pragma unroll
    for (int f = 0; f < DH / 4; ++f) q4[f] = reinterpret_cast<const float4*>(q)[f];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (32 * k >= span) break;  // warp-uniform
      const bool act = lane + 32 * k < span;
      const float4* row = reinterpret_cast<const float4*>(K + (size_t)slot[k] * DH);
      float4 k4[DH / 4];
#pragma unroll
      for (int f = 0; f < DH / 4; ++f) k4[f] = act ? row[f] : make_float4(0.f, 0.f, 0.f, 0.f);
      float acc = 0.f;
#pragma unroll
      for (int f = 0; f < DH / 4; ++f) {
        acc = __fmaf_rn(q4[f].x, k4[f].x, acc);
        acc = __fmaf_rn(q4[f].y, k4[f].y, acc);
        acc = __fmaf_rn(q4[f].z, k4[f].z, acc);
        acc = __fmaf_rn(q4[f].w, k4[f].w, acc);
      }
      sc[k] = acc;
    }
  } else {
    for (int e = 0; e < dh; ++e) {
      const float qe = q[e];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (lane + 32 * k < span) sc[k] = __fmaf_rn(qe, K[(size_t)slot[k] * dh + e], sc[k]);
    }
  }
  float m = -3.402823466e38f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (lane + 32 * k < span) {
      sc[k] = __fmul_rn(sc[k], a.scale);
      m = fmaxf(m, sc[k]);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (lane + 32 * k < span) {
      sc[k] = ref_vec_exp(__fsub_rn(sc[k], m));
      sum = __fadd_rn(sum, sc[k]);
    } else {
      sc[k] = 0.f;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
  const float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
  for (int k = 0; k < 4; ++k) sc[k] = __fmul_rn(sc[k], inv);

  // o[e] for e = lane, lane + 32 (dh <= 64), the window in order, sixteen value rows at a time
  float o0 = 0.f, o1 = 0.f;
  const bool has0 = lane < dh, has1 = lane + 32 < dh;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int j0 = 32 * k + 16 * half;
      if (j0 >= span) break;  // warp-uniform
      float v0[16], v1[16];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        int sl = lo_slot + j0 + jj;
        if (sl >= cache) sl -= cache;
        if (sl >= cache) sl -= cache;
        const bool in = j0 + jj < span;
        const float* vr = V + (size_t)sl * dh;
        v0[jj] = (in && has0) ? vr[lane] : 0.f;
        v1[jj] = (in && has1) ? vr[lane + 32] : 0.f;
      }
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const float p = __shfl_sync(0xffffffffu, sc[k], 16 * half + jj);
        if (j0 + jj < span) {
          o0 = __fmaf_rn(p, v0[jj], o0);
          o1 = __fmaf_rn(p, v1[jj], o1);
        }
      }
    }
  }
  float* out = a.att + (size_t)grow * D + h * dh;
  float om = 0.f;
  if (has0) {
    out[lane] = o0;
    om = fabsf(o0);
  }
  if (has1) {
    out[lane + 32] = o1;
    om = fmaxf(om, fabsf(o1));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) om = fmaxf(om, __shfl_xor_sync(0xffffffffu, om, o));
  if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(a.att_rowmax + grow), __float_as_uint(om));
}

// One decode item (session, head) of the staged attention, shared by the staged kernel and the
// persistent decode loop. The window of a session at position pos: the first ring slot and the
// number of keys (at most the cache length, 128).
struct AttnWindow {
  int lo_slot, span;
};

__device__ __forceinline__ AttnWindow attn_window(int pos, int window, int cache) {
  int ws = 0;
  if (window > 0 && pos - window + 1 > 0) ws = pos - window + 1;
  const int lo = max(ws, pos - cache + 1);
  AttnWindow w;
  w.span = pos - lo + 1;
  w.lo_slot = lo % cache;
  return w;
}

// q rotated like the key reads: qr[f] = q4[(f + lane) % NF] (loaded ahead of the key wait).
template <int DH>
__device__ __forceinline__ void attn_load_q(const float* q, float4 (&qr)[DH / 4], int lane) {
#pragma unroll
  for (int f = 0; f < DH / 4; ++f) qr[f] = reinterpret_cast<const float4*>(q)[(f + lane) % (DH / 4)];
}

// Scores of the window's keys (lane i: keys lo+i, lo+i+32, ...; 16-byte columns in a per-lane
// rotation), the max shift, the reference's exp polynomial and one reciprocal: the softmax
// weights of the window's positions into pbuf[0..128).
template <int DH>
__device__ __forceinline__ void attn_scores(const float4 (&qr)[DH / 4], const float* Ks, AttnWindow w, int cache,
                                            float scale, float* pbuf, int lane) {
  constexpr int NF = DH / 4;
  float sc[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int j = lane + 32 * u;
    float acc = 0.f;
    if (j < w.span) {
      int sl = w.lo_slot + j;
      if (sl >= cache) sl -= cache;
      if (sl >= cache) sl -= cache;
      const float4* row = reinterpret_cast<const float4*>(Ks + (size_t)sl * DH);
#pragma unroll
      for (int f = 0; f < NF; ++f) {
        const float4 k4 = row[(f + lane) % NF];
        acc = __fmaf_rn(qr[f].x, k4.x, acc);
        acc = __fmaf_rn(qr[f].y, k4.y, acc);
        acc = __fmaf_rn(qr[f].z, k4.z, acc);
        acc = __fmaf_rn(qr[f].w, k4.w, acc);
      }
    }
    sc[u] = acc;
  }
  float mx = -3.402823466e38f;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    if (lane + 32 * u < w.span) {
      sc[u] = __fmul_rn(sc[u], scale);
      mx = fmaxf(mx, sc[u]);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    if (lane + 32 * u < w.span) {
      sc[u] = ref_vec_exp(__fsub_rn(sc[u], mx));
      sum = __fadd_rn(sum, sc[u]);
    } else {
      sc[u] = 0.f;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
  const float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
  for (int u = 0; u < 4; ++u) pbuf[lane + 32 * u] = __fmul_rn(sc[u], inv);
}

// The weighted sum of the window's values (lanes own (row group, 16-byte column) pairs; the groups
// combine on shuffles) into out[0..DH), and max |out| into *rowmax (atomic max of the float bits).
template <int DH>
__device__ __forceinline__ void attn_values(const float* Vs, const float* pbuf, AttnWindow w, int cache, float* out,
                                            float* rowmax, int lane) {
  constexpr int NF = DH / 4;  // float4 columns of a head row
  constexpr int G = 32 / NF;  // row groups
  const int c = lane % NF, g = lane / NF;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  if (g < G) {
    int sl = w.lo_slot + g;
    if (sl >= cache) sl -= cache;
    const float4* V4 = reinterpret_cast<const float4*>(Vs);
#pragma unroll 4
    for (int j = g; j < w.span; j += G) {
      const float p = pbuf[j];
      const float4 v = V4[(size_t)sl * NF + c];
      o.x = __fmaf_rn(p, v.x, o.x);
      o.y = __fmaf_rn(p, v.y, o.y);
      o.z = __fmaf_rn(p, v.z, o.z);
      o.w = __fmaf_rn(p, v.w, o.w);
      sl += G;
      if (sl >= cache) sl -= cache;
    }
  }
#pragma unroll
  for (int off = (G / 2) * NF; off >= NF; off >>= 1) {
    o.x = __fadd_rn(o.x, __shfl_down_sync(0xffffffffu, o.x, off));
    o.y = __fadd_rn(o.y, __shfl_down_sync(0xffffffffu, o.y, off));
    o.z = __fadd_rn(o.z, __shfl_down_sync(0xffffffffu, o.z, off));
    o.w = __fadd_rn(o.w, __shfl_down_sync(0xffffffffu, o.w, off));
  }
  float om = 0.f;
  if (lane < NF) {
    reinterpret_cast<float4*>(out)[lane] = o;
    om = fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w)));
  }
#pragma unroll
  for (int k = 16; k; k >>= 1) om = fmaxf(om, __shfl_xor_sync(0xffffffffu, om, k));
  if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(rowmax), __float_as_uint(om));
}

// Decode with the key/value windows staged in shared memory: a persistent grid (one CTA per SM)
// deals the (session, head) items to its warps round-robin, CTA-major. Each warp
// owns two shared-memory buffers, one for a key ring and one for a value ring (each one
// contiguous block in the head-major layout), each with its own mbarrier. Lane 0 of the warp
// fetches them with bulk copies: the keys of the next item as soon as this item's scores are
// done, its values as soon as this item's values are done. So a copy is always in flight while
// the warp computes, and every buffer has one producer and one consumer (the same warp), which
// waits on its phases in order.
//   scores  lane i scores window positions lo+i, lo+i+32, ... (its key rows, 16-byte columns
//           read in a per-lane rotation: conflict-free), one independent sum per key;
//   softmax the max shift, the reference's exp polynomial and one reciprocal, on warp shuffles;
//   values  the probabilities go to a per-warp shared buffer; lanes own (row group, 16-byte
//           column) pairs and accumulate float4 rows of their group, then the groups combine.
constexpr int kAsMaxWarps = 12;
constexpr size_t kAsSmemBudget = 200 * 1024;  // key/value buffers; the launch limit is kAsSmemMax
constexpr size_t kAsSmemMax = 227 * 1024;

struct AttnStaging {
  int warps = 0;
  size_t smem = 0;
};

inline size_t attn_staged_smem(int cache, int dh, int warps) {
  return 128 + (size_t)warps * (2 * (size_t)cache * dh * 4 + 128 * 4 + 2 * 8);
}

// Warps of the staged decode kernel (warps == 0: not usable; the bulk copies need 16-byte
// multiples, and the value phase's row groups, 32 / (dh / 4), a power of two).
inline AttnStaging attn_staging(int cache, int dh) {
  AttnStaging st;
  const size_t ring = (size_t)cache * dh * 4;
  if (ring % 16 != 0 || !(dh == 4 || dh == 8 || dh == 16 || dh == 32 || dh == 48 || dh == 64)) return st;
  int w = (int)((kAsSmemBudget - 1024) / (2 * ring));
  if (w > kAsMaxWarps) w = kAsMaxWarps;
  if (w < 1) return st;
  st.warps = w;
  st.smem = attn_staged_smem(cache, dh, w);
  return st;
}

template <int DH>  // head width (a multiple of 4, at most 64)
__global__ void __launch_bounds__(kAsMaxWarps * 32) attn_decode_staged_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  constexpr int NF = DH / 4;  // float4 columns of a head row
  const int cache = a.cache, D = a.D, heads = a.heads;
  const uint32_t ring_bytes = (uint32_t)(cache * DH * 4);
  const int nwarps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* Ks = reinterpret_cast<float*>(sm + (size_t)warp * 2 * ring_bytes);
  float* Vs = Ks + (size_t)cache * DH;
  float* pbuf = reinterpret_cast<float*>(sm + (size_t)nwarps * 2 * ring_bytes) + warp * 128;
  uint64_t* kfull = reinterpret_cast<uint64_t*>(sm + (size_t)nwarps * (2 * ring_bytes + 512)) + warp * 2;
  uint64_t* vfull = kfull + 1;
  // item m of this warp: base + stride * m (the whole grid walks the items in order, so the rings
  // read at any moment form one contiguous region)
  const int items = a.n_sess * heads;  // < 2^31 (checked by the launcher)
  const int base = blockIdx.x + gridDim.x * warp;
  const int stride = gridDim.x * nwarps;
  const int nm = base < items ? (int)((items - base + stride - 1) / stride) : 0;
  if (lane == 0) {
    mbar_init(kfull, 1);
    mbar_init(vfull, 1);
    fence_barrier_init();
  }
  __syncwarp();

  // lane 0: fetch the key (which 0) or value (1) ring of the warp's m-th item (an idle session:
  // arrival only). issued[which] counts the copies, for the final drain.
  int issued[2] = {0, 0};
  auto issue = [&](int m, int which) {
    if (m >= nm) return;
    issued[which] = m + 1;
    const int it = base + stride * m;
    const int s = it / heads, h = it - s * heads;
    uint64_t* bar = which ? vfull : kfull;
    if (a.seglen[s] <= 0) {
      mbar_arrive(bar);
      return;
    }
    const float* src = a.kv + ((size_t)a.attn_slot * a.n_sess + s) * 2 * (size_t)cache * D + (size_t)which * cache * D +
                       (size_t)h * cache * DH;
    mbar_arrive_expect_tx(bar, ring_bytes);
    bulk_load_hint(which ? Vs : Ks, src, ring_bytes, bar, l2_policy_evict_first());
  };
  if (lane == 0) {
    issue(0, 0);
    issue(0, 1);
  }

  bool healthy = true;  // false after a wait gave up: issue nothing more, drain what is in flight
  for (int m = 0; m < nm; ++m) {
    const int it = base + stride * m;
    const int s = it / heads, h = it - s * heads;
    const bool active = a.seglen[s] > 0;
    const AttnWindow w = attn_window(a.pos0[s], a.window, cache);
    const int grow = s;  // decode: the q and output row of session s is row s
    float4 qr[NF];
    if (active) attn_load_q<DH>(a.qbuf + (size_t)grow * D + h * DH, qr, lane);
    // ---- scores and softmax from the key ring ----
    bool got = __all_sync(0xffffffffu, healthy && mbar_wait_or_abort(kfull, m & 1, kErrWaitFull));
    if (!got) healthy = false;
    if (got && active) attn_scores<DH>(qr, Ks, w, cache, a.scale, pbuf, lane);
    __syncwarp();
    if (lane == 0 && healthy) issue(m + 1, 0);  // the key buffer is free: next item's keys
    // ---- values from the value ring ----
    got = __all_sync(0xffffffffu, healthy && mbar_wait_or_abort(vfull, m & 1, kErrWaitFull));
    if (!got) healthy = false;
    if (got && active) attn_values<DH>(Vs, pbuf, w, cache, a.att + (size_t)grow * D + h * DH, a.att_rowmax + grow, lane);
    __syncwarp();
    if (lane == 0 && healthy) issue(m + 1, 1);  // the value buffer is free: next item's values
  }
  // never leave with a copy still writing this warp's buffers (bounded waits; only an aborted wait
  // above can leave one): the last copy into each buffer was its phase issued - 1
  if (lane == 0) {
    if (issued[0] > 0) mbar_wait(kfull, (issued[0] - 1) & 1, kErrWaitFull);
    if (issued[1] > 0) mbar_wait(vfull, (issued[1] - 1) & 1, kErrWaitFull);
  }
}

// Prefill: one CTA per session. The segment's keys and values (written by the block kernel to
// kvlin, [t][K|V][D]) arrive in shared memory by one bulk copy; the warps take the (query, head)
// items in turn. Per item: lane i scores keys lo+i, lo+i+32, ... (16-byte columns in a per-lane
// rotation, q read as rotated 16-byte broadcasts), the softmax on warp shuffles, then lanes own
// (row group, 16-byte column) pairs of the value rows as in the staged decode kernel. max |o| of
// each row accumulates in shared memory across the heads.
template <int DH>  // head width: 4, 8, 16, 32, 48 or 64 (32 / (DH / 4) row groups, a power of two)
// Four CTAs per SM (64 registers) for head widths up to 32, whose segments are short enough to fit
// four in shared memory; two for wider heads (their rotated q rows need the registers).
__global__ void __launch_bounds__(kAttnThreads, DH <= 32 ? 4 : 2) attn_prefill_fast_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  float* sm = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  constexpr int NF = DH / 4;
  constexpr int G = 32 / NF;
  const int s = a.sess_list ? a.sess_list[blockIdx.x] : a.sess0 + (int)blockIdx.x;
  const int len = a.seglen[s];
  if (len <= 0) return;
  const int D = a.D, heads = a.heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float* kvs = sm;                                   // [len][2][D]
  float* pbuf = kvs + (size_t)len * 2 * D + warp * 128;
  unsigned int* rmax = reinterpret_cast<unsigned int*>(kvs + (size_t)len * 2 * D + nw * 128);  // [128]
  uint64_t* bar = reinterpret_cast<uint64_t*>(rmax + 128);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < 128; i += blockDim.x) rmax[i] = 0u;
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t bytes = (uint32_t)(len * 2 * D * 4);
    mbar_arrive_expect_tx(bar, bytes);
    bulk_load(kvs, a.kvlin + (size_t)s * a.P * 2 * D, bytes, bar);
  }
  const bool ok = __all_sync(0xffffffffu, mbar_wait_or_abort(bar, 0, kErrWaitFull));
  const int p0 = a.pos0[s];
  if (ok) {
    // last_only: the segment's keys and values are all staged (the last query's window needs them),
    // but only the last position's queries run
    const int t_first = a.last_only ? len - 1 : 0;
    for (int item = warp; item < (len - t_first) * heads; item += nw) {
      const int t = t_first + item / heads, h = item - (item / heads) * heads;
      const int pos = p0 + t;
      int ws = 0;
      if (a.window > 0 && pos - a.window + 1 > 0) ws = pos - a.window + 1;
      const int lo = max(max(ws, pos - a.cache + 1), p0) - p0;  // in-segment index of the first key
      const int span = t - lo + 1;                               // <= 128
      const int grow = grow_of(a, s, t);
      const float4* q4 = reinterpret_cast<const float4*>(a.qbuf + (size_t)grow * D + h * DH);
      float4 qr[NF];
#pragma unroll
      for (int f = 0; f < NF; ++f) qr[f] = q4[(f + lane) % NF];
      float sc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = lane + 32 * u;
        float acc = 0.f;
        if (j < span) {
          const float4* row = reinterpret_cast<const float4*>(kvs + (size_t)(lo + j) * 2 * D + h * DH);
#pragma unroll
          for (int f = 0; f < NF; ++f) {
            const float4 k4 = row[(f + lane) % NF];
            acc = __fmaf_rn(qr[f].x, k4.x, acc);
            acc = __fmaf_rn(qr[f].y, k4.y, acc);
            acc = __fmaf_rn(qr[f].z, k4.z, acc);
            acc = __fmaf_rn(qr[f].w, k4.w, acc);
          }
        }
        sc[u] = acc;
      }
      float mx = -3.402823466e38f;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (lane + 32 * u < span) {
          sc[u] = __fmul_rn(sc[u], a.scale);
          mx = fmaxf(mx, sc[u]);
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float sum = 0.f;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (lane + 32 * u < span) {
          sc[u] = ref_vec_exp(__fsub_rn(sc[u], mx));
          sum = __fadd_rn(sum, sc[u]);
        } else {
          sc[u] = 0.f;
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
      const float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
      for (int u = 0; u < 4; ++u) pbuf[lane + 32 * u] = __fmul_rn(sc[u], inv);
      __syncwarp();
      const int c = lane % NF, g = lane / NF;
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
      if (g < G) {
#pragma unroll 4
        for (int j = g; j < span; j += G) {
          const float p = pbuf[j];
          const float4 v = reinterpret_cast<const float4*>(kvs + (size_t)(lo + j) * 2 * D + D + h * DH)[c];
          o.x = __fmaf_rn(p, v.x, o.x);
          o.y = __fmaf_rn(p, v.y, o.y);
          o.z = __fmaf_rn(p, v.z, o.z);
          o.w = __fmaf_rn(p, v.w, o.w);
        }
      }
#pragma unroll
      for (int off = (G / 2) * NF; off >= NF; off >>= 1) {
        o.x = __fadd_rn(o.x, __shfl_down_sync(0xffffffffu, o.x, off));
        o.y = __fadd_rn(o.y, __shfl_down_sync(0xffffffffu, o.y, off));
        o.z = __fadd_rn(o.z, __shfl_down_sync(0xffffffffu, o.z, off));
        o.w = __fadd_rn(o.w, __shfl_down_sync(0xffffffffu, o.w, off));
      }
      float om = 0.f;
      if (lane < NF) {
        reinterpret_cast<float4*>(a.att + (size_t)grow * D + h * DH)[lane] = o;
        om = fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w)));
      }
#pragma unroll
      for (int k = 16; k; k >>= 1) om = fmaxf(om, __shfl_xor_sync(0xffffffffu, om, k));
      if (lane == 0) atomicMax(&rmax[t], __float_as_uint(om));
      __syncwarp();
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < len; t += blockDim.x) a.att_rowmax[grow_of(a, s, t)] = __uint_as_float(rmax[t]);
}

inline bool attn_prefill_fast_ok(int dh) { return dh == 4 || dh == 8 || dh == 16 || dh == 32 || dh == 48 || dh == 64; }

inline size_t attn_prefill_fast_smem(int P, int D) {
  return 128 + (size_t)P * 2 * D * 4 + (size_t)(kAttnThreads / 32) * 128 * 4 + 128 * 4 + 16;
}

// Prefill (head widths without a fast kernel): one CTA per session; the segment's keys and values
// (written by the block kernel to kvlin) are staged into shared memory; one warp per (query, head)
// item.
__global__ void __launch_bounds__(kAttnThreads) attn_prefill_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  float* sm = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int s = a.sess_list ? a.sess_list[blockIdx.x] : a.sess0 + (int)blockIdx.x;
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
