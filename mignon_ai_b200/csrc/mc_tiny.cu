// Whole-job greedy generation for small models without attention (config 1: D 64, H 128, two
// blocks, vocabulary 1024), one CTA per session.
//
// A batch of a few dozen sessions gives the tensor-core kernels one 128-row tile, so each decode
// step is a chain of latency-bound launches around a few thousand multiply-adds per session. Here
// one CTA carries its session through the prompt and every decode step in a single launch:
// appendPosition (internal/quant/stream.go:141-193) per token, then headLogits (:233-248) and
// argmaxProb (generate/greedy.go:90-102), with the blocks' int8 weights resident in shared
// memory. The products keep the engine's arithmetic: each GEMM input row is cut into the same
// three int8 digit planes (slice3_bits, the row's step from its largest magnitude), the plane dot
// products are exact int32 sums (dp4a, four int8 products per instruction), and dequant, bias,
// sigmoid, latch, GLU and highway are the same float operations as the decode kernel's epilogues.
// A decode step therefore produces the logits of block_decode_kernel; the prompt positions run
// the step-by-step recurrence (the reference's) where the batched prefill scans the latch in
// chunks, which differs by float rounding only.
#include "mc_engine.cuh"

namespace mc {
namespace eng {

constexpr int kTinyThreads = 128;
constexpr int kTinyMaxBlocks = 8;
constexpr int kTinyMaxD = 128;                 // the norms run on one warp, one float4 per lane
constexpr size_t kTinySmemMax = 200 * 1024;

struct TinyBlock {
  const uint32_t* w;  // [W_select rows | W1 rows | W2 rows], int8 rows padded to odd quad strides
  float s_sel, s1, s2;
  const float *b1, *b2, *gamma;
  int steps, bs0;
  int dil[kMaxSteps];
};

struct TinyArgs {
  int S, D, H, V, nblocks, total_steps, ring, P, n_new, out_stride;
  int kw_sel, kw1, kw2;  // row strides in 32-bit words: D/4, 3D/4, H/4, each made an odd number of quads
  int blk_words;         // words per block in w (a multiple of 4)
  const int8_t* embed;   // [V][D]: the embedding and the tied head
  float embed_scale, head_scale;
  const float *head_b, *final_gain, *latch_base;
  const int32_t* tok;    // [S][P] prompt segments (trimmed to the window)
  int32_t *seglen, *pos, *next_tok, *step;
  float *latch, *norm_ring;  // [S][total_steps][D], [S][total_steps][ring][D]
  int32_t* out_tok;
  float* out_prob;
  // append: one token per session (next_tok at position pos, the state carried in from global
  // memory) instead of a whole job; logits: each session's logits row [S][V] when not null
  int append;
  float* logits;
  TinyBlock blk[kTinyMaxBlocks];
};

// Row strides of the padded weight rows: an odd number of 16-byte quads, so that the eight rows a
// quarter-warp reads at once with 128-bit loads fall in eight different quad banks. k_bytes is a
// multiple of 16.
inline int tiny_stride_words(int k_bytes) {
  int q = k_bytes / 16;
  if (!(q & 1)) ++q;
  return 4 * q;
}

inline int tiny_block_words(int D, int H) {
  const int w = D * tiny_stride_words(D) + 2 * H * tiny_stride_words(3 * D) + 2 * D * tiny_stride_words(H);
  return (w + 3) & ~3;
}

// The logits row is padded to whole quads so that the digit planes after it are 16-byte aligned.
__host__ __device__ inline int tiny_vocab_pad(int V) { return (V + 3) & ~3; }

inline size_t tiny_smem_bytes(int D, int H, int V, int nblocks, int total_steps, int ring) {
  const int kwp = std::max(3 * D, H) / 4;
  return (size_t)nblocks * tiny_block_words(D, H) * 4 +
         ((size_t)total_steps * D * (1 + ring) + 4 * (size_t)D + H + tiny_vocab_pad(V)) * 4 + (size_t)3 * kwp * 4;
}

// The three digit planes of four consecutive values as one word per plane.
__device__ __forceinline__ void tiny_slice4(float4 v, float is, uint32_t* pl, int kwp, int word) {
  uint32_t a0, a1, a2, a3, b0, b1, b2, b3, c0, c1, c2, c3;
  slice3_bits(v.x, is, a0, b0, c0);
  slice3_bits(v.y, is, a1, b1, c1);
  slice3_bits(v.z, is, a2, b2, c2);
  slice3_bits(v.w, is, a3, b3, c3);
  pl[word] = pack_low_bytes(a0, a1, a2, a3);
  pl[kwp + word] = pack_low_bytes(b0, b1, b2, b3);
  pl[2 * kwp + word] = pack_low_bytes(c0, c1, c2, c3);
}

// Four words of one weight row against the same four words of the three planes.
__device__ __forceinline__ void tiny_dot4(uint4 x, uint4 y1, uint4 y2, uint4 y3, int& a1, int& a2, int& a3) {
  a1 = __dp4a((int)x.x, (int)y1.x, a1);
  a2 = __dp4a((int)x.x, (int)y2.x, a2);
  a3 = __dp4a((int)x.x, (int)y3.x, a3);
  a1 = __dp4a((int)x.y, (int)y1.y, a1);
  a2 = __dp4a((int)x.y, (int)y2.y, a2);
  a3 = __dp4a((int)x.y, (int)y3.y, a3);
  a1 = __dp4a((int)x.z, (int)y1.z, a1);
  a2 = __dp4a((int)x.z, (int)y2.z, a2);
  a3 = __dp4a((int)x.z, (int)y3.z, a3);
  a1 = __dp4a((int)x.w, (int)y1.w, a1);
  a2 = __dp4a((int)x.w, (int)y2.w, a2);
  a3 = __dp4a((int)x.w, (int)y3.w, a3);
}

// The three plane dot products of one padded weight row with the planes (nw words of K, a multiple
// of 4; the row and the planes 16-byte aligned): 128-bit shared-memory loads, four words per load.
__device__ __forceinline__ void tiny_dot(const uint32_t* w, const uint32_t* pl, int kwp, int nw, int& a1, int& a2, int& a3) {
  a1 = a2 = a3 = 0;
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
  const uint4* p1 = reinterpret_cast<const uint4*>(pl);
  const uint4* p2 = reinterpret_cast<const uint4*>(pl + kwp);
  const uint4* p3 = reinterpret_cast<const uint4*>(pl + 2 * kwp);
#pragma unroll 2
  for (int q = 0; q < nw / 4; ++q) tiny_dot4(w4[q], p1[q], p2[q], p3[q], a1, a2, a3);
}

__device__ __forceinline__ float4 ld4s(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4s(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

__global__ void __launch_bounds__(kTinyThreads, 1) tiny_generate_kernel(const __grid_constant__ TinyArgs a) {
  extern __shared__ __align__(16) uint32_t tsm[];
  __shared__ float s_step;
  __shared__ int s_next;
  __shared__ float red_v[kTinyThreads / 32];
  __shared__ int red_i[kTinyThreads / 32];
  __shared__ double red_d[kTinyThreads / 32];
  const int s = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (s == 0 && tid == 0) *a.step = a.n_new;  // the step counter as the batched job leaves it
  const int n = a.seglen[s];
  if (n <= 0) return;  // a session without a prompt (or finished) runs nothing, as in the batched kernels
  const int D = a.D, H = a.H, V = a.V, nf = D / 4;
  const int kwp = max(3 * D, H) / 4;
  // shared memory: the blocks' weights, the session state, the working rows, the digit planes
  uint32_t* sW = tsm;
  float* f = reinterpret_cast<float*>(tsm + (size_t)a.nblocks * a.blk_words);
  float* sLatch = f;
  f += (size_t)a.total_steps * D;
  float* sRing = f;
  f += (size_t)a.total_steps * a.ring * D;
  float* sCur = f;
  f += D;
  float* sIn = f;
  f += D;
  float* sNrm = f;
  f += D;
  float* sLam = f;
  f += D;
  float* sHid = f;
  f += H;
  float* sLog = f;
  f += tiny_vocab_pad(V);
  uint32_t* sPl = reinterpret_cast<uint32_t*>(f);  // 16-byte aligned: every region above is whole quads

  {
    const uint4* src = reinterpret_cast<const uint4*>(a.blk[0].w);  // the blocks' weights are one allocation
    uint4* dst = reinterpret_cast<uint4*>(sW);
    const int n4 = a.nblocks * a.blk_words / 4;
    for (int i = tid; i < n4; i += kTinyThreads) dst[i] = src[i];
    const size_t ring_n = (size_t)a.total_steps * a.ring * D;
    const float* gr = a.norm_ring + (size_t)s * ring_n;
    for (size_t i = tid; i < ring_n; i += kTinyThreads) sRing[i] = gr[i];
    // prefill resets the latch (quantSeqState.reset, stream.go:116-121); an append carries it on
    const float* gl = a.latch + (size_t)s * a.total_steps * D;
    for (int i = tid; i < a.total_steps * D; i += kTinyThreads) sLatch[i] = a.append ? gl[i] : 0.f;
  }
  __syncthreads();

  // RMSNorm of sCur with gain g (null: none) into out, by warp 0 as the decode kernel's norm_rows
  // does for one row; its digit planes (for a GEMM of K = D) into sPl and the step into s_step.
  auto norm_slice = [&](const float* g, float* out) {
    if (warp == 0) {
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      float4 x = lane < nf ? ld4s(sCur + 4 * lane) : z;
      float ss = 0.f;
      ss = __fmaf_rn(x.x, x.x, ss);
      ss = __fmaf_rn(x.y, x.y, ss);
      ss = __fmaf_rn(x.z, x.z, ss);
      ss = __fmaf_rn(x.w, x.w, ss);
      ss = warp_sum_d(ss);
      if (g) {
        const float inv = __fdiv_rn(1.0f, (float)sqrt((double)__fadd_rn(__fdiv_rn(ss, (float)D), 1e-5f)));
        const float4 gg = lane < nf ? ld4s(g + 4 * lane) : make_float4(1.f, 1.f, 1.f, 1.f);
        x.x = __fmul_rn(__fmul_rn(x.x, inv), gg.x);
        x.y = __fmul_rn(__fmul_rn(x.y, inv), gg.y);
        x.z = __fmul_rn(__fmul_rn(x.z, inv), gg.z);
        x.w = __fmul_rn(__fmul_rn(x.w, inv), gg.w);
      }
      if (out && lane < nf) st4s(out + 4 * lane, x);
      float m = lane < nf ? max4_d(x) : 0.f;
      m = warp_max_d(m);
      if (lane < nf) tiny_slice4(x, row_inv_step(m), sPl, kwp, lane);
      if (lane == 0) s_step = row_step(m);
    }
    __syncthreads();
  };

  // appendPosition of token tok at position pos; without need_out the last rule step of the last
  // block stops after its latch update (stream.go:176-178).
  auto append = [&](int tok, int pos, bool need_out) {
    if (tok < 0 || tok >= V) tok = 0;
    for (int d = tid; d < D; d += kTinyThreads) {
      const float y = __fmul_rn((float)a.embed[(size_t)tok * D + d], a.embed_scale);
      sCur[d] = y;
      sIn[d] = y;
    }
    __syncthreads();
    for (int b = 0; b < a.nblocks; ++b) {
      const TinyBlock& B = a.blk[b];
      const uint32_t* wsel = sW + (size_t)b * a.blk_words;
      const uint32_t* w1 = wsel + (size_t)D * a.kw_sel;
      const uint32_t* w2 = w1 + (size_t)2 * H * a.kw1;
      if (b > 0) {  // blockIn += cur; cur = blockIn (stream.go:158-163)
        for (int d = tid; d < D; d += kTinyThreads) {
          const float y = __fadd_rn(sIn[d], sCur[d]);
          sCur[d] = y;
          sIn[d] = y;
        }
        __syncthreads();
      }
      bool stop = false;
      for (int st = 0; st < B.steps && !stop; ++st) {
        const int bs = B.bs0 + st, dil = B.dil[st];
        float* ring = sRing + (size_t)bs * a.ring * D;
        float* latch = sLatch + (size_t)bs * D;
        // norm cell n, sliced for W_select
        norm_slice(B.gamma, sNrm);
        // lambda = sigmoid(W_select n s_sel + base)
        for (int r = tid; r < D; r += kTinyThreads) {
          const float base_r = a.latch_base[r];
          int x1, x2, x3;
          tiny_dot(wsel + (size_t)r * a.kw_sel, sPl, kwp, D / 4, x1, x2, x3);
          sLam[r] = sigmoid_clamped(__fadd_rn(dequant(x1, x2, x3, s_step, B.s_sel), base_r));
        }
        __syncthreads();
        // latch update, ring write, and x = [n | n(pos - dil) | latch] sliced for W1
        if (warp == 0) {
          const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
          float4 nv = z, lv = z, lf = z;
          if (lane < nf) {
            nv = ld4s(sNrm + 4 * lane);
            const float4 lam = ld4s(sLam + 4 * lane);
            const float4 o = pos > 0 ? ld4s(latch + 4 * lane) : z;
            lv.x = __fadd_rn(__fmul_rn(lam.x, o.x), __fmul_rn(__fsub_rn(1.0f, lam.x), nv.x));
            lv.y = __fadd_rn(__fmul_rn(lam.y, o.y), __fmul_rn(__fsub_rn(1.0f, lam.y), nv.y));
            lv.z = __fadd_rn(__fmul_rn(lam.z, o.z), __fmul_rn(__fsub_rn(1.0f, lam.z), nv.z));
            lv.w = __fadd_rn(__fmul_rn(lam.w, o.w), __fmul_rn(__fsub_rn(1.0f, lam.w), nv.w));
            if (pos - dil >= 0) lf = ld4s(ring + (size_t)((pos - dil) % a.ring) * D + 4 * lane);
            st4s(latch + 4 * lane, lv);
            st4s(ring + (size_t)(pos % a.ring) * D + 4 * lane, nv);
          }
          float m = lane < nf ? fmaxf(max4_d(nv), fmaxf(max4_d(lv), max4_d(lf))) : 0.f;
          m = warp_max_d(m);
          const float is = row_inv_step(m);
          if (lane < nf) {
            tiny_slice4(nv, is, sPl, kwp, lane);
            tiny_slice4(lf, is, sPl, kwp, nf + lane);
            tiny_slice4(lv, is, sPl, kwp, 2 * nf + lane);
          }
          if (lane == 0) s_step = row_step(m);
        }
        __syncthreads();
        if (!need_out && b == a.nblocks - 1 && st == B.steps - 1) {
          stop = true;
          continue;
        }
        // hidden = (W1v x s1 + b1v) * sigmoid(W1g x s1 + b1g)
        for (int h = tid; h < H; h += kTinyThreads) {
          const float bv = B.b1[h], bg = B.b1[H + h];
          int v1, v2, v3, g1, g2, g3;
          tiny_dot(w1 + (size_t)h * a.kw1, sPl, kwp, 3 * D / 4, v1, v2, v3);
          tiny_dot(w1 + (size_t)(H + h) * a.kw1, sPl, kwp, 3 * D / 4, g1, g2, g3);
          const float hv = __fadd_rn(dequant(v1, v2, v3, s_step, B.s1), bv);
          const float gt = __fadd_rn(dequant(g1, g2, g3, s_step, B.s1), bg);
          sHid[h] = __fmul_rn(hv, sigmoid_clamped(gt));
        }
        __syncthreads();
        // the hidden row sliced for W2
        if (warp == 0) {
          float m = 0.f;
          for (int q = lane; q < H / 4; q += 32) m = fmaxf(m, max4_d(ld4s(sHid + 4 * q)));
          m = warp_max_d(m);
          const float is = row_inv_step(m);
          for (int q = lane; q < H / 4; q += 32) tiny_slice4(ld4s(sHid + 4 * q), is, sPl, kwp, q);
          if (lane == 0) s_step = row_step(m);
        }
        __syncthreads();
        // o = W2 hidden s2 + b2; gate = sigmoid(o_gate); cur = (1 - gate) cur + gate o_delta
        for (int d = tid; d < D; d += kTinyThreads) {
          const float bd = B.b2[d], bg = B.b2[D + d];
          int v1, v2, v3, g1, g2, g3;
          tiny_dot(w2 + (size_t)d * a.kw2, sPl, kwp, H / 4, v1, v2, v3);
          tiny_dot(w2 + (size_t)(D + d) * a.kw2, sPl, kwp, H / 4, g1, g2, g3);
          const float od = __fadd_rn(dequant(v1, v2, v3, s_step, B.s2), bd);
          const float og = __fadd_rn(dequant(g1, g2, g3, s_step, B.s2), bg);
          const float gate = sigmoid_clamped(og);
          sCur[d] = __fadd_rn(__fmul_rn(__fsub_rn(1.0f, gate), sCur[d]), __fmul_rn(gate, od));
        }
        __syncthreads();
      }
    }
  };

  // headLogits + argmaxProb: the first index of the largest logit, probability 1 / sum exp(l - max)
  // in double; the token and probability go to output column col.
  auto head = [&](int col) {
    norm_slice(a.final_gain, nullptr);
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int v = tid; v < V; v += kTinyThreads) {
      const float hb = a.head_b[v];
      const uint32_t* e = reinterpret_cast<const uint32_t*>(a.embed + (size_t)v * D);
      int x1 = 0, x2 = 0, x3 = 0;
      for (int j0 = 0; j0 < D / 4; j0 += 4)  // D % 16 == 0: whole uint4s
        tiny_dot4(*reinterpret_cast<const uint4*>(e + j0), *reinterpret_cast<const uint4*>(sPl + j0),
                  *reinterpret_cast<const uint4*>(sPl + kwp + j0), *reinterpret_cast<const uint4*>(sPl + 2 * kwp + j0),
                  x1, x2, x3);
      const float l = __fadd_rn(dequant(x1, x2, x3, s_step, a.head_scale), hb);
      sLog[v] = l;
      if (a.logits) a.logits[(size_t)s * V + v] = l;
      if (l > bv || (l == bv && v < bi)) bv = l, bi = v;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
    }
    if (lane == 0) red_v[warp] = bv, red_i[warp] = bi;
    __syncthreads();
    bv = red_v[0];
    bi = red_i[0];
    for (int w = 1; w < kTinyThreads / 32; ++w)
      if (red_v[w] > bv || (red_v[w] == bv && red_i[w] < bi)) bv = red_v[w], bi = red_i[w];
    double sum = 0.0;
    for (int v = tid; v < V; v += kTinyThreads) sum += exp((double)sLog[v] - (double)bv);
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    __syncthreads();  // every thread has read red_v / red_i
    if (lane == 0) red_d[warp] = sum;
    __syncthreads();
    if (tid == 0) {
      double S = 0.0;
      for (int w = 0; w < kTinyThreads / 32; ++w) S += red_d[w];
      a.out_tok[(size_t)s * a.out_stride + col] = bi;
      a.out_prob[(size_t)s * a.out_stride + col] = (float)(1.0 / S);
      s_next = bi;
    }
    __syncthreads();
  };

  const int p_app = a.append ? a.pos[s] : 0;  // the pending token's position (read before any write)
  if (a.append) {
    append(a.next_tok[s], p_app, true);  // appendPosition of the pending token, then the head
    head(0);
  } else {
    for (int i = 0; i < n; ++i) append(a.tok[(size_t)s * a.P + i], i, i == n - 1);
    head(0);
    for (int k = 1; k < a.n_new; ++k) {
      append(s_next, n + k - 1, true);
      head(k);
    }
  }
  // the session continues as after the batched kernels: state, position, pending token
  {
    const size_t ring_n = (size_t)a.total_steps * a.ring * D;
    float* gr = a.norm_ring + (size_t)s * ring_n;
    for (size_t i = tid; i < ring_n; i += kTinyThreads) gr[i] = sRing[i];
    float* gl = a.latch + (size_t)s * a.total_steps * D;
    for (int i = tid; i < a.total_steps * D; i += kTinyThreads) gl[i] = sLatch[i];
    if (tid == 0) {
      a.pos[s] = a.append ? p_app + 1 : n + a.n_new - 1;
      a.seglen[s] = 1;
      a.next_tok[s] = s_next;
    }
  }
}

}  // namespace eng
}  // namespace mc
