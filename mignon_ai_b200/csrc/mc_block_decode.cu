// The decode block kernel: one CTA advances R sessions (16 or 32) by one position through one CA
// block.
//
// The arithmetic is block_kernel's (mc_block.cu) for one position per session, operation for
// operation, with the roles of the GEMM operands swapped. The weights are the MMA's M side (128
// output channels per tile) and the sessions its N side (R per CTA), so a batch of S sessions
// spreads over S/R CTAs (at state width 128: 256 CTAs of 16 sessions for 4096 sessions, two per
// multiprocessor, against 32 CTAs of 128 rows). The three digit planes of each K tile are
// stacked along N (plane p's rows follow plane p-1's), so one MMA of N = 3R computes all three
// plane accumulators: 3R TMEM columns per M-tile, four tiles in flight while the epilogue drains
// earlier ones. Each epilogue thread owns one output channel (TMEM lane) and
// R/4 sessions (TMEM columns). The GLU value/gate (W1) and highway delta/gate (W2) halves come
// from two consecutive M-tiles: their weight images hold 128 value rows, then the 128 matching
// gate rows. The sessions' rows (cur, the norm cell, the latch gate, the hidden layer) stay in
// shared memory for the whole block; only the session state (latch, norm ring, key/value ring)
// and the rows handed to the next kernel go through global memory.
//
// Roles: 16 row warps (row phases: one warp per session row; epilogues: thread = channel), one
// MMA warp (one elected thread issues tcgen05.mma), one producer warp (bulk copies of the
// pre-tiled weight tiles through a 6-stage ring, 3 stages at R = 16). All mbarrier waits are
// bounded.
#include "mc_engine.cuh"

namespace mc {
namespace eng {

constexpr int kDMaxR = 32;                       // sessions per CTA (MMA N): 32, or 16 for wide models
constexpr int kDRowWarps = 16;
constexpr int kDRowThreads = kDRowWarps * 32;
constexpr int kDThreads = kDRowThreads + 64;     // + MMA warp + producer warp
constexpr int kDMmaWarp = kDRowWarps;
constexpr int kDProducerWarp = kDRowWarps + 1;
constexpr int kDMaxWStages = 6;                  // weight-tile ring (16 KB tiles): 6, or 3 for wide models
constexpr int kDSlots = 4;                       // TMEM accumulator slots

struct DBars {
  uint64_t w_full[kDMaxWStages], w_empty[kDMaxWStages], s_full[kDSlots], s_empty[kDSlots], b_full;
  uint32_t tmem;
  int valid[kDMaxR], tok[kDMaxR], pos[kDMaxR];
  // attention blocks: offset in kv of each session's key ring row for its position (value ring
  // and other heads follow at fixed distances)
  unsigned long long kvoff[kDMaxR];
  float rstep[kDMaxR];  // step of each session row of the current GEMM's activation planes
  // fused head: per quadrant warp, each session's running (max, sum of exp, first argmax)
  float red_m[4][kDMaxR], red_s[4][kDMaxR];
  int red_i[4][kDMaxR];
};

constexpr size_t kDecodeSmemMax = 227 * 1024;  // the per-block opt-in limit of sm_100
constexpr size_t kSmemPerSm = 228 * 1024;      // shared memory of one sm_100 multiprocessor (1 KB reserved per CTA)

// Dynamic shared memory of the decode kernel for state width D, hidden width H, kt K tiles of
// activation planes (kt = ceil(max(3D, H) / 128)), R sessions per CTA and ws weight stages.
inline size_t decode_smem_bytes(int D, int H, int kt, int R, int ws) {
  return 1024 + (size_t)ws * kTile + (size_t)3 * kt * R * 128 + (size_t)4 * R * (2 * D + (D > H ? D : H)) + sizeof(DBars);
}

__device__ __forceinline__ void row_bar_d() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

__device__ __forceinline__ float warp_sum_d(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max_d(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float max4_d(float4 v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

// The three digit planes of four consecutive activations (K indices e..e+3, e % 4 == 0) of
// session row r, written into K tile e / 128 (one 32-bit store per plane). A K tile holds the
// planes stacked as one 3R-row operand: row p * R + r is plane p of session row r (R is a
// multiple of 8, so the 128-byte swizzle of row r is the same in every plane).
template <int R>
__device__ __forceinline__ void put_planes(uint8_t* sB, int r, int e, float4 v, float inv) {
  constexpr int kDBTile = R * 128;  // one digit plane of one K tile of the sessions
  uint8_t* tile = sB + (e >> 7) * 3 * kDBTile;
  const int k = e & 127;
  const uint32_t off = sw128_offset(r, k >> 4) + (k & 15);
  uint32_t a0, a1, a2, a3, b0, b1, b2, b3, c0, c1, c2, c3;
  slice3_bits(v.x, inv, a0, b0, c0);
  slice3_bits(v.y, inv, a1, b1, c1);
  slice3_bits(v.z, inv, a2, b2, c2);
  slice3_bits(v.w, inv, a3, b3, c3);
  *reinterpret_cast<uint32_t*>(tile + off) = pack_low_bytes(a0, a1, a2, a3);
  *reinterpret_cast<uint32_t*>(tile + kDBTile + off) = pack_low_bytes(b0, b1, b2, b3);
  *reinterpret_cast<uint32_t*>(tile + 2 * kDBTile + off) = pack_low_bytes(c0, c1, c2, c3);
}

// M-tiles whose MMAs the decode kernel interleaves: the value/gate pairs of W1 and W2 (their
// epilogue needs both tiles at once: two independent accumulation chains in flight finish the pair
// sooner than one chain after the other); single tiles otherwise.
__device__ __forceinline__ int decode_mma_group(const GemmSpec& G) { return (G.type == kGW1 || G.type == kGW2) ? 2 : 1; }

// CTAs of the decode kernel resident on one multiprocessor: two for 16 sessions per CTA at state
// widths up to 128 (each then holds half of the TMEM and at most 56 registers per thread), so the
// latency chains of two CTAs interleave; one otherwise.
__host__ __device__ constexpr int decode_ctas_per_sm(int kf, int r) { return (r == 16 && kf == 1) ? 2 : 1; }

// Shared memory of a decode CTA: the weight ring, the sessions' activation planes, the norm and
// auxiliary rows, the cur rows, then the barriers.
struct DecodeLayout {
  uint8_t* sW;   // [WS][128 x 128] weight tiles
  uint8_t* sB;   // [KT][3 planes][R rows x 128] activation planes, stacked along N
  float* sNrm;   // [R][D] norm cell
  float* sAux;   // [R][max(D, H)] latch gate, then hidden
  float* sCur;   // [R][D] the block's state rows
  DBars* bars;
};

template <int R, int WS>
__device__ __forceinline__ DecodeLayout decode_layout(uint8_t* smem_raw, int D, int H, int KT) {
  DecodeLayout L;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int DH = D > H ? D : H;
  L.sW = smem;
  L.sB = L.sW + WS * kTile;
  L.sNrm = reinterpret_cast<float*>(L.sB + 3 * KT * R * 128);
  L.sAux = L.sNrm + R * D;
  L.sCur = L.sAux + R * DH;
  L.bars = reinterpret_cast<DBars*>(L.sCur + R * D);
  return L;
}

// One thread's running state through a block: ring and slot counters, the GEMMs whose planes
// were published, trace points, and whether every wait so far succeeded (after a wait gave up,
// the thread skips all further waits, so a failure costs one wait limit).
struct DecodeRun {
  uint32_t widx = 0, sidx = 0, gidx = 0;
  int tp = 0;
  bool ok = true;
};

template <int KF, int R, int WS>
__device__ __forceinline__ void decode_init(const DecodeLayout& L) {
  DBars* bars = L.bars;
  if (threadIdx.x == 0) {
    for (int i = 0; i < WS; ++i) {
      mbar_init(&bars->w_full[i], 1);
      mbar_init(&bars->w_empty[i], 1);
    }
    for (int i = 0; i < kDSlots; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_empty[i], kDRowWarps);
    }
    mbar_init(&bars->b_full, kDRowThreads);
    fence_barrier_init();
  }
}

// One CA block for the CTA's R sessions, every role (weight producer, MMA issuer, row warps)
// with its running state.
template <int KF, int R, int WS>
__device__ __forceinline__ void decode_block(const BlockArgs& a, const DecodeLayout& L, uint32_t tmem, DecodeRun& run) {
  constexpr int kDR = R;
  constexpr int kDWStages = WS;
  constexpr int kDBTile = R * 128;               // one digit plane of one K tile of the sessions
  constexpr int kDRowsPerWarp = R / kDRowWarps;  // session rows per row warp
  constexpr int kDCols = R / 4;                  // sessions per epilogue thread
  constexpr int kDSlotCols = R == 32 ? 128 : 64; // three planes of R columns, padded
  const int D = a.D, H = a.H;
  uint8_t* sW = L.sW;
  uint8_t* sB = L.sB;
  float* sCur = L.sCur;
  float* sNrm = L.sNrm;
  float* sAux = L.sAux;
  DBars* bars = L.bars;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int s0 = blockIdx.x * kDR;
  // the row warps run on after a failed wait (skipping every wait and epilogue) so that they all
  // meet at each of their named barriers
  if (!run.ok && warp >= kDRowWarps) return;

  if (warp == kDProducerWarp) {
    // ---------------- weight tiles, in the order the MMA warp consumes them ----------------
    if (lane == 0) {
      uint32_t& widx = run.widx;
      bool& ok = run.ok;
      const uint64_t policy = l2_policy_evict_last();
      uint32_t st = widx % kDWStages, ph = (widx / kDWStages) & 1;  // stage, and the parity of its fill
      for (int g = 0; g < a.ngemms && ok; ++g) {
        const GemmSpec& G = a.gemms[g];
        const int gs = decode_mma_group(G);
        for (int c0 = 0; c0 < G.nchunks && ok; c0 += gs)
          for (int kt = 0; kt < G.ktiles && ok; ++kt)
            for (int c = c0; c < c0 + gs && c < G.nchunks; ++c, ++widx) {
              // the stage's previous fill (parity ph ^ 1) has been consumed
              if (widx >= kDWStages && !mbar_wait_or_abort(&bars->w_empty[st], ph ^ 1, kErrWaitEmpty)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&bars->w_full[st], kTile);
              bulk_load_hint(sW + st * kTile, G.tiles + ((size_t)c * G.ktiles + kt) * kTile, kTile, &bars->w_full[st],
                             policy);
              if (++st == kDWStages) {
                st = 0;
                ph ^= 1;
              }
            }
      }
    }
  } else if (warp == kDMmaWarp) {
    // ---------------- MMA issuer: D[channel][session] += W[channel][k] * X[session][k] ----------------
    if (lane == 0) {
      uint32_t& widx = run.widx;
      uint32_t& sidx = run.sidx;
      const uint32_t idesc = idesc_i8(128, 3 * kDR);  // the three planes stacked along N
      const uint64_t desc_w0 = smem_desc_sw128(sW), desc_b0 = smem_desc_sw128(sB);
      bool& ok = run.ok;
      for (int g = 0; g < a.ngemms && ok; ++g) {
        const GemmSpec& G = a.gemms[g];
        if (!mbar_wait_or_abort(&bars->b_full, (run.gidx++) & 1, kErrWaitFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // gs M-tiles at a time (a value/gate pair: two independent accumulation chains, their
        // MMAs alternating K step by K step), each in its own TMEM slot
        const int gs = decode_mma_group(G);
        for (int c0 = 0; c0 < G.nchunks && ok; c0 += gs) {
          const int n = min(gs, G.nchunks - c0);
          for (int q = 0; q < n && ok; ++q) {
            const uint32_t si = sidx + q;
            if (si >= kDSlots && !mbar_wait_or_abort(&bars->s_empty[si % kDSlots], ((si / kDSlots) - 1) & 1, kErrWaitAccFree))
              ok = false;
          }
          if (!ok) break;
          tc_fence_after();
          // descriptors advance by their encoded start address (bytes / 16): a weight stage is
          // kTile bytes, a K tile of the planes 3 * kDBTile
          const uint32_t dt0 = tmem + (sidx % kDSlots) * kDSlotCols;
          const uint32_t dt1 = tmem + ((sidx + 1) % kDSlots) * kDSlotCols;
          uint32_t st = widx % kDWStages, ph = (widx / kDWStages) & 1;
          for (int kt = 0; kt < G.ktiles && ok; ++kt) {
            const uint64_t db = desc_b0 + (uint64_t)(kt * (3 * kDBTile >> 4));
            const int ksteps = min(4, (G.K - kt * 128 + 31) / 32);
            for (int q = 0; q < n; ++q, ++widx) {
              if (!mbar_wait_or_abort(&bars->w_full[st], ph, kErrWaitFull)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t da = desc_w0 + (uint64_t)(st * (kTile >> 4));
              const uint32_t dt = q == 0 ? dt0 : dt1;
              if (ksteps == 4) {
                mma_i8(dt, da, db, idesc, kt > 0 ? 1u : 0u);
                mma_i8(dt, da + 2, db + 2, idesc, 1u);
                mma_i8(dt, da + 4, db + 4, idesc, 1u);
                mma_i8(dt, da + 6, db + 6, idesc, 1u);
              } else {
                for (int kk = 0; kk < ksteps; ++kk)
                  mma_i8(dt, da + 2 * kk, db + 2 * kk, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
              }
              mma_commit(&bars->w_empty[st]);
              if (++st == kDWStages) {
                st = 0;
                ph ^= 1;
              }
            }
          }
          if (!ok) break;
          for (int q = 0; q < n; ++q) mma_commit(&bars->s_full[(sidx + q) % kDSlots]);
          sidx += n;
        }
      }
    }
  } else {
    // ---------------- row warps ----------------
    const int t = threadIdx.x;
    const int chl = 32 * (warp & 3) + lane;  // channel within an M-tile = TMEM lane
    const int r0 = kDCols * (warp >> 2);      // first of this thread's epilogue sessions = TMEM column
    const int nf = D / 4;
    uint32_t& sidx = run.sidx;
    bool& ok = run.ok;
    int& tp = run.tp;
    trace_point(a, tp++);
    if (t < kDR) {
      const int s = s0 + t;
      const bool v = s < a.n_sess && a.seglen[s] > 0;
      bars->valid[t] = v ? 1 : 0;
      bars->pos[t] = v ? a.pos0[s] : 0;
      if (a.has_attn && v)
        bars->kvoff[t] = ((size_t)a.attn_slot * a.n_sess + s) * 2 * (size_t)a.cache * D + (size_t)(a.pos0[s] % a.cache) * a.dh;
      int tok = 0;
      if (v && a.embed_first) {
        tok = a.tokens[s];
        if (tok < 0 || tok >= a.V) tok = 0;
      }
      bars->tok[t] = tok;
    }
    row_bar_d();

    auto publish = [&]() {
      fence_proxy_async_smem();
      mbar_arrive(&bars->b_full);
      row_bar_d();
    };
    auto wait_slot = [&](int slot, uint32_t k) {
      const bool got =
          __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&bars->s_full[slot], (k / kDSlots) & 1, kErrWaitAcc));
      if (!got) ok = false;
      tc_fence_after();
    };
    auto release_slot = [&](int slot) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->s_empty[slot]);
    };
    // this thread's three plane accumulators of a slot: loads issued (acc_issue), then waited for
    auto acc_issue = [&](int slot, uint32_t(&x1)[kDCols], uint32_t(&x2)[kDCols], uint32_t(&x3)[kDCols]) {
      const uint32_t base = tmem_addr(tmem, 32 * (warp & 3), slot * kDSlotCols + r0);
      if constexpr (kDCols == 8) {
        tmem_ld8(base, x1);
        tmem_ld8(base + kDR, x2);
        tmem_ld8(base + 2 * kDR, x3);
      } else {
        tmem_ld4(base, x1);
        tmem_ld4(base + kDR, x2);
        tmem_ld4(base + 2 * kDR, x3);
      }
    };
    auto acc8 = [&](int slot, uint32_t(&x1)[kDCols], uint32_t(&x2)[kDCols], uint32_t(&x3)[kDCols]) {
      acc_issue(slot, x1, x2, x3);
      tmem_wait_ld();
    };
    auto load_steps = [&](float(&stp)[kDCols]) {
#pragma unroll
      for (int j = 0; j < kDCols; ++j) stp[j] = bars->rstep[r0 + j];
    };
    // The M-tiles of one GEMM, one accumulator each: fn(tile, steps, planes).
    // pre(tile) returns the tile's per-channel vectors (biases), loaded before the accumulator
    // wait so that their latency overlaps it; the epilogue reads them from pv.
    float2 pv = make_float2(0.f, 0.f);
    auto tiles1 = [&](const GemmSpec& G, auto&& pre, auto&& fn) {
      float stp[kDCols];
      load_steps(stp);
      for (int c = 0; c < G.nchunks; ++c, ++sidx) {
        const int slot = sidx % kDSlots;
        pv = pre(c);
        wait_slot(slot, sidx);
        if (a.trace_fine) trace_point(a, tp++);
        uint32_t x1[kDCols], x2[kDCols], x3[kDCols];
        acc8(slot, x1, x2, x3);
        release_slot(slot);
        fn(c, stp, x1, x2, x3);
        if (a.trace_fine) trace_point(a, tp++);
      }
    };
    // Pairs of M-tiles (value/delta tile, gate tile): fn(pair, steps, value planes, gate planes).
    auto tiles2 = [&](const GemmSpec& G, auto&& pre, auto&& fn) {
      float stp[kDCols];
      load_steps(stp);
      for (int c = 0; c + 1 < G.nchunks; c += 2, sidx += 2) {
        const int sv = sidx % kDSlots, sg = (sidx + 1) % kDSlots;
        uint32_t v1[kDCols], v2[kDCols], v3[kDCols], g1[kDCols], g2[kDCols], g3[kDCols];
        pv = pre(c / 2);
        wait_slot(sv, sidx);
        wait_slot(sg, sidx + 1);  // the pair's MMAs complete together
        if (a.trace_fine) trace_point(a, tp++);
        acc_issue(sv, v1, v2, v3);
        acc_issue(sg, g1, g2, g3);
        tmem_wait_ld();
        release_slot(sv);
        release_slot(sg);
        fn(c / 2, stp, v1, v2, v3, g1, g2, g3);
        if (a.trace_fine) trace_point(a, tp++);
      }
    };
    // RMSNorm (nn/rmsnorm.go:14-32) of the cur rows with gain `gain` (null: identity, no norm).
    // Writes the result to `out` (shared or global rows of stride D; null: none), max |y| of the
    // row to rmax_g (global, if given), and if slice its digit planes as the next GEMM's input.
    auto norm_rows = [&](const float* gain, float* out, bool out_global, float* rmax_g, bool slice) {
#pragma unroll
      for (int u = 0; u < kDRowsPerWarp; ++u) {
        const int rr = warp + kDRowWarps * u;
        const int s = s0 + rr;
        const bool v = bars->valid[rr] != 0;
        float4 x[KF], gg[KF];
        const float4* c4 = reinterpret_cast<const float4*>(sCur + rr * D);
#pragma unroll
        for (int k = 0; k < KF; ++k) {
          const int f = lane + 32 * k;
          x[k] = (v && f < nf) ? c4[f] : make_float4(0.f, 0.f, 0.f, 0.f);
          gg[k] = (gain && f < nf) ? reinterpret_cast<const float4*>(gain)[f] : make_float4(1.f, 1.f, 1.f, 1.f);
        }
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < KF; ++k) {
          ss = __fmaf_rn(x[k].x, x[k].x, ss);
          ss = __fmaf_rn(x[k].y, x[k].y, ss);
          ss = __fmaf_rn(x[k].z, x[k].z, ss);
          ss = __fmaf_rn(x[k].w, x[k].w, ss);
        }
        ss = warp_sum_d(ss);
        float inv = 1.f;
        if (gain) inv = __fdiv_rn(1.0f, (float)sqrt((double)__fadd_rn(__fdiv_rn(ss, (float)D), 1e-5f)));
        float m = 0.f;
        float4* o4 = out ? reinterpret_cast<float4*>(out + (size_t)(out_global ? s : rr) * D) : nullptr;
#pragma unroll
        for (int k = 0; k < KF; ++k) {
          const int f = lane + 32 * k;
          if (f < nf && gain) {
            x[k].x = __fmul_rn(__fmul_rn(x[k].x, inv), gg[k].x);
            x[k].y = __fmul_rn(__fmul_rn(x[k].y, inv), gg[k].y);
            x[k].z = __fmul_rn(__fmul_rn(x[k].z, inv), gg[k].z);
            x[k].w = __fmul_rn(__fmul_rn(x[k].w, inv), gg[k].w);
          }
          if (o4 && f < nf && (v || !out_global)) o4[f] = x[k];
          if (f < nf) m = fmaxf(m, max4_d(x[k]));
        }
        m = v ? warp_max_d(m) : 0.f;
        if (lane == 0) {
          bars->rstep[rr] = row_step(m);
          if (rmax_g && s < a.n_sess) rmax_g[s] = m;
        }
        if (slice) {
          const float is = row_inv_step(m);
#pragma unroll
          for (int k = 0; k < KF; ++k) {
            const int f = lane + 32 * k;
            if (f < nf) put_planes<R>(sB, rr, 4 * f, x[k], is);
          }
        }
      }
    };

    int gi = 0;
    // ---- the sessions' cur rows: the token embedding (block 0) or the previous block's output ----
#pragma unroll
    for (int u = 0; u < kDRowsPerWarp; ++u) {
      const int rr = warp + kDRowWarps * u;
      const int s = s0 + rr;
      const bool v = bars->valid[rr] != 0;
      float4* c4 = reinterpret_cast<float4*>(sCur + rr * D);
      const char4* e4 = reinterpret_cast<const char4*>(a.embed + (size_t)bars->tok[rr] * D);
      const float4* g4 = reinterpret_cast<const float4*>(a.cur + (size_t)s * D);
#pragma unroll
      for (int k = 0; k < KF; ++k) {
        const int f = lane + 32 * k;
        if (f >= nf) continue;
        float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
        if (v) {
          if (a.embed_first) {
            const char4 q = e4[f];
            y = make_float4(__fmul_rn((float)q.x, a.embed_scale), __fmul_rn((float)q.y, a.embed_scale),
                            __fmul_rn((float)q.z, a.embed_scale), __fmul_rn((float)q.w, a.embed_scale));
            reinterpret_cast<float4*>(a.blockin + (size_t)s * D)[f] = y;
          } else {
            y = g4[f];
          }
        }
        c4[f] = y;
      }
    }

    trace_point(a, tp++);
    // ---- output projection of the previous block's attention: cur += Out att s_out ----
    if (a.has_out) {
#pragma unroll
      for (int u = 0; u < kDRowsPerWarp; ++u) {
        const int rr = warp + kDRowWarps * u;
        const int s = s0 + rr;
        const bool v = bars->valid[rr] != 0;
        const float m = v ? a.att_rowmax[s] : 0.f;
        const float is = row_inv_step(m);
        if (lane == 0) bars->rstep[rr] = row_step(m);
        const float4* a4 = reinterpret_cast<const float4*>(a.att + (size_t)s * D);
#pragma unroll
        for (int k = 0; k < KF; ++k) {
          const int f = lane + 32 * k;
          if (f < nf) put_planes<R>(sB, rr, 4 * f, v ? a4[f] : make_float4(0.f, 0.f, 0.f, 0.f), is);
        }
      }
      publish();
      trace_point(a, tp++);
      tiles1(a.gemms[gi++], [](int) { return make_float2(0.f, 0.f); }, [&](int c, const float(&stp)[kDCols], uint32_t(&x1)[kDCols], uint32_t(&x2)[kDCols],
                                uint32_t(&x3)[kDCols]) {
        const int n = c * 128 + chl;
        if (n >= D) return;
#pragma unroll
        for (int j = 0; j < kDCols; ++j) {
          const int rr = r0 + j;
          if (!bars->valid[rr]) continue;
          float* p = sCur + rr * D + n;
          *p = __fadd_rn(*p, dequant(x1[j], x2[j], x3[j], stp[j], a.gemms[gi - 1].scale));
        }
      });
      row_bar_d();
    }

    // ---- inter-block residual: blockIn += cur; cur = blockIn (stream.go:158-163) ----
    if (a.residual && !a.embed_first) {
#pragma unroll
      for (int u = 0; u < kDRowsPerWarp; ++u) {
        const int rr = warp + kDRowWarps * u;
        const int s = s0 + rr;
        if (!bars->valid[rr]) continue;
        float4* c4 = reinterpret_cast<float4*>(sCur + rr * D);
        float4* b4 = reinterpret_cast<float4*>(a.blockin + (size_t)s * D);
#pragma unroll
        for (int k = 0; k < KF; ++k) {
          const int f = lane + 32 * k;
          if (f >= nf) continue;
          const float4 b = b4[f], c = c4[f];
          const float4 y = make_float4(__fadd_rn(b.x, c.x), __fadd_rn(b.y, c.y), __fadd_rn(b.z, c.z), __fadd_rn(b.w, c.w));
          c4[f] = y;
          b4[f] = y;
        }
      }
      row_bar_d();
    }

    // ---- rule steps ----
    for (int st = 0; st < a.nsteps; ++st) {
      const int bs = a.bs0 + st;
      const int dil = a.dil[st];
      // the session state this step reads (latch, left neighbour in the norm ring), fetched now
      float4 lo[kDRowsPerWarp][KF], lf[kDRowsPerWarp][KF];
#pragma unroll
      for (int u = 0; u < kDRowsPerWarp; ++u) {
        const int rr = warp + kDRowWarps * u;
        const int s = s0 + rr;
        const bool v = bars->valid[rr] != 0;
        const int pos = bars->pos[rr];
        const size_t so = (size_t)s * a.total_steps + bs;
        const float4* ls4 = reinterpret_cast<const float4*>(a.latch + so * D);
        const float4* ring4 = reinterpret_cast<const float4*>(a.norm_ring + so * a.ring * D);
        const int lpos = pos - dil;
#pragma unroll
        for (int k = 0; k < KF; ++k) {
          const int f = lane + 32 * k;
          const bool in = v && f < nf;
          const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
          lo[u][k] = (in && pos > 0) ? ls4[f] : z;
          lf[u][k] = (in && lpos >= 0) ? ring4[(size_t)(lpos % a.ring) * nf + f] : z;
        }
      }
      // norm cell n, kept in shared memory and sliced for W_select
      trace_point(a, tp++);
      norm_rows(a.gamma, sNrm, false, nullptr, true);
      publish();
      trace_point(a, tp++);
      // lambda = sigmoid(W_select n s_sel + base), into the latch-gate rows
      tiles1(a.gemms[gi++], [&](int c) {
        const int n = c * 128 + chl;
        return make_float2(n < D ? a.latch_base[n] : 0.f, 0.f);
      }, [&](int c, const float(&stp)[kDCols], uint32_t(&x1)[kDCols], uint32_t(&x2)[kDCols], uint32_t(&x3)[kDCols]) {
        const int n = c * 128 + chl;
        if (n >= D) return;
        const float base = pv.x;
        const float scale = a.gemms[gi - 1].scale;
#pragma unroll
        for (int j = 0; j < kDCols; ++j)
          sAux[(r0 + j) * D + n] = sigmoid_clamped(__fadd_rn(dequant(x1[j], x2[j], x3[j], stp[j], scale), base));
      });
      row_bar_d();
      trace_point(a, tp++);
      // latch update, ring write, and x = [n | n(pos - dil) | latch] sliced for W1
#pragma unroll
      for (int u = 0; u < kDRowsPerWarp; ++u) {
        const int rr = warp + kDRowWarps * u;
        const int s = s0 + rr;
        const bool v = bars->valid[rr] != 0;
        const int pos = bars->pos[rr];
        const size_t so = (size_t)s * a.total_steps + bs;
        float4* ls4 = reinterpret_cast<float4*>(a.latch + so * D);
        float4* ring4 = reinterpret_cast<float4*>(a.norm_ring + so * a.ring * D);
        const float4* n4 = reinterpret_cast<const float4*>(sNrm + rr * D);
        const float4* l4 = reinterpret_cast<const float4*>(sAux + rr * D);
        float4 nv[KF], lv[KF];
        float m = 0.f;
#pragma unroll
        for (int k = 0; k < KF; ++k) {
          const int f = lane + 32 * k;
          const bool in = v && f < nf;
          const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
          nv[k] = in ? n4[f] : z;
          const float4 lam = in ? l4[f] : z;
          const float4 o = lo[u][k];
          float4 l;
          l.x = __fadd_rn(__fmul_rn(lam.x, o.x), __fmul_rn(__fsub_rn(1.0f, lam.x), nv[k].x));
          l.y = __fadd_rn(__fmul_rn(lam.y, o.y), __fmul_rn(__fsub_rn(1.0f, lam.y), nv[k].y));
          l.z = __fadd_rn(__fmul_rn(lam.z, o.z), __fmul_rn(__fsub_rn(1.0f, lam.z), nv[k].z));
          l.w = __fadd_rn(__fmul_rn(lam.w, o.w), __fmul_rn(__fsub_rn(1.0f, lam.w), nv[k].w));
          lv[k] = l;
          if (in) {
            ls4[f] = l;
            ring4[(size_t)(pos % a.ring) * nf + f] = nv[k];
          }
          if (f < nf) m = fmaxf(m, fmaxf(max4_d(nv[k]), fmaxf(max4_d(l), max4_d(lf[u][k]))));
        }
        m = v ? warp_max_d(m) : 0.f;
        if (lane == 0) bars->rstep[rr] = row_step(m);
        const float is = row_inv_step(m);
#pragma unroll
        for (int k = 0; k < KF; ++k) {
          const int f = lane + 32 * k;
          if (f < nf) {
            put_planes<R>(sB, rr, 4 * f, nv[k], is);
            put_planes<R>(sB, rr, D + 4 * f, lf[u][k], is);
            put_planes<R>(sB, rr, 2 * D + 4 * f, lv[k], is);
          }
        }
      }
      publish();
      trace_point(a, tp++);
      // hidden = (W1v x s1 + b1v) * sigmoid(W1g x s1 + b1g)   (applyRule layer 1, stream.go:212-220)
      tiles2(a.gemms[gi++], [&](int c) {
        const int hu = c * 128 + chl;
        return hu < H ? make_float2(a.b1[hu], a.b1[H + hu]) : make_float2(0.f, 0.f);
      }, [&](int c, const float(&stp)[kDCols], uint32_t(&v1)[kDCols], uint32_t(&v2)[kDCols], uint32_t(&v3)[kDCols],
             uint32_t(&g1)[kDCols], uint32_t(&g2)[kDCols], uint32_t(&g3)[kDCols]) {
        const int hu = c * 128 + chl;
        if (hu >= H) return;
        const float bv = pv.x, bg = pv.y;
        const float scale = a.gemms[gi - 1].scale;
#pragma unroll
        for (int j = 0; j < kDCols; ++j) {
          const float hv = __fadd_rn(dequant(v1[j], v2[j], v3[j], stp[j], scale), bv);
          const float gt = __fadd_rn(dequant(g1[j], g2[j], g3[j], stp[j], scale), bg);
          sAux[(r0 + j) * H + hu] = __fmul_rn(hv, sigmoid_clamped(gt));
        }
      });
      row_bar_d();
      trace_point(a, tp++);
      // the hidden rows sliced for W2 (max |hidden| of each row)
      {
        const int hf = H / 4;
#pragma unroll
        for (int u = 0; u < kDRowsPerWarp; ++u) {
          const int rr = warp + kDRowWarps * u;
          const bool v = bars->valid[rr] != 0;
          const float4* h4 = reinterpret_cast<const float4*>(sAux + rr * H);
          float m = 0.f;
          for (int f = lane; f < hf; f += 32) m = fmaxf(m, max4_d(h4[f]));
          m = v ? warp_max_d(m) : 0.f;
          if (lane == 0) bars->rstep[rr] = row_step(m);
          const float is = row_inv_step(m);
          for (int f = lane; f < hf; f += 32) put_planes<R>(sB, rr, 4 * f, v ? h4[f] : make_float4(0.f, 0.f, 0.f, 0.f), is);
        }
      }
      publish();
      trace_point(a, tp++);
      // o = W2 hidden s2 + b2; gate = sigmoid(o_gate); cur = (1 - gate) cur + gate o_delta (:222-229)
      tiles2(a.gemms[gi++], [&](int c) {
        const int d = c * 128 + chl;
        return d < D ? make_float2(a.b2[d], a.b2[D + d]) : make_float2(0.f, 0.f);
      }, [&](int c, const float(&stp)[kDCols], uint32_t(&v1)[kDCols], uint32_t(&v2)[kDCols], uint32_t(&v3)[kDCols],
             uint32_t(&g1)[kDCols], uint32_t(&g2)[kDCols], uint32_t(&g3)[kDCols]) {
        const int d = c * 128 + chl;
        if (d >= D) return;
        const float bd = pv.x, bg = pv.y;
        const float scale = a.gemms[gi - 1].scale;
#pragma unroll
        for (int j = 0; j < kDCols; ++j) {
          const int rr = r0 + j;
          if (!bars->valid[rr]) continue;
          const float od = __fadd_rn(dequant(v1[j], v2[j], v3[j], stp[j], scale), bd);
          const float og = __fadd_rn(dequant(g1[j], g2[j], g3[j], stp[j], scale), bg);
          const float gate = sigmoid_clamped(og);
          float* p = sCur + rr * D + d;
          *p = __fadd_rn(__fmul_rn(__fsub_rn(1.0f, gate), *p), __fmul_rn(gate, od));
        }
      });
      row_bar_d();
    }

    // ---- attention sublayer: norm (sliced for QKV) + QKV, keys/values into the ring ----
    if (a.has_attn) {
      norm_rows(a.attn_norm, nullptr, false, nullptr, true);
      if (lane == 0) {
#pragma unroll
        for (int u = 0; u < kDRowsPerWarp; ++u) {
          const int rr = warp + kDRowWarps * u;
          if (bars->valid[rr]) a.att_rowmax[s0 + rr] = 0.f;  // the attention kernel max-accumulates it
        }
      }
      publish();
      trace_point(a, tp++);
      const int dh = a.dh;
      tiles1(a.gemms[gi++], [](int) { return make_float2(0.f, 0.f); }, [&](int c, const float(&stp)[kDCols], uint32_t(&x1)[kDCols], uint32_t(&x2)[kDCols],
                                uint32_t(&x3)[kDCols]) {
        const int n = c * 128 + chl;
        if (n >= 3 * D) return;
        const int part = n / D, e = n - part * D;
        const int hh = part > 0 ? e / dh : 0;
        const float scale = a.gemms[gi - 1].scale;
        // key/value rings, head-major: [K|V][head][slot][dh]; this channel's place past the
        // session's key-ring row
        const size_t cofs = (size_t)(part - 1) * a.cache * D + (size_t)hh * a.cache * dh + (e - hh * dh);
#pragma unroll
        for (int j = 0; j < kDCols; ++j) {
          const int rr = r0 + j;
          if (!bars->valid[rr]) continue;
          const float y = dequant(x1[j], x2[j], x3[j], stp[j], scale);
          if (part == 0) a.qbuf[(size_t)(s0 + rr) * D + e] = y;
          else a.kv[bars->kvoff[rr] + cofs] = y;
        }
      });
    }

    trace_point(a, tp++);
    // ---- final RMSNorm (the head's input) ----
    if (a.final_norm && !a.fuse_head) norm_rows(a.final_gain, a.fnorm, true, a.fnorm_rowmax, false);

    // ---- fused greedy head: logits = E c s_e + head_b (headLogits, stream.go:233-248), then
    // argmaxProb (generate/greedy.go:90-102): first index of the max, probability 1 / sum exp(l - max)
    if (a.final_norm && a.fuse_head) {
      norm_rows(a.final_gain, nullptr, false, nullptr, true);
      publish();
      const int step = a.head_logits ? 0 : *a.step;  // read before this CTA's arrival below, so before any increment
      float hm[kDCols], hs[kDCols];
      int hi[kDCols];
#pragma unroll
      for (int j = 0; j < kDCols; ++j) {
        hm[j] = -INFINITY;
        hs[j] = 0.f;
        hi[j] = 0x7fffffff;
      }
      tiles1(a.gemms[gi++], [&](int c) {
        const int v = c * 128 + chl;
        return make_float2(v < a.V ? a.head_b[v] : 0.f, 0.f);
      }, [&](int c, const float(&stp)[kDCols], uint32_t(&x1)[kDCols], uint32_t(&x2)[kDCols], uint32_t(&x3)[kDCols]) {
        const int v = c * 128 + chl;
        if (v >= a.V) return;
        const float scale = a.gemms[gi - 1].scale;
        if (a.head_logits) {  // the policy's logits: 32 consecutive channels of a session per warp
#pragma unroll
          for (int j = 0; j < kDCols; ++j)
            if (bars->valid[r0 + j])
              a.head_logits[(size_t)(s0 + r0 + j) * a.V + v] = __fadd_rn(dequant(x1[j], x2[j], x3[j], stp[j], scale), pv.x);
          return;
        }
#pragma unroll
        for (int j = 0; j < kDCols; ++j) {
          const float l = __fadd_rn(dequant(x1[j], x2[j], x3[j], stp[j], scale), pv.x);
          // the probability's sum of exponentials takes the fast exp (ex2 of x log2 e, a few ulp):
          // the selection itself is exact, and the probability stays far inside its 1e-4 bar
          if (l > hm[j]) {  // channels arrive in increasing order: ties keep the first index
            hs[j] = __fmul_rn(hs[j], __expf(hm[j] - l));
            hm[j] = l;
            hi[j] = v;
          }
          hs[j] = __fadd_rn(hs[j], __expf(l - hm[j]));
        }
      });
      if (a.head_logits) goto head_done;
      {
      // combine over the 32 channels of the warp, then over the four quadrant warps
      auto combine = [](float& m, float& sm, int& i, float m2, float s2, int i2) {
        const float M = fmaxf(m, m2);
        if (M == -INFINITY) return;
        const float sa = m == -INFINITY ? 0.f : __fmul_rn(sm, expf(m - M));
        const float sb = m2 == -INFINITY ? 0.f : __fmul_rn(s2, expf(m2 - M));
        i = (m == M && m2 == M) ? min(i, i2) : (m == M ? i : i2);
        m = M;
        sm = __fadd_rn(sa, sb);
      };
#pragma unroll
      for (int j = 0; j < kDCols; ++j) {
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          const float m2 = __shfl_xor_sync(0xffffffffu, hm[j], o);
          const float s2 = __shfl_xor_sync(0xffffffffu, hs[j], o);
          const int i2 = __shfl_xor_sync(0xffffffffu, hi[j], o);
          combine(hm[j], hs[j], hi[j], m2, s2, i2);
        }
        if (lane == 0) {
          bars->red_m[warp & 3][r0 + j] = hm[j];
          bars->red_s[warp & 3][r0 + j] = hs[j];
          bars->red_i[warp & 3][r0 + j] = hi[j];
        }
      }
      row_bar_d();
      if (t < kDR && bars->valid[t]) {
        float m = bars->red_m[0][t], sm = bars->red_s[0][t];
        int i = bars->red_i[0][t];
        for (int q = 1; q < 4; ++q) combine(m, sm, i, bars->red_m[q][t], bars->red_s[q][t], bars->red_i[q][t]);
        const int s = s0 + t;
        bool stop = false;
        for (int k = 0; k < a.n_stops; ++k) stop |= i == a.stops[k];
        if (stop) {
          a.seglen_w[s] = 0;  // greedyLoop ends before a stop token (generate/greedy.go:75-77)
        } else {
          const int col = a.gen_n ? a.gen_n[s] : step;
          a.next_tok[s] = i;
          if (a.out_tok) a.out_tok[(size_t)s * a.out_stride + col] = i;
          if (a.out_prob) a.out_prob[(size_t)s * a.out_stride + col] = __fdiv_rn(1.0f, sm);
          a.pos_w[s] = bars->pos[t] + 1;
          if (a.gen_n) {  // per-session generation: the session ends after its last token
            a.gen_n[s] = col + 1;
            if (a.limit && col + 1 >= a.limit[s]) a.seglen_w[s] = 0;
          }
        }
      }
      // the last CTA to finish advances the step counter (every CTA has read it by then)
      row_bar_d();
      if (t == 0) {
        __threadfence();
        if (atomicAdd(a.done, 1) == (int)gridDim.x - 1) {
          *a.step += 1;
          *a.done = 0;
          __threadfence();
        }
      }
      }
    head_done:;
    }

    // ---- the block's output rows for the next kernel ----
    if (!a.final_norm) {
      row_bar_d();
#pragma unroll
      for (int u = 0; u < kDRowsPerWarp; ++u) {
        const int rr = warp + kDRowWarps * u;
        if (!bars->valid[rr]) continue;
        const float4* c4 = reinterpret_cast<const float4*>(sCur + rr * D);
        float4* g4 = reinterpret_cast<float4*>(a.cur + (size_t)(s0 + rr) * D);
#pragma unroll
        for (int k = 0; k < KF; ++k) {
          const int f = lane + 32 * k;
          if (f < nf) g4[f] = c4[f];
        }
      }
    }
    trace_point(a, tp++);
  }
}

template <int KF, int R, int WS>  // float4 columns per state row lane (ceil(D / 128)), sessions per CTA, weight stages
__global__ void __launch_bounds__(kDThreads, decode_ctas_per_sm(KF, R)) block_decode_kernel(const __grid_constant__ BlockArgs a) {
  constexpr uint32_t kDTmemCols = kDSlots * (R == 32 ? 128 : 64);  // 512 or 256 (a power of two >= 32)
  extern __shared__ uint8_t smem_raw[];
  const DecodeLayout L = decode_layout<R, WS>(smem_raw, a.D, a.H, a.dec_kt);
  const int warp = threadIdx.x / 32;
  decode_init<KF, R, WS>(L);
  if (warp == kDMmaWarp) tmem_alloc(&L.bars->tmem, kDTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = L.bars->tmem;
  DecodeRun run;
  decode_block<KF, R, WS>(a, L, tmem, run);
  tc_fence_before();
  __syncthreads();
  if (warp == kDMmaWarp) tmem_dealloc(tmem, kDTmemCols);
}

}  // namespace eng
}  // namespace mc
