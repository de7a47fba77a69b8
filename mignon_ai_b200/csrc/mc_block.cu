// The block kernel: one CTA runs one CA block (all its rule steps, and the attention sublayer's
// norm and QKV projection) for a tile of 128 rows.
//
// Per rule step it restates appendPosition's inner loop (internal/quant/stream.go:165-186) for
// every row of the tile at once:
//   n      = RMSNorm(cur) * gamma                         (nn/rmsnorm.go:14-32)
//   lambda = sigmoid(W_select n * s_sel + base)           updateLatch (stream.go:197-205)
//   latch  = lambda * latch + (1 - lambda) * n            (a scan over the rows of a segment)
//   x      = [n | n(pos - dil) or 0 | latch]              AssembleNeighborhood (ca/neighborhood.go)
//   hidden = (W1v x s1 + b1v) * sigmoid(W1g x s1 + b1g)   applyRule layer 1 (stream.go:212-220)
//   o      = W2 hidden s2 + b2; g = sigmoid(o_gate)       applyRule layer 2 (:222-229)
//   cur    = (1 - g) * cur + g * o_delta
// and, when the block has attention, n_a = RMSNorm(cur) * norm_a and qkv = QKV n_a s_qkv with the
// key and value written to the session's ring (attention.go:74-81). A block whose predecessor had
// attention first applies that sublayer's output projection, cur += Out att s_out (:101-104), then
// the inter-block residual blockIn += cur; cur = blockIn (stream.go:158-163).
//
// Every product runs on the tensor core (tcgen05.mma kind::i8, TMEM accumulators): the
// activation rows are sliced into three int8 digit planes in shared memory by the four row warps,
// the pre-tiled weights stream in by TMA bulk copies (warp 5) through a 4-stage ring, and warp 4
// issues the MMAs. The epilogues (dequantization, GLU, highway, latch gate) run in the row warps
// straight from TMEM. Prefill tiles hold whole session segments, so the latch recurrence and the
// left-neighbour lookups stay inside the CTA.
#include "mc_engine.cuh"

namespace mc {
namespace eng {

constexpr int kBlockThreads = 192;
constexpr int kSmemA = kASlots * kASlot;        // 144 KB
constexpr int kSmemB = kBStages * kTile;        // 64 KB
constexpr int kBlockSmem = kSmemA + kSmemB + 1024 /*align*/ + 1024 /*barriers, row data*/;

struct Bars {
  uint64_t a_full[kASlots], a_empty[kASlots], b_full[kBStages], b_empty[kBStages], acc_full, acc_empty;
  uint32_t tmem;
  uint32_t rowmax_ll[kRows];  // float bits of max |left|, |latch| per row
};

__device__ __forceinline__ void row_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Slices K tile kt of one activation row into the three digit planes of an A slot.
__device__ __forceinline__ void gen_tile(uint8_t* slot, int r, const float* rowp, int K, int kt, float inv, bool valid) {
#pragma unroll 1
  for (int ch = 0; ch < 8; ++ch) {
    const int k = kt * 128 + ch * 16;
    float x[16];
    if (valid && k + 16 <= K && ((reinterpret_cast<uintptr_t>(rowp + k) & 15) == 0)) {
      const float4* p = reinterpret_cast<const float4*>(rowp + k);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 v = p[q];
        x[4 * q] = v.x; x[4 * q + 1] = v.y; x[4 * q + 2] = v.z; x[4 * q + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) x[e] = (valid && k + e < K) ? rowp[k + e] : 0.f;
    }
    uint32_t p1[4], p2[4], p3[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      Digits3 d[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) d[e] = slice3(x[4 * q + e], inv);
      p1[q] = pack4(d[0].d1, d[1].d1, d[2].d1, d[3].d1);
      p2[q] = pack4(d[0].d2, d[1].d2, d[2].d2, d[3].d2);
      p3[q] = pack4(d[0].d3, d[1].d3, d[2].d3, d[3].d3);
    }
    const uint32_t off = sw128_offset(r, ch);
    *reinterpret_cast<uint4*>(slot + off) = make_uint4(p1[0], p1[1], p1[2], p1[3]);
    *reinterpret_cast<uint4*>(slot + kTile + off) = make_uint4(p2[0], p2[1], p2[2], p2[3]);
    *reinterpret_cast<uint4*>(slot + 2 * kTile + off) = make_uint4(p3[0], p3[1], p3[2], p3[3]);
  }
}

// Loads 16 columns of the three slice accumulators of this thread's row.
__device__ __forceinline__ void load_acc16(uint32_t tmem, int warp, int col, uint32_t (&a1)[16], uint32_t (&a2)[16],
                                          uint32_t (&a3)[16]) {
  const uint32_t base = tmem_addr(tmem, 32 * (warp & 3), col);
  tmem_ld16(base, a1);
  tmem_ld16(base + kNC, a2);
  tmem_ld16(base + 2 * kNC, a3);
  tmem_wait_ld();
}

// RMSNorm of one row (nn/rmsnorm.go:14-32): out = (x * (1/rms)) * gain. Returns max |out|.
__device__ __forceinline__ float rmsnorm_row(const float* x, const float* gain, float* out, int D) {
  float ss = 0.f;
  for (int d = 0; d < D; ++d) ss = __fmaf_rn(x[d], x[d], ss);
  const float ms = __fadd_rn(__fdiv_rn(ss, (float)D), 1e-5f);
  const float rms = (float)sqrt((double)ms);
  const float inv = __fdiv_rn(1.0f, rms);
  float m = 0.f;
  for (int d = 0; d < D; ++d) {
    const float v = gain ? __fmul_rn(__fmul_rn(x[d], inv), gain[d]) : x[d];
    out[d] = v;
    m = fmaxf(m, fabsf(v));
  }
  return m;
}

__global__ void __launch_bounds__(kBlockThreads, 1) block_kernel(const __grid_constant__ BlockArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kSmemA;
  Bars* bars = reinterpret_cast<Bars*>(sB + kSmemB);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tile = blockIdx.x;
  const int D = a.D, H = a.H;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kASlots; ++i) {
      mbar_init(&bars->a_full[i], 128);
      mbar_init(&bars->a_empty[i], 1);
    }
    for (int i = 0; i < kBStages; ++i) {
      mbar_init(&bars->b_full[i], 1);
      mbar_init(&bars->b_empty[i], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, 128);
    fence_barrier_init();
  }
  if (threadIdx.x < kRows) bars->rowmax_ll[threadIdx.x] = 0u;
  if (warp == 4) tmem_alloc(&bars->tmem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;

  if (warp == 5) {
    // ---------------- weight-tile producer (TMA bulk copies) ----------------
    if (lane == 0) {
      uint32_t bidx = 0;
      bool ok = true;
      for (int g = 0; g < a.ngemms && ok; ++g) {
        const GemmSpec& G = a.gemms[g];
        for (int c = 0; c < G.nchunks && ok; ++c)
          for (int kt = 0; kt < G.ktiles && ok; ++kt, ++bidx) {
            const int st = bidx % kBStages;
            if (bidx >= kBStages && !mbar_wait_or_abort(&bars->b_empty[st], ((bidx / kBStages) - 1) & 1, kErrWaitEmpty)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars->b_full[st], kTile);
            bulk_load(sB + st * kTile, G.tiles + ((size_t)c * G.ktiles + kt) * kTile, kTile, &bars->b_full[st]);
          }
      }
    }
  } else if (warp == 4) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t bidx = 0, chunk_idx = 0;
      uint32_t afill[kASlots] = {0, 0, 0};
      const uint32_t idesc = idesc_i8(kRows, kNC);
      bool ok = true;
      for (int g = 0; g < a.ngemms && ok; ++g) {
        const GemmSpec& G = a.gemms[g];
        const bool resident = G.ktiles <= kASlots;
        for (int c = 0; c < G.nchunks && ok; ++c) {
          if (chunk_idx > 0 && !mbar_wait_or_abort(&bars->acc_empty, (chunk_idx - 1) & 1, kErrWaitAccFree)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int kt = 0; kt < G.ktiles; ++kt, ++bidx) {
            const int slot = kt % kASlots;
            if (c == 0 || !resident) {
              if (!mbar_wait_or_abort(&bars->a_full[slot], afill[slot] & 1, kErrWaitFull)) {
                ok = false;
                break;
              }
              afill[slot]++;
            }
            const int st = bidx % kBStages;
            if (!mbar_wait_or_abort(&bars->b_full[st], (bidx / kBStages) & 1, kErrWaitFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t db = smem_desc_sw128(sB + st * kTile);
            const int ksteps = min(4, (G.K - kt * 128 + 31) / 32);
#pragma unroll
            for (int p = 0; p < 3; ++p) {
              const uint64_t da = smem_desc_sw128(sA + slot * kASlot + p * kTile);
              for (int kk = 0; kk < ksteps; ++kk)
                mma_i8(tmem + p * kNC, da + 2 * kk, db + 2 * kk, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
            }
            mma_commit(&bars->b_empty[st]);
            if (!resident || c == G.nchunks - 1) mma_commit(&bars->a_empty[slot]);
          }
          if (!ok) break;
          mma_commit(&bars->acc_full);
          ++chunk_idx;
        }
      }
    }
  } else {
    // ---------------- row warps: activations, epilogues, row/channel phases ----------------
    const int r = threadIdx.x;  // row in tile (TMEM lane)
    const int grow = tile * kRows + r;
    const RowInfo ri = row_info(a, grow);
    uint32_t afill[kASlots] = {0, 0, 0};
    uint32_t chunk_idx = 0;
    bool ok = true;
    float rowmax_n = 0.f;   // max |norm cell| of this row (current step)
    float rowmax_h = 0.f;   // max |hidden| of this row

    // Runs GEMM g with activation rows src (row stride ld) whose max |.| is amax; the epilogue
    // callback receives the chunk index.
    auto run_gemm = [&](int g, const float* src, int ld, float amax, auto&& epilogue) {
      const GemmSpec& G = a.gemms[g];
      const bool resident = G.ktiles <= kASlots;
      const float inv = row_inv_step(amax);
      const float step = row_step(amax);
      const float* rowp = src + (size_t)grow * ld;
      for (int c = 0; c < G.nchunks; ++c) {
        if (c == 0 || !resident) {
          for (int kt = 0; kt < G.ktiles; ++kt) {
            const int slot = kt % kASlots;
            if (ok && afill[slot] >= 1 &&
                !mbar_wait_or_abort(&bars->a_empty[slot], (afill[slot] - 1) & 1, kErrWaitEmpty))
              ok = false;
            afill[slot]++;
            if (ok) gen_tile(sA + slot * kASlot, r, rowp, G.K, kt, inv, ri.valid);
            fence_proxy_async_smem();
            mbar_arrive(&bars->a_full[slot]);
          }
        }
        const bool got = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&bars->acc_full, chunk_idx & 1, kErrWaitAcc));
        if (!got) ok = false;
        if (ok) {
          tc_fence_after();
          epilogue(c, step, G.scale);
        }
        tc_fence_before();
        mbar_arrive(&bars->acc_empty);
        ++chunk_idx;
      }
    };

    int g = 0;
    // ---- output projection of the previous block's attention: cur += Out att s_out ----
    if (a.has_out) {
      const float amax = a.att_rowmax[grow];
      run_gemm(g++, a.att, D, amax, [&](int c, float step, float scale) {
        for (int j0 = 0; j0 < kNC; j0 += 16) {
          uint32_t a1[16], a2[16], a3[16];
          load_acc16(tmem, warp, j0, a1, a2, a3);
          if (!ri.valid) continue;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = c * kNC + j0 + j;
            if (n < D) {
              float* p = a.cur + (size_t)grow * D + n;
              *p = __fadd_rn(*p, dequant(a1[j], a2[j], a3[j], step, scale));
            }
          }
        }
      });
      row_bar();
    }
    // ---- embedding (first block) or inter-block residual ----
    if (a.embed_first || a.residual) {
      for (int rr = 0; rr < kRows; ++rr) {
        const int gr = tile * kRows + rr;
        const RowInfo rj = row_info(a, gr);
        if (!rj.valid) continue;
        float* cur = a.cur + (size_t)gr * D;
        float* bin = a.blockin + (size_t)gr * D;
        if (a.embed_first) {
          int tok = a.tokens[(size_t)rj.session * a.P + rj.t];
          if (tok < 0 || tok >= a.V) tok = 0;
          const int8_t* e = a.embed + (size_t)tok * D;
          for (int d = r; d < D; d += 128) {
            const float v = __fmul_rn((float)e[d], a.embed_scale);
            cur[d] = v;
            bin[d] = v;
          }
        } else {
          for (int d = r; d < D; d += 128) {
            const float v = __fadd_rn(bin[d], cur[d]);
            bin[d] = v;
            cur[d] = v;
          }
        }
      }
      row_bar();
    }

    // ---- rule steps ----
    for (int s = 0; s < a.nsteps; ++s) {
      const int bs = a.bs0 + s;
      const int dil = a.dil[s];
      float* xrow = a.xbuf + (size_t)grow * 3 * D;
      // norm cell n -> xbuf[:, 0:D]
      if (ri.valid) {
        rowmax_n = rmsnorm_row(a.cur + (size_t)grow * D, a.gamma, xrow, D);
      } else {
        rowmax_n = 0.f;
      }
      bars->rowmax_ll[r] = 0u;
      row_bar();
      // W_select: lambda -> xbuf[:, 2D:3D]
      run_gemm(g++, a.xbuf, 3 * D, rowmax_n, [&](int c, float step, float scale) {
        for (int j0 = 0; j0 < kNC; j0 += 16) {
          uint32_t a1[16], a2[16], a3[16];
          load_acc16(tmem, warp, j0, a1, a2, a3);
          if (!ri.valid) continue;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = c * kNC + j0 + j;
            if (n < D) {
              const float z = __fadd_rn(dequant(a1[j], a2[j], a3[j], step, scale), a.latch_base[n]);
              xrow[2 * D + n] = sigmoid_clamped(z);
            }
          }
        }
      });
      row_bar();
      // latch scan and left neighbours (channel-parallel over the rows of the tile)
      for (int d = r; d < D; d += 128) {
        for (int slot = 0; slot < a.spt; ++slot) {
          const int sess = tile * a.spt + slot;
          if (sess >= a.n_sess) break;
          const int len = a.seglen[sess];
          if (len <= 0) continue;
          const int p0 = a.pos0[sess];
          float* lstate = a.latch + ((size_t)sess * a.total_steps + bs) * D + d;
          float l = (p0 == 0) ? 0.f : *lstate;
          const float* ring = a.norm_ring + ((size_t)sess * a.total_steps + bs) * a.ring * D + d;
          for (int t = 0; t < len; ++t) {
            const int gr = tile * kRows + slot * a.P + t;
            float* x = a.xbuf + (size_t)gr * 3 * D;
            const float lam = x[2 * D + d];
            const float nv = x[d];
            l = __fadd_rn(__fmul_rn(lam, l), __fmul_rn(__fsub_rn(1.0f, lam), nv));
            x[2 * D + d] = l;
            float left = 0.f;
            if (t >= dil) left = a.xbuf[(size_t)(gr - dil) * 3 * D + d];
            else if (p0 + t - dil >= 0) left = ring[(size_t)((p0 + t - dil) % a.ring) * D];
            x[D + d] = left;
            const float m = fmaxf(fabsf(l), fabsf(left));
            const unsigned wm = __reduce_max_sync(__activemask(), __float_as_uint(m));
            if (lane == 0 || (d & 31) == 0) atomicMax(&bars->rowmax_ll[slot * a.P + t], wm);
          }
          *lstate = l;
        }
      }
      row_bar();
      // norm ring: the last `ring` positions of each segment
      for (int d = r; d < D; d += 128)
        for (int slot = 0; slot < a.spt; ++slot) {
          const int sess = tile * a.spt + slot;
          if (sess >= a.n_sess) break;
          const int len = a.seglen[sess];
          const int p0 = a.pos0[sess];
          for (int t = max(0, len - a.ring); t < len; ++t) {
            const int gr = tile * kRows + slot * a.P + t;
            a.norm_ring[(((size_t)sess * a.total_steps + bs) * a.ring + (size_t)((p0 + t) % a.ring)) * D + d] =
                a.xbuf[(size_t)gr * 3 * D + d];
          }
        }
      // W1 + GLU -> hbuf
      const float xmax = fmaxf(rowmax_n, __uint_as_float(bars->rowmax_ll[r]));
      rowmax_h = 0.f;
      run_gemm(g++, a.xbuf, 3 * D, xmax, [&](int c, float step, float scale) {
        const int h0 = c * kHalfChunk;
        for (int j0 = 0; j0 < kHalfChunk; j0 += 16) {
          uint32_t v1[16], v2[16], v3[16], g1[16], g2[16], g3[16];
          load_acc16(tmem, warp, j0, v1, v2, v3);
          load_acc16(tmem, warp, kHalfChunk + j0, g1, g2, g3);
          if (!ri.valid) continue;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int h = h0 + j0 + j;
            if (h < H) {
              const float v = __fadd_rn(dequant(v1[j], v2[j], v3[j], step, scale), a.b1[h]);
              const float gt = __fadd_rn(dequant(g1[j], g2[j], g3[j], step, scale), a.b1[H + h]);
              const float hid = __fmul_rn(v, sigmoid_clamped(gt));
              a.hbuf[(size_t)grow * H + h] = hid;
              rowmax_h = fmaxf(rowmax_h, fabsf(hid));
            }
          }
        }
      });
      // W2 + highway -> cur
      run_gemm(g++, a.hbuf, H, rowmax_h, [&](int c, float step, float scale) {
        const int d0 = c * kHalfChunk;
        for (int j0 = 0; j0 < kHalfChunk; j0 += 16) {
          uint32_t o1[16], o2[16], o3[16], q1[16], q2[16], q3[16];
          load_acc16(tmem, warp, j0, o1, o2, o3);
          load_acc16(tmem, warp, kHalfChunk + j0, q1, q2, q3);
          if (!ri.valid) continue;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int d = d0 + j0 + j;
            if (d < D) {
              const float od = __fadd_rn(dequant(o1[j], o2[j], o3[j], step, scale), a.b2[d]);
              const float og = __fadd_rn(dequant(q1[j], q2[j], q3[j], step, scale), a.b2[D + d]);
              const float gate = sigmoid_clamped(og);
              float* cp = a.cur + (size_t)grow * D + d;
              *cp = __fadd_rn(__fmul_rn(__fsub_rn(1.0f, gate), *cp), __fmul_rn(gate, od));
            }
          }
        }
      });
      row_bar();
    }

    // ---- attention sublayer: norm + QKV, keys/values into the ring ----
    if (a.has_attn) {
      float* nrow = a.xbuf + (size_t)grow * 3 * D;
      float amax = 0.f;
      if (ri.valid) amax = rmsnorm_row(a.cur + (size_t)grow * D, a.attn_norm, nrow, D);
      row_bar();
      float* kvs = a.kv + ((size_t)ri.session * a.n_attn + a.attn_slot) * 2 * (size_t)a.cache * D;
      const bool to_ring = ri.valid && ri.t >= ri.len - a.cache;
      const int rslot = ri.pos % a.cache;
      float* lin = a.kvlin ? a.kvlin + ((size_t)ri.session * a.P + ri.t) * 2 * D : nullptr;
      run_gemm(g++, a.xbuf, 3 * D, amax, [&](int c, float step, float scale) {
        for (int j0 = 0; j0 < kNC; j0 += 16) {
          uint32_t a1[16], a2[16], a3[16];
          load_acc16(tmem, warp, j0, a1, a2, a3);
          if (!ri.valid) continue;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = c * kNC + j0 + j;
            if (n >= 3 * D) continue;
            const float v = dequant(a1[j], a2[j], a3[j], step, scale);
            if (n < D) {
              a.qbuf[(size_t)grow * D + n] = v;
            } else {
              const int which = n < 2 * D ? 0 : 1;
              const int e = n - D - which * D;
              if (to_ring) kvs[((size_t)which * a.cache + rslot) * D + e] = v;
              if (lin) lin[which * D + e] = v;
            }
          }
        }
      });
    }

    // ---- final RMSNorm (the head's input) ----
    if (a.final_norm) {
      float m = 0.f;
      if (ri.valid) {
        if (a.final_gain) m = rmsnorm_row(a.cur + (size_t)grow * D, a.final_gain, a.fnorm + (size_t)grow * D, D);
        else {
          for (int d = 0; d < D; ++d) {
            const float v = a.cur[(size_t)grow * D + d];
            a.fnorm[(size_t)grow * D + d] = v;
            m = fmaxf(m, fabsf(v));
          }
        }
      }
      a.fnorm_rowmax[grow] = m;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) tmem_dealloc(tmem, 512);
}

}  // namespace eng
}  // namespace mc
