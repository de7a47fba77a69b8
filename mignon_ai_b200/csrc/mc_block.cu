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
// activation rows are sliced into three int8 digit planes in shared memory by sixteen row warps
// (four threads per row, each a quarter of the K bytes), the pre-tiled weights stream in by TMA
// bulk copies (the producer warp) through a 4-stage ring, and the MMA warp issues the MMAs. The
// epilogues run in the row warps straight from TMEM, four threads per row splitting the columns;
// each fetches its global operands before waiting for the accumulator.
//
// Decode rows (one position per session) update the latch, read the left neighbour from the
// session's norm ring and write the ring inside the W_select epilogue, each thread on its own row.
// Prefill tiles hold whole session segments; there the latch is a scan over the segment's rows
// (channel-parallel) and left neighbours inside the segment are rows of the same tile.
#include "mc_engine.cuh"

namespace mc {
namespace eng {

constexpr int kRowThreads = 512;                 // four threads per row
constexpr int kRowWarps = kRowThreads / 32;
constexpr int kTPR = kRowThreads / kRows;          // threads per row
constexpr int kBlockThreads = kRowThreads + 64;  // + MMA warp + weight producer warp
constexpr int kMmaWarp = kRowWarps;
constexpr int kProducerWarp = kRowWarps + 1;
constexpr int kSmemA = kASlots * kASlot;        // 144 KB
constexpr int kSmemB = kBStages * kTile;        // 64 KB
constexpr int kBlockSmem = kSmemA + kSmemB + 1024 /*align*/ + 16384 /*barriers, row data*/;

constexpr int kVecMax = 2048;  // floats of a staged epilogue vector (b1 of hidden widths up to 1024)

struct Bars {
  uint64_t a_full[kASlots], a_empty[kASlots], a_tma[kASlots], b_full[kBStages], b_empty[kBStages], acc_full, acc_empty;
  uint64_t a_pre;                      // the row warps wrote a GEMM's planes straight into the plane cache
  uint32_t tmem;
  float rowmax_n[kRows];               // max |norm cell| per row
  float rowmax_part[kTPR][kRows];       // per-thread partial maxima of an epilogue output
  alignas(16) float vec[kVecMax];      // the per-channel vector of the current GEMM's epilogue
                                       // (latch base, b1 or b2), staged from global memory
  int rvalid[kRows];                   // row holds a position of an active session
  int rtok[kRows];                     // its token (clamped to the vocabulary)
  int rsess[kRows];                    // its session
  int rpos[kRows];                     // its position
  float rowmax_a[kRows];               // max |A row| of the next GEMM (x, att)
  float rowmax_h[kRows];               // max |hidden| per row
};
static_assert(sizeof(Bars) <= 16384, "barrier block");

__device__ __forceinline__ void row_bar() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

// 16 consecutive floats p[n0 .. n0+16) with n < lim, zeros past lim.
__device__ __forceinline__ void ld16(const float* __restrict__ p, int n0, int lim, float (&v)[16]) {
  if (n0 + 16 <= lim && ((reinterpret_cast<uintptr_t>(p + n0) & 15) == 0)) {
    const float4* q = reinterpret_cast<const float4*>(p + n0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 t = q[i];
      v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = (n0 + e < lim) ? p[n0 + e] : 0.f;
  }
}

__device__ __forceinline__ void st16(float* __restrict__ p, int n0, int lim, const float (&v)[16]) {
  if (n0 + 16 <= lim && ((reinterpret_cast<uintptr_t>(p + n0) & 15) == 0)) {
    float4* q = reinterpret_cast<float4*>(p + n0);
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
#pragma unroll
    for (int e = 0; e < 16; ++e)
      if (n0 + e < lim) p[n0 + e] = v[e];
  }
}

// Slices the 16-byte chunks [ch0, ch0 + NCH) of K tile kt of one activation row into the three
// digit planes of an A slot (row r of the 128-row tile). All loads are issued before any slicing.
template <int NCH>
__device__ __forceinline__ void gen_tile(uint8_t* slot, int r, const float* __restrict__ rowp, int K, int kt, float inv,
                                         bool valid, int ch0) {
  float x[NCH][16];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    if (valid) ld16(rowp, kt * 128 + (ch0 + c) * 16, K, x[c]);
    else {
#pragma unroll
      for (int e = 0; e < 16; ++e) x[c][e] = 0.f;
    }
  }
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    uint32_t p1[4], p2[4], p3[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t u1[4], u2[4], u3[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) slice3_bits(x[c][4 * q + e], inv, u1[e], u2[e], u3[e]);
      p1[q] = pack_low_bytes(u1[0], u1[1], u1[2], u1[3]);
      p2[q] = pack_low_bytes(u2[0], u2[1], u2[2], u2[3]);
      p3[q] = pack_low_bytes(u3[0], u3[1], u3[2], u3[3]);
    }
    const uint32_t off = sw128_offset(r, ch0 + c);
    *reinterpret_cast<uint4*>(slot + off) = make_uint4(p1[0], p1[1], p1[2], p1[3]);
    *reinterpret_cast<uint4*>(slot + kTile + off) = make_uint4(p2[0], p2[1], p2[2], p2[3]);
    *reinterpret_cast<uint4*>(slot + 2 * kTile + off) = make_uint4(p3[0], p3[1], p3[2], p3[3]);
  }
}

// Loads 16 columns of the three slice accumulators of this thread's row (warp-collective).
__device__ __forceinline__ void load_acc16(uint32_t tmem, int warp, int col, uint32_t (&a1)[16], uint32_t (&a2)[16],
                                          uint32_t (&a3)[16]) {
  const uint32_t base = tmem_addr(tmem, 32 * (warp & 3), col);
  tmem_ld16(base, a1);
  tmem_ld16(base + kNC, a2);
  tmem_ld16(base + 2 * kNC, a3);
  tmem_wait_ld();
}

// 8 columns of the three slice accumulators at two column offsets (a value tile and its gate
// tile): all six loads in flight before one wait (warp-collective).
__device__ __forceinline__ void load_acc8x2(uint32_t tmem, int warp, int col_a, int col_b, uint32_t (&a1)[8],
                                           uint32_t (&a2)[8], uint32_t (&a3)[8], uint32_t (&b1)[8], uint32_t (&b2)[8],
                                           uint32_t (&b3)[8]) {
  const uint32_t ba = tmem_addr(tmem, 32 * (warp & 3), col_a), bb = tmem_addr(tmem, 32 * (warp & 3), col_b);
  tmem_ld8(ba, a1);
  tmem_ld8(ba + kNC, a2);
  tmem_ld8(ba + 2 * kNC, a3);
  tmem_ld8(bb, b1);
  tmem_ld8(bb + kNC, b2);
  tmem_ld8(bb + 2 * kNC, b3);
  tmem_wait_ld();
}

__device__ __forceinline__ void ld8(const float* __restrict__ p, int n0, int lim, float (&v)[8]) {
  if (n0 + 8 <= lim && ((reinterpret_cast<uintptr_t>(p + n0) & 15) == 0)) {
    const float4 t0 = reinterpret_cast<const float4*>(p + n0)[0], t1 = reinterpret_cast<const float4*>(p + n0)[1];
    v[0] = t0.x; v[1] = t0.y; v[2] = t0.z; v[3] = t0.w; v[4] = t1.x; v[5] = t1.y; v[6] = t1.z; v[7] = t1.w;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = (n0 + e < lim) ? p[n0 + e] : 0.f;
  }
}

__device__ __forceinline__ void st8(float* __restrict__ p, int n0, int lim, const float (&v)[8]) {
  if (n0 + 8 <= lim && ((reinterpret_cast<uintptr_t>(p + n0) & 15) == 0)) {
    reinterpret_cast<float4*>(p + n0)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p + n0)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (n0 + e < lim) p[n0 + e] = v[e];
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void trace_point(const BlockArgs& a, int i) {
  if (a.trace && blockIdx.x == 0 && threadIdx.x == 0 && i < 64) a.trace[i] = global_timer_ns();
}

// Writes the three digit planes of four consecutive activations (K indices e..e+3, e % 4 == 0)
// of tile row r into the A slot holding K tile e / 128. One 32-bit store per plane; a warp
// writing 128 consecutive K values of a row touches every bank once.
__device__ __forceinline__ void put4(uint8_t* sA, int r, int e, float4 v, float inv) {
  const int kt = e >> 7, k = e & 127;
  uint8_t* tile = sA + (kt % kASlots) * kASlot;
  const uint32_t off = sw128_offset(r, k >> 4) + (k & 15);
  uint32_t a0, a1, a2, a3, b0, b1, b2, b3, c0, c1, c2, c3;
  slice3_bits(v.x, inv, a0, b0, c0);
  slice3_bits(v.y, inv, a1, b1, c1);
  slice3_bits(v.z, inv, a2, b2, c2);
  slice3_bits(v.w, inv, a3, b3, c3);
  *reinterpret_cast<uint32_t*>(tile + off) = pack_low_bytes(a0, a1, a2, a3);
  *reinterpret_cast<uint32_t*>(tile + kTile + off) = pack_low_bytes(b0, b1, b2, b3);
  *reinterpret_cast<uint32_t*>(tile + 2 * kTile + off) = pack_low_bytes(c0, c1, c2, c3);
}

// put4 that also writes the same three words at the same offsets of a global copy of the A
// slots' contents (gA: K tile 0 of the copy; K tile kt at gA + kt * kASlot).
__device__ __forceinline__ void put4_2(uint8_t* sA, uint8_t* gA, int r, int e, float4 v, float inv) {
  const int kt = e >> 7, k = e & 127;
  uint8_t* tile = sA + (kt % kASlots) * kASlot;
  uint8_t* gtile = gA + (size_t)kt * kASlot;
  const uint32_t off = sw128_offset(r, k >> 4) + (k & 15);
  uint32_t a0, a1, a2, a3, b0, b1, b2, b3, c0, c1, c2, c3;
  slice3_bits(v.x, inv, a0, b0, c0);
  slice3_bits(v.y, inv, a1, b1, c1);
  slice3_bits(v.z, inv, a2, b2, c2);
  slice3_bits(v.w, inv, a3, b3, c3);
  const uint32_t p1 = pack_low_bytes(a0, a1, a2, a3), p2 = pack_low_bytes(b0, b1, b2, b3), p3 = pack_low_bytes(c0, c1, c2, c3);
  *reinterpret_cast<uint32_t*>(tile + off) = p1;
  *reinterpret_cast<uint32_t*>(tile + kTile + off) = p2;
  *reinterpret_cast<uint32_t*>(tile + 2 * kTile + off) = p3;
  *reinterpret_cast<uint32_t*>(gtile + off) = p1;
  *reinterpret_cast<uint32_t*>(gtile + kTile + off) = p2;
  *reinterpret_cast<uint32_t*>(gtile + 2 * kTile + off) = p3;
}

// The three digit planes of four consecutive activations (K indices e..e+3) of tile row r written
// only to the global copy of the A slots (the per-SM plane cache; K tile kt at gA + kt * kASlot).
// A warp writing 128 consecutive K values of a row stores one whole 128-byte line per plane.
__device__ __forceinline__ void put4_g(uint8_t* gA, int r, int e, float4 v, float inv) {
  const int kt = e >> 7, k = e & 127;
  uint8_t* gtile = gA + (size_t)kt * kASlot;
  const uint32_t off = sw128_offset(r, k >> 4) + (k & 15);
  uint32_t a0, a1, a2, a3, b0, b1, b2, b3, c0, c1, c2, c3;
  slice3_bits(v.x, inv, a0, b0, c0);
  slice3_bits(v.y, inv, a1, b1, c1);
  slice3_bits(v.z, inv, a2, b2, c2);
  slice3_bits(v.w, inv, a3, b3, c3);
  *reinterpret_cast<uint32_t*>(gtile + off) = pack_low_bytes(a0, a1, a2, a3);
  *reinterpret_cast<uint32_t*>(gtile + kTile + off) = pack_low_bytes(b0, b1, b2, b3);
  *reinterpret_cast<uint32_t*>(gtile + 2 * kTile + off) = pack_low_bytes(c0, c1, c2, c3);
}

// How the A slots are filled for chunk c of GEMM G: 0 not at all (a resident GEMM's later chunks),
// 1 by the row warps (sliced, published on a_full), 2 by the producer from the per-SM cache
// (bulk copies completing on a_tma). presliced: the row warps wrote every K tile of the planes to
// the cache before the GEMM (announced on a_pre), so every chunk comes from the cache.
__device__ __forceinline__ int a_fill_kind(const GemmSpec& G, int c, bool cache, bool presliced) {
  if (G.ktiles <= kASlots) return c == 0 ? 1 : 0;
  if (presliced) return 2;
  return (c > 0 && cache) ? 2 : 1;
}

__device__ __forceinline__ float4 ld4_or0(const float* p, int e, int K, bool valid) {
  if (!valid || e >= K) return make_float4(0.f, 0.f, 0.f, 0.f);
  if (e + 4 <= K) return *reinterpret_cast<const float4*>(p + e);
  float4 v = make_float4(p[e], 0.f, 0.f, 0.f);
  if (e + 1 < K) v.y = p[e + 1];
  if (e + 2 < K) v.z = p[e + 2];
  return v;
}

__device__ __forceinline__ float max4(float4 v) { return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))); }

constexpr int kRowsPerWarp = kRows / kRowWarps;  // 8

template <int KF, bool CACHE>  // float4 columns per lane per row: ceil(D / 128); whether the plane cache is in use
__global__ void __launch_bounds__(kBlockThreads, 1) block_kernel(const __grid_constant__ BlockArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kSmemA;
  Bars* bars = reinterpret_cast<Bars*>(sB + kSmemB);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tile = a.tile_list ? a.tile_list[blockIdx.x] : a.tile0 + (int)blockIdx.x;
  const int D = a.D, H = a.H;
  // this SM's plane cache (one block-kernel CTA per SM at a time: its shared memory)
  uint8_t* acache = nullptr;
  {
    uint32_t id;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(id));
    if (a.a_cache && (int)id < a.a_cache_sms) acache = a.a_cache + (size_t)id * a.a_cache_kt * kASlot;
  }
  // the cache serves GEMM G when it holds all of G's K tiles and G has chunks after the first
  // (instances without CACHE compile none of its code)
  auto use_cache = [&](const GemmSpec& G) {
    return CACHE && acache != nullptr && G.ktiles <= a.a_cache_kt && G.nchunks > 1;
  };
  // W1 with more K tiles than A slots: the pass that builds its input rows x = [n | left | latch]
  // slices them straight into the plane cache (no fp32 copy of x, no slicing pass of its own)
  auto presliced = [&](const GemmSpec& G) { return G.type == kGW1 && G.ktiles > kASlots && use_cache(G); };
  // a tile whose sessions all sit this pass out (seglen 0: idle, finished, or kept out of a
  // scheduler's admission pass) has nothing to do
  {
    const int sess = tile * a.spt + (int)threadIdx.x;
    const bool live = (int)threadIdx.x < a.spt && sess < a.n_sess && a.seglen[sess] > 0;
    if (!__syncthreads_or(live)) return;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < kASlots; ++i) {
      mbar_init(&bars->a_full[i], kRowThreads);
      mbar_init(&bars->a_empty[i], 1);
      mbar_init(&bars->a_tma[i], 1);
    }
    for (int i = 0; i < kBStages; ++i) {
      mbar_init(&bars->b_full[i], 1);
      mbar_init(&bars->b_empty[i], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, kRowThreads);
    mbar_init(&bars->a_pre, kRowThreads);
    fence_barrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc(&bars->tmem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;

  if (warp == kProducerWarp) {
    // ---------------- weight-tile producer (TMA bulk copies) ----------------
    if (lane == 0) {
      uint32_t bidx = 0;
      // fills of each A slot so far (by anyone) and by the row warps, in the consumption order
      uint32_t fills[kASlots] = {0, 0, 0}, rfills[kASlots] = {0, 0, 0};
      uint32_t npre = 0;  // presliced GEMMs so far (phases of a_pre)
      bool ok = true;
      for (int g = 0; g < a.ngemms && ok; ++g) {
        const GemmSpec& G = a.gemms[g];
        const bool cache = use_cache(G);
        const bool pre = presliced(G);
        for (int c = 0; c < G.nchunks && ok; ++c) {
          const int kind = a_fill_kind(G, c, cache, pre);
          if (kind == 2 && c == 1 && !pre) {
            // the first chunk's row fills wrote every K tile to the cache: acquire their writes
            for (int sl = 0; sl < kASlots && ok; ++sl)
              if (rfills[sl] > 0 && !mbar_wait_or_abort(&bars->a_full[sl], (rfills[sl] - 1) & 1, kErrWaitFull)) ok = false;
          }
          for (int kt = 0; kt < G.ktiles && ok; ++kt, ++bidx) {
            const int slot = kt % kASlots;
            // the weight tile first: it does not depend on the row warps
            const int st = bidx % kBStages;
            if (bidx >= kBStages && !mbar_wait_or_abort(&bars->b_empty[st], ((bidx / kBStages) - 1) & 1, kErrWaitEmpty)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars->b_full[st], kTile);
            bulk_load(sB + st * kTile, G.tiles + ((size_t)c * G.ktiles + kt) * kTile, kTile, &bars->b_full[st]);
            if (kind == 1) {
              ++fills[slot];
              ++rfills[slot];
            } else if (kind == 2) {
              if (pre && c == 0 && kt == 0) {
                // the row warps' cache writes (each fenced for the async proxy before its arrival)
                if (!mbar_wait_or_abort(&bars->a_pre, npre & 1, kErrWaitFull)) {
                  ok = false;
                  break;
                }
                ++npre;
              }
              if (fills[slot] >= 1 && !mbar_wait_or_abort(&bars->a_empty[slot], (fills[slot] - 1) & 1, kErrWaitEmpty)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&bars->a_tma[slot], kASlot);
              bulk_load(sA + slot * kASlot, acache + (size_t)kt * kASlot, kASlot, &bars->a_tma[slot]);
              ++fills[slot];
            }
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t bidx = 0, chunk_idx = 0;
      uint32_t afill[kASlots] = {0, 0, 0}, tfill[kASlots] = {0, 0, 0};  // row fills, cache fills consumed
      const uint32_t idesc = idesc_i8(kRows, kNC);
      const uint64_t desc_a0 = smem_desc_sw128(sA), desc_b0 = smem_desc_sw128(sB);
      bool ok = true;
      for (int g = 0; g < a.ngemms && ok; ++g) {
        const GemmSpec& G = a.gemms[g];
        const bool resident = G.ktiles <= kASlots;
        const bool cache = use_cache(G);
        const bool pre = presliced(G);
        for (int c = 0; c < G.nchunks && ok; ++c) {
          if (chunk_idx > 0 && !mbar_wait_or_abort(&bars->acc_empty, (chunk_idx - 1) & 1, kErrWaitAccFree)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int kind = a_fill_kind(G, c, cache, pre);
          for (int kt = 0; kt < G.ktiles; ++kt, ++bidx) {
            const int slot = kt % kASlots;
            if (kind == 1) {
              if (!mbar_wait_or_abort(&bars->a_full[slot], afill[slot] & 1, kErrWaitFull)) {
                ok = false;
                break;
              }
              afill[slot]++;
            } else if (kind == 2) {
              if (!mbar_wait_or_abort(&bars->a_tma[slot], tfill[slot] & 1, kErrWaitFull)) {
                ok = false;
                break;
              }
              tfill[slot]++;
            }
            const int st = bidx % kBStages;
            if (!mbar_wait_or_abort(&bars->b_full[st], (bidx / kBStages) & 1, kErrWaitFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            // descriptors advance by their encoded start address (bytes / 16)
            const uint64_t db = desc_b0 + (uint64_t)(st * (kTile >> 4));
            const uint64_t da = desc_a0 + (uint64_t)(slot * (kASlot >> 4));
            const int ksteps = min(4, (G.K - kt * 128 + 31) / 32);
            // planes innermost: three independent accumulation chains in flight
            for (int kk = 0; kk < ksteps; ++kk) {
              const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
#pragma unroll
              for (int p = 0; p < 3; ++p)
                mma_i8(tmem + p * kNC, da + (uint64_t)(p * (kTile >> 4)) + 2 * kk, db + 2 * kk, idesc, acc);
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
    // ---------------- row warps ----------------
    // Two views of the 128 rows: row-owner (thread t owns TMEM lane r = t % 128 and a quarter h of
    // the columns; used by the accumulator epilogues) and warp-per-row (warp w owns rows w + 16u,
    // lane l the float4 columns l + 32k; used by every phase that moves rows through memory).
    const int t = threadIdx.x;
    const int r = t & (kRows - 1);
    const int h = t >> 7;
    const int grow = tile * kRows + r;
    const RowInfo ri = row_info(a, grow);
    const bool decode = a.P == 1;
    const int nf = D / 4;
    uint32_t afill[kASlots] = {0, 0, 0};
    uint32_t chunk_idx = 0;
    bool ok = true;
    int tp = 0;
    trace_point(a, tp++);
    if (h == 0) {
      bars->rvalid[r] = ri.valid ? 1 : 0;
      int tok = 0;
      if (ri.valid && a.embed_first) {
        tok = a.tokens[(size_t)ri.session * a.P + ri.t];
        if (tok < 0 || tok >= a.V) tok = 0;
      }
      bars->rtok[r] = tok;
      bars->rsess[r] = ri.session;
      bars->rpos[r] = ri.pos;
    }
    row_bar();

    auto acquire = [&](int slot) {
      if (ok && afill[slot] >= 1 && !mbar_wait_or_abort(&bars->a_empty[slot], (afill[slot] - 1) & 1, kErrWaitEmpty))
        ok = false;
      afill[slot]++;
    };
    auto publish = [&](int slot, bool cached = false) {
      fence_proxy_async_smem();
      if (cached) fence_proxy_async_global();  // the cache copy, read back by bulk copies
      mbar_arrive(&bars->a_full[slot]);
    };
    // Warp-per-row slicing of K tile kt of the rows' fp32 source (coalesced loads, all of the
    // warp's rows in flight together) with per-row maxima rmax (shared memory).
    auto gen_rows = [&](int kt, const float* src, int ld, int K, const float* rmax, uint8_t* gA) {
      float4 v[kRowsPerWarp];
      const int e = kt * 128 + 4 * lane;
#pragma unroll
      for (int u = 0; u < kRowsPerWarp; ++u) {
        const int rr = warp + kRowWarps * u;
        v[u] = ld4_or0(src + (size_t)(tile * kRows + rr) * ld, e, K, bars->rvalid[rr] != 0);
      }
#pragma unroll
      for (int u = 0; u < kRowsPerWarp; ++u) {
        const int rr = warp + kRowWarps * u;
        if (gA) put4_2(sA, gA, rr, e, v[u], row_inv_step(rmax[rr]));
        else put4(sA, rr, e, v[u], row_inv_step(rmax[rr]));
      }
    };
    // Runs GEMM g. prefilled: its (resident) A tiles were already published by a fused phase;
    // otherwise they are sliced from src with the row maxima rmax. The epilogue gets the chunk and
    // this thread's row step and weight scale.
    // prefetch(c) runs before chunk c's accumulator wait: global loads the epilogue needs,
    // issued so that their latency overlaps the MMAs.
    auto run_gemm_pre = [&](int g, bool prefilled, const float* src, int ld, const float* rmax, auto&& prefetch,
                            auto&& epilogue) {
      const GemmSpec& G = a.gemms[g];
      const bool cache = use_cache(G);
      const bool pre = presliced(G);
      const float step = row_step(rmax[r]);
      for (int c = 0; c < G.nchunks; ++c) {
        const int kind = a_fill_kind(G, c, cache, pre);
        if (!prefilled && kind == 1) {
          for (int kt = 0; kt < G.ktiles; ++kt) {
            const int slot = kt % kASlots;
            acquire(slot);
            if (ok) gen_rows(kt, src, ld, G.K, rmax, cache && c == 0 ? acache : nullptr);
            publish(slot, cache && c == 0);
          }
        } else if (kind == 2) {
          for (int kt = 0; kt < G.ktiles; ++kt) afill[kt % kASlots]++;  // filled by the producer
        }
        if (a.trace && a.trace_fine) trace_point(a, tp++);
        prefetch(c);
        const bool got = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&bars->acc_full, chunk_idx & 1, kErrWaitAcc));
        if (a.trace && a.trace_fine) trace_point(a, tp++);
        if (!got) ok = false;
        if (ok) {
          tc_fence_after();
          epilogue(c, step, G.scale);
        }
        tc_fence_before();
        mbar_arrive(&bars->acc_empty);
        ++chunk_idx;
        if (a.trace && a.trace_fine) trace_point(a, tp++);
      }
    };
    auto run_gemm = [&](int g, bool prefilled, const float* src, int ld, const float* rmax, auto&& epilogue) {
      run_gemm_pre(g, prefilled, src, ld, rmax, [](int) {}, epilogue);
    };
    // Warp-per-row RMSNorm (nn/rmsnorm.go:14-32) of cur, after the embedding (mode 1) or the
    // inter-block residual (mode 2) when asked: writes out (fp32, row stride out_ld), max |out|
    // per row (rmax, and rmax_g in global memory if given) and, if slice, the digit planes of the
    // normed row into the A slots of a GEMM with K = D (acquired and published here).
    auto norm_phase = [&](int mode, const float* gain, float* out, int out_ld, float* rmax, float* rmax_g, bool slice) {
      const int kts = (D + 127) / 128;
      if (slice)
        for (int kt = 0; kt < kts; ++kt) acquire(kt % kASlots);
#pragma unroll 2
      for (int u = 0; u < kRowsPerWarp; ++u) {
        const int rr = warp + kRowWarps * u;
        const int gr = tile * kRows + rr;
        const bool v = bars->rvalid[rr] != 0;
        float4 x[KF];
        float4* cur4 = reinterpret_cast<float4*>(a.cur + (size_t)gr * D);
        float4* bin4 = reinterpret_cast<float4*>(a.blockin + (size_t)gr * D);
        if (mode == 1) {
          const char4* e4 = reinterpret_cast<const char4*>(a.embed + (size_t)bars->rtok[rr] * D);
#pragma unroll
          for (int k = 0; k < KF; ++k) {
            const int f = lane + 32 * k;
            float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
            if (v && f < nf) {
              const char4 q = e4[f];
              y = make_float4(__fmul_rn((float)q.x, a.embed_scale), __fmul_rn((float)q.y, a.embed_scale),
                              __fmul_rn((float)q.z, a.embed_scale), __fmul_rn((float)q.w, a.embed_scale));
              cur4[f] = y;
              bin4[f] = y;
            }
            x[k] = y;
          }
        } else if (mode == 2) {
          float4 c4[KF], b4[KF];
#pragma unroll
          for (int k = 0; k < KF; ++k) {
            const int f = lane + 32 * k;
            const bool in = v && f < nf;
            c4[k] = in ? cur4[f] : make_float4(0.f, 0.f, 0.f, 0.f);
            b4[k] = in ? bin4[f] : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int k = 0; k < KF; ++k) {
            const int f = lane + 32 * k;
            float4 y = make_float4(__fadd_rn(b4[k].x, c4[k].x), __fadd_rn(b4[k].y, c4[k].y), __fadd_rn(b4[k].z, c4[k].z),
                                   __fadd_rn(b4[k].w, c4[k].w));
            if (v && f < nf) {
              cur4[f] = y;
              bin4[f] = y;
            }
            x[k] = y;
          }
        } else {
#pragma unroll
          for (int k = 0; k < KF; ++k) {
            const int f = lane + 32 * k;
            x[k] = (v && f < nf) ? cur4[f] : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < KF; ++k) {
          ss = __fmaf_rn(x[k].x, x[k].x, ss);
          ss = __fmaf_rn(x[k].y, x[k].y, ss);
          ss = __fmaf_rn(x[k].z, x[k].z, ss);
          ss = __fmaf_rn(x[k].w, x[k].w, ss);
        }
        ss = warp_sum(ss);
        float inv = 1.f;
        if (gain) inv = __fdiv_rn(1.0f, (float)sqrt((double)__fadd_rn(__fdiv_rn(ss, (float)D), 1e-5f)));
        float m = 0.f;
        float4* o4 = reinterpret_cast<float4*>(out + (size_t)gr * out_ld);
#pragma unroll
        for (int k = 0; k < KF; ++k) {
          const int f = lane + 32 * k;
          if (f < nf && gain) {
            const float4 gg = reinterpret_cast<const float4*>(gain)[f];
            x[k].x = __fmul_rn(__fmul_rn(x[k].x, inv), gg.x);
            x[k].y = __fmul_rn(__fmul_rn(x[k].y, inv), gg.y);
            x[k].z = __fmul_rn(__fmul_rn(x[k].z, inv), gg.z);
            x[k].w = __fmul_rn(__fmul_rn(x[k].w, inv), gg.w);
          }
          if (v && f < nf) o4[f] = x[k];
          if (f < nf) m = fmaxf(m, max4(x[k]));
        }
        m = v ? warp_max(m) : 0.f;
        if (lane == 0) {
          rmax[rr] = m;
          if (rmax_g) rmax_g[gr] = m;
        }
        if (slice) {
          const float is = row_inv_step(m);
#pragma unroll
          for (int k = 0; k < KF; ++k) {
            const int f = lane + 32 * k;
            if (f < nf) put4(sA, rr, 4 * f, x[k], is);
          }
        }
      }
      if (slice)
        for (int kt = 0; kt < kts; ++kt) publish(kt % kASlots);
    };
    // The per-channel vector src[0..n) of the next GEMM's epilogue, copied into shared memory
    // (between two row barriers: the previous epilogue's reads of the buffer are done, and every
    // row thread sees the copy), so the epilogues read it without global-memory latency. Vectors
    // longer than the buffer stay in global memory.
    auto stage_vec = [&](const float* src, int n) -> const float* {
      if (n > kVecMax) return src;
      row_bar();
      for (int i = t; i < n; i += kRowThreads) bars->vec[i] = src[i];
      row_bar();
      return bars->vec;
    };
    // max over the four threads of a row (each ran the epilogue on its columns) into rmax
    auto row_max_quad = [&](float mine, float* rmax) {
      bars->rowmax_part[h][r] = mine;
      row_bar();
      if (h == 0)
        rmax[r] = fmaxf(fmaxf(bars->rowmax_part[0][r], bars->rowmax_part[1][r]),
                        fmaxf(bars->rowmax_part[2][r], bars->rowmax_part[3][r]));
      row_bar();
    };

    int g = 0;
    // ---- output projection of the previous block's attention: cur += Out att s_out ----
    if (a.has_out) {
      if (h == 0) bars->rowmax_a[r] = ri.valid ? a.att_rowmax[grow] : 0.f;
      row_bar();
      float* cur = a.cur + (size_t)grow * D;
      run_gemm(g++, false, a.att, D, bars->rowmax_a, [&](int c, float step, float scale) {
        for (int j0 = h * 32; j0 < h * 32 + 32; j0 += 16) {
          const int n0 = c * kNC + j0;
          const bool act = ri.valid && n0 < D;
          float v[16];
          if (act) ld16(cur, n0, D, v);
          uint32_t a1[16], a2[16], a3[16];
          load_acc16(tmem, warp, j0, a1, a2, a3);
          if (!act) continue;
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], dequant(a1[j], a2[j], a3[j], step, scale));
          st16(cur, n0, D, v);
        }
      });
      row_bar();
      trace_point(a, tp++);
    }

    // ---- rule steps ----
    for (int s = 0; s < a.nsteps; ++s) {
      const int bs = a.bs0 + s;
      const int dil = a.dil[s];
      // norm cell n (after the embedding / residual on the first step), sliced for W_select
      norm_phase(s == 0 ? (a.embed_first ? 1 : (a.residual ? 2 : 0)) : 0, a.gamma, a.xbuf, 3 * D, bars->rowmax_n,
                 nullptr, true);
      row_bar();
      trace_point(a, tp++);
      // W_select epilogue: lambda = sigmoid(dot * s_sel + base) into the latch slot of xbuf
      float* xrow = a.xbuf + (size_t)grow * 3 * D;
      const float* lbase = stage_vec(a.latch_base, D);
      run_gemm(g++, true, nullptr, 0, bars->rowmax_n, [&](int c, float step, float scale) {
        for (int j0 = h * 32; j0 < h * 32 + 32; j0 += 16) {
          const int n0 = c * kNC + j0;
          const bool act = ri.valid && n0 < D;
          float base[16];
          if (act) ld16(lbase, n0, D, base);
          uint32_t a1[16], a2[16], a3[16];
          load_acc16(tmem, warp, j0, a1, a2, a3);
          if (!act) continue;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            base[j] = sigmoid_clamped(__fadd_rn(dequant(a1[j], a2[j], a3[j], step, scale), base[j]));
          st16(xrow + 2 * D, n0, D, base);
        }
      });
      row_bar();
      trace_point(a, tp++);
      const bool w1_resident = a.gemms[g].ktiles <= kASlots;
      // W1's planes go straight into this SM's plane cache (every chunk then comes from it)
      const bool w1_pre = !w1_resident && presliced(a.gemms[g]);
      bool w1_prefilled = false;
      // x's planes written to the cache: each thread fences its writes for the async proxy (the
      // producer's bulk copies read them) and arrives on a_pre
      auto announce_pre = [&]() {
        fence_proxy_async_global();
        mbar_arrive(&bars->a_pre);
      };
      if (decode) {
        // ---- decode: latch update, left neighbour, ring write; one warp per row ----
        const bool slice = w1_resident;
        const int kts = a.gemms[g].ktiles;
        if (slice)
          for (int kt = 0; kt < kts; ++kt) acquire(kt % kASlots);
#pragma unroll 2
        for (int u = 0; u < kRowsPerWarp; ++u) {
          const int rr = warp + kRowWarps * u;
          const int gr = tile * kRows + rr;
          const bool v = bars->rvalid[rr] != 0;
          const int pos = bars->rpos[rr];
          const size_t so = ((size_t)bars->rsess[rr] * a.total_steps + bs);
          const float4* x4 = reinterpret_cast<const float4*>(a.xbuf + (size_t)gr * 3 * D);
          float4* ls4 = reinterpret_cast<float4*>(a.latch + so * D);
          float4* ring4 = reinterpret_cast<float4*>(a.norm_ring + so * a.ring * D);
          const int lpos = pos - dil;
          float4 nv[KF], lam[KF], lo[KF], lf[KF];
#pragma unroll
          for (int k = 0; k < KF; ++k) {
            const int f = lane + 32 * k;
            const bool in = v && f < nf;
            const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
            nv[k] = in ? x4[f] : z;
            lam[k] = in ? x4[2 * nf + f] : z;
            lo[k] = (in && pos > 0) ? ls4[f] : z;
            lf[k] = (in && lpos >= 0) ? ring4[(size_t)(lpos % a.ring) * nf + f] : z;
          }
          float m = 0.f;
#pragma unroll
          for (int k = 0; k < KF; ++k) {
            const int f = lane + 32 * k;
            float4 l;
            l.x = __fadd_rn(__fmul_rn(lam[k].x, lo[k].x), __fmul_rn(__fsub_rn(1.0f, lam[k].x), nv[k].x));
            l.y = __fadd_rn(__fmul_rn(lam[k].y, lo[k].y), __fmul_rn(__fsub_rn(1.0f, lam[k].y), nv[k].y));
            l.z = __fadd_rn(__fmul_rn(lam[k].z, lo[k].z), __fmul_rn(__fsub_rn(1.0f, lam[k].z), nv[k].z));
            l.w = __fadd_rn(__fmul_rn(lam[k].w, lo[k].w), __fmul_rn(__fsub_rn(1.0f, lam[k].w), nv[k].w));
            lo[k] = l;
            if (v && f < nf) {
              ls4[f] = l;
              ring4[(size_t)(pos % a.ring) * nf + f] = nv[k];
              if (!slice && !w1_pre) {
                float4* xw = reinterpret_cast<float4*>(a.xbuf + (size_t)gr * 3 * D);
                xw[nf + f] = lf[k];
                xw[2 * nf + f] = l;
              }
            }
            if (f < nf) m = fmaxf(m, fmaxf(max4(nv[k]), fmaxf(max4(l), max4(lf[k]))));
          }
          m = v ? warp_max(m) : 0.f;
          if (lane == 0) bars->rowmax_a[rr] = m;
          if (slice || w1_pre) {
            const float is = row_inv_step(m);
#pragma unroll
            for (int k = 0; k < KF; ++k) {
              const int f = lane + 32 * k;
              if (f < nf) {
                if (slice) {
                  put4(sA, rr, 4 * f, nv[k], is);
                  put4(sA, rr, D + 4 * f, lf[k], is);
                  put4(sA, rr, 2 * D + 4 * f, lo[k], is);
                } else {
                  put4_g(acache, rr, 4 * f, nv[k], is);
                  put4_g(acache, rr, D + 4 * f, lf[k], is);
                  put4_g(acache, rr, 2 * D + 4 * f, lo[k], is);
                }
              }
            }
          }
        }
        if (slice) {
          for (int kt = 0; kt < kts; ++kt) publish(kt % kASlots);
          w1_prefilled = true;
        }
        if (w1_pre) announce_pre();
        row_bar();
      } else {
        // ---- prefill: latch scan, left neighbours, ring write and row maxima, in passes ----
        // (1) the latch recurrence over each segment, l_t = lam_t l_{t-1} + (1 - lam_t) n_t
        //     (updateLatch, stream.go:197-205), one (session slot, channel) at a time
        constexpr int kLC = 16;  // positions per chunk of the scan
        if (a.P <= kLC) {
          // short segments: the recurrence step by step, the loads of each run issued first
          for (int task = t; task < a.spt * D; task += kRowThreads) {
            const int slot = task / D, d = task - slot * D;
            const int sess = tile * a.spt + slot;
            if (sess >= a.n_sess) continue;
            const int len = a.seglen[sess];
            if (len <= 0) continue;
            const int p0 = a.pos0[sess];
            const size_t st_off = ((size_t)sess * a.total_steps + bs);
            float l = p0 == 0 ? 0.f : a.latch[st_off * D + d];
            float* x0 = a.xbuf + (size_t)(tile * kRows + slot * a.P) * 3 * D + d;
            for (int c0 = 0; c0 < len; c0 += 8) {
              float lam[8], nv[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const bool in = c0 + i < len;
                lam[i] = in ? x0[(size_t)(c0 + i) * 3 * D + 2 * D] : 0.f;
                nv[i] = in ? x0[(size_t)(c0 + i) * 3 * D] : 0.f;
              }
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                if (c0 + i < len) {
                  l = __fadd_rn(__fmul_rn(lam[i], l), __fmul_rn(__fsub_rn(1.0f, lam[i]), nv[i]));
                  x0[(size_t)(c0 + i) * 3 * D + 2 * D] = l;
                }
              }
            }
            a.latch[st_off * D + d] = l;
          }
        } else {
          // longer segments: a scan in chunks of kLC positions. The recurrence is affine in l, so
          // a chunk maps its input l to A l + B (A the product of its lambdas, B its output from
          // l = 0). (a) every chunk's (A, B) at once; (b) the chunks' inputs in order, per
          // channel; (c) every chunk replays the recurrence from its input, step by step as the
          // reference writes it. The chunks' (A, B) and inputs live in the free A slots (the
          // W_select MMAs that read them are complete; W1's planes are not written yet).
          const int nch = (a.P + kLC - 1) / kLC;
          float* cA = reinterpret_cast<float*>(sA);       // [spt][nch][D]: A, then the chunk's input
          float* cB = cA + (size_t)a.spt * nch * D;         // [spt][nch][D]: B
          const int ntask = a.spt * nch * D;
          auto chunk_of = [&](int task, int& slot, int& ch, int& d, int& sess, int& len, int& c0) {
            d = task % D;
            const int rest = task / D;
            ch = rest % nch;
            slot = rest / nch;
            sess = tile * a.spt + slot;
            len = sess < a.n_sess ? a.seglen[sess] : 0;
            c0 = ch * kLC;
            return c0 < len;
          };
          for (int task = t; task < ntask; task += kRowThreads) {
            int slot, ch, d, sess, len, c0;
            if (!chunk_of(task, slot, ch, d, sess, len, c0)) continue;
            const float* x0 = a.xbuf + (size_t)(tile * kRows + slot * a.P + c0) * 3 * D + d;
            float lam[kLC], nv[kLC];
#pragma unroll
            for (int i = 0; i < kLC; ++i) {
              const bool in = c0 + i < len;
              lam[i] = in ? x0[(size_t)i * 3 * D + 2 * D] : 1.f;
              nv[i] = in ? x0[(size_t)i * 3 * D] : 0.f;
            }
            float A = 1.f, B = 0.f;
#pragma unroll
            for (int i = 0; i < kLC; ++i) {
              B = __fadd_rn(__fmul_rn(lam[i], B), __fmul_rn(__fsub_rn(1.0f, lam[i]), nv[i]));
              A = __fmul_rn(A, lam[i]);
            }
            cA[task] = A;
            cB[task] = B;
          }
          row_bar();
          for (int task = t; task < a.spt * D; task += kRowThreads) {
            const int slot = task / D, d = task - slot * D;
            const int sess = tile * a.spt + slot;
            if (sess >= a.n_sess) continue;
            const int len = a.seglen[sess];
            if (len <= 0) continue;
            const size_t st_off = ((size_t)sess * a.total_steps + bs);
            float l = a.pos0[sess] == 0 ? 0.f : a.latch[st_off * D + d];
            for (int ch = 0; ch * kLC < len; ++ch) {
              const size_t i = ((size_t)slot * nch + ch) * D + d;
              const float A = cA[i];
              cA[i] = l;
              l = __fadd_rn(__fmul_rn(A, l), cB[i]);
            }
          }
          row_bar();
          for (int task = t; task < ntask; task += kRowThreads) {
            int slot, ch, d, sess, len, c0;
            if (!chunk_of(task, slot, ch, d, sess, len, c0)) continue;
            float* x0 = a.xbuf + (size_t)(tile * kRows + slot * a.P + c0) * 3 * D + d;
            float lam[kLC], nv[kLC];
#pragma unroll
            for (int i = 0; i < kLC; ++i) {
              const bool in = c0 + i < len;
              lam[i] = in ? x0[(size_t)i * 3 * D + 2 * D] : 0.f;
              nv[i] = in ? x0[(size_t)i * 3 * D] : 0.f;
            }
            float l = cA[task];
#pragma unroll
            for (int i = 0; i < kLC; ++i) {
              if (c0 + i < len) {
                l = __fadd_rn(__fmul_rn(lam[i], l), __fmul_rn(__fsub_rn(1.0f, lam[i]), nv[i]));
                x0[(size_t)i * 3 * D + 2 * D] = l;
              }
            }
            if (c0 + kLC >= len) a.latch[((size_t)sess * a.total_steps + bs) * D + d] = l;  // the segment's last
          }
        }
        if (a.trace && a.trace_fine) trace_point(a, tp++);
        if (w1_resident || w1_pre) {
          // (2) one warp per row: the left neighbour n(pos - dil) (from the segment, or from the
          //     ring before it), max |x| over x = [n | left | latch], and x sliced straight into
          //     W1's A slots (resident W1) or into this SM's plane cache (no fp32 copy of x goes
          //     back to memory)
          row_bar();  // the latch scan's rows
          const int kts = a.gemms[g].ktiles;
          if (w1_resident)
            for (int kt = 0; kt < kts; ++kt) acquire(kt % kASlots);
#pragma unroll 2
          for (int u = 0; u < kRowsPerWarp; ++u) {
            const int rr = warp + kRowWarps * u;
            const bool v = bars->rvalid[rr] != 0;
            const int tt = rr - (rr / a.P) * a.P;
            const int sess = bars->rsess[rr], lpos = bars->rpos[rr] - dil;
            const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
            const float4* x4 = reinterpret_cast<const float4*>(a.xbuf + (size_t)(tile * kRows + rr) * 3 * D);
            const float4* left4 =
                tt >= dil ? reinterpret_cast<const float4*>(a.xbuf + (size_t)(tile * kRows + rr - dil) * 3 * D)
                          : reinterpret_cast<const float4*>(a.norm_ring + ((size_t)sess * a.total_steps + bs) * a.ring * D +
                                                            (size_t)((lpos >= 0 ? lpos : 0) % a.ring) * D);
            const bool has_left = v && (tt >= dil || lpos >= 0);
            float4 nv[KF], lt[KF], lf[KF];
#pragma unroll
            for (int k = 0; k < KF; ++k) {
              const int f = lane + 32 * k;
              const bool in = v && f < nf;
              nv[k] = in ? x4[f] : z;
              lt[k] = in ? x4[2 * nf + f] : z;
              lf[k] = (in && has_left) ? left4[f] : z;
            }
            float m = 0.f;
#pragma unroll
            for (int k = 0; k < KF; ++k) m = fmaxf(m, fmaxf(max4(nv[k]), fmaxf(max4(lf[k]), max4(lt[k]))));
            m = v ? warp_max(m) : 0.f;
            if (lane == 0) bars->rowmax_a[rr] = m;
            const float is = row_inv_step(m);
#pragma unroll
            for (int k = 0; k < KF; ++k) {
              const int f = lane + 32 * k;
              if (f >= nf) continue;
              if (w1_resident) {
                put4(sA, rr, 4 * f, nv[k], is);
                put4(sA, rr, D + 4 * f, lf[k], is);
                put4(sA, rr, 2 * D + 4 * f, lt[k], is);
              } else {
                put4_g(acache, rr, 4 * f, nv[k], is);
                put4_g(acache, rr, D + 4 * f, lf[k], is);
                put4_g(acache, rr, 2 * D + 4 * f, lt[k], is);
              }
            }
          }
          if (w1_resident) {
            for (int kt = 0; kt < kts; ++kt) publish(kt % kASlots);
            w1_prefilled = true;
          } else {
            announce_pre();
          }
          row_bar();  // row maxima; the ring reads above come before the ring writes below
          if (a.trace && a.trace_fine) trace_point(a, tp++);
          // (3) the ring keeps the segment's last norm cells: task (slot, j, channel) copies
          //     position len - 1 - j (j < ring), four tasks' loads in flight before their stores
          const int rn = min(a.ring, a.P);
          const int ntask = a.spt * rn * D;
          for (int t0 = t; t0 < ntask; t0 += 4 * kRowThreads) {
            float val[4];
            float* dst[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              dst[q] = nullptr;
              val[q] = 0.f;
              const int task = t0 + q * kRowThreads;
              if (task >= ntask) continue;
              const int d = task % D, rest = task / D;
              const int j = rest % rn, slot = rest / rn;
              const int sess = tile * a.spt + slot;
              if (sess >= a.n_sess) continue;
              const int len = a.seglen[sess], tt = len - 1 - j;
              if (tt < 0) continue;
              val[q] = a.xbuf[(size_t)(tile * kRows + slot * a.P + tt) * 3 * D + d];
              dst[q] = a.norm_ring + ((size_t)sess * a.total_steps + bs) * a.ring * D +
                       (size_t)((a.pos0[sess] + tt) % a.ring) * D + d;
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (dst[q]) *dst[q] = val[q];
          }
          if (a.trace && a.trace_fine) trace_point(a, tp++);
        } else {
          // (2) left neighbours n(pos - dil): from the segment, or from the ring before it
          for (int idx = t; idx < kRows * D; idx += kRowThreads) {
            const int rr = idx / D, d = idx - rr * D;
            if (!bars->rvalid[rr]) continue;
            const int slot = rr / a.P, tt = rr - slot * a.P;
            const int sess = tile * a.spt + slot;
            const int p0 = a.pos0[sess];
            float* x = a.xbuf + (size_t)(tile * kRows + rr) * 3 * D;
            float left = 0.f;
            if (tt >= dil) left = a.xbuf[(size_t)(tile * kRows + rr - dil) * 3 * D + d];
            else if (p0 + tt - dil >= 0)
              left = a.norm_ring[((size_t)sess * a.total_steps + bs) * a.ring * D + (size_t)((p0 + tt - dil) % a.ring) * D + d];
            x[D + d] = left;
          }
          row_bar();
          if (a.trace && a.trace_fine) trace_point(a, tp++);
          // (3) the ring keeps the segment's last norm cells
          for (int task = t; task < a.spt * D; task += kRowThreads) {
            const int slot = task / D, d = task - slot * D;
            const int sess = tile * a.spt + slot;
            if (sess >= a.n_sess) continue;
            const int len = a.seglen[sess];
            const int p0 = a.pos0[sess];
            float* rg = a.norm_ring + ((size_t)sess * a.total_steps + bs) * a.ring * D + d;
            for (int tt = max(0, len - a.ring); tt < len; ++tt)
              rg[(size_t)((p0 + tt) % a.ring) * D] = a.xbuf[(size_t)(tile * kRows + slot * a.P + tt) * 3 * D + d];
          }
          if (a.trace && a.trace_fine) trace_point(a, tp++);
          // (4) max |x| of each row, one warp per row
#pragma unroll 2
          for (int u = 0; u < kRowsPerWarp; ++u) {
            const int rr = warp + kRowWarps * u;
            float m = 0.f;
            if (bars->rvalid[rr]) {
              const float* x = a.xbuf + (size_t)(tile * kRows + rr) * 3 * D;
              for (int e = lane; e < 3 * D; e += 32) m = fmaxf(m, fabsf(x[e]));
            }
            m = warp_max(m);
            if (lane == 0) bars->rowmax_a[rr] = m;
          }
        }
        row_bar();
      }
      trace_point(a, tp++);
      // W1 + GLU -> hidden (fp32 rows in hbuf), per-thread max |hidden|
      float hmax = 0.f;
      float* hrow = a.hbuf + (size_t)grow * H;
      const float* b1 = stage_vec(a.b1, 2 * H);
      run_gemm(g++, w1_prefilled, a.xbuf, 3 * D, bars->rowmax_a, [&](int c, float step, float scale) {
        for (int j0 = h * 16; j0 < h * 16 + 16; j0 += 8) {  // this thread's 16 of the chunk's 64 hidden units
          const int u0 = c * kHalfChunk + j0;
          const bool act = ri.valid && u0 < H;
          float bv[8], bg[8], hid[8];
          if (act) {
            ld8(b1, u0, H, bv);
            ld8(b1 + H, u0, H, bg);
          }
          uint32_t x1[8], x2[8], x3[8], y1[8], y2[8], y3[8];
          load_acc8x2(tmem, warp, j0, kHalfChunk + j0, x1, x2, x3, y1, y2, y3);  // value and gate columns
#pragma unroll
          for (int j = 0; j < 8; ++j) hid[j] = __fadd_rn(dequant(x1[j], x2[j], x3[j], step, scale), bv[j]);
          if (act) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float gt = __fadd_rn(dequant(y1[j], y2[j], y3[j], step, scale), bg[j]);
              hid[j] = __fmul_rn(hid[j], sigmoid_clamped(gt));
              if (u0 + j < H) hmax = fmaxf(hmax, fabsf(hid[j]));
            }
            st8(hrow, u0, H, hid);
          }
        }
      });
      row_max_quad(hmax, bars->rowmax_h);
      trace_point(a, tp++);
      // W2 + highway -> cur
      float* crow = a.cur + (size_t)grow * D;
      const float* b2 = stage_vec(a.b2, 2 * D);
      float cvp[16];  // this thread's cur values of the chunk, loaded before the accumulator wait
      auto cur_pre = [&](int c) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int d0 = c * kHalfChunk + h * 16 + 8 * i;
          if (ri.valid && d0 < D) ld8(crow, d0, D, *reinterpret_cast<float(*)[8]>(cvp + 8 * i));
        }
      };
      run_gemm_pre(g++, false, a.hbuf, H, bars->rowmax_h, cur_pre, [&](int c, float step, float scale) {
        for (int j0 = h * 16; j0 < h * 16 + 16; j0 += 8) {  // this thread's 16 of the chunk's 64 state channels
          const int d0 = c * kHalfChunk + j0;
          const bool act = ri.valid && d0 < D;
          float bd[8], bg[8], cv[8], od[8];
          if (act) {
            ld8(b2, d0, D, bd);
            ld8(b2 + D, d0, D, bg);
#pragma unroll
            for (int j = 0; j < 8; ++j) cv[j] = cvp[j0 - h * 16 + j];
          }
          uint32_t x1[8], x2[8], x3[8], y1[8], y2[8], y3[8];
          load_acc8x2(tmem, warp, j0, kHalfChunk + j0, x1, x2, x3, y1, y2, y3);  // delta and gate columns
#pragma unroll
          for (int j = 0; j < 8; ++j) od[j] = __fadd_rn(dequant(x1[j], x2[j], x3[j], step, scale), bd[j]);
          if (act) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float og = __fadd_rn(dequant(y1[j], y2[j], y3[j], step, scale), bg[j]);
              const float gate = sigmoid_clamped(og);
              cv[j] = __fadd_rn(__fmul_rn(__fsub_rn(1.0f, gate), cv[j]), __fmul_rn(gate, od[j]));
            }
            st8(crow, d0, D, cv);
          }
        }
      });
      row_bar();
      trace_point(a, tp++);
    }

    // ---- attention sublayer: norm (sliced for QKV) + QKV, keys/values into the ring ----
    if (a.has_attn) {
      norm_phase(a.nsteps == 0 ? (a.embed_first ? 1 : (a.residual ? 2 : 0)) : 0, a.attn_norm, a.xbuf, 3 * D,
                 bars->rowmax_n, nullptr, true);
      if (h == 0 && ri.valid) a.att_rowmax[grow] = 0.f;  // the attention kernel max-accumulates it
      row_bar();
      trace_point(a, tp++);
      // key/value rings, head-major: [K|V][head][slot][dh] (each head's window is contiguous)
      float* kvs = a.kv + ((size_t)a.attn_slot * a.n_sess + ri.session) * 2 * (size_t)a.cache * D;
      const bool to_ring = ri.valid && ri.t >= ri.len - a.cache;
      const int rslot = ri.pos % a.cache;
      const int dh = a.dh;
      float* lin = a.kvlin ? a.kvlin + ((size_t)ri.session * a.P + ri.t) * 2 * D : nullptr;
      float* qrow = a.qbuf + (size_t)grow * D;
      auto ring_at = [&](int which, int e) {  // element e (< D) of the key (0) or value (1)
        const int hh = e / dh;
        return kvs + (size_t)which * a.cache * D + ((size_t)hh * a.cache + rslot) * dh + (e - hh * dh);
      };
      run_gemm(g++, true, nullptr, 0, bars->rowmax_n, [&](int c, float step, float scale) {
        for (int j0 = h * 32; j0 < h * 32 + 32; j0 += 16) {
          uint32_t a1[16], a2[16], a3[16];
          load_acc16(tmem, warp, j0, a1, a2, a3);
          const int n0 = c * kNC + j0;
          if (!ri.valid || n0 >= 3 * D) continue;
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = dequant(a1[j], a2[j], a3[j], step, scale);
          const int part = n0 / D;
          const int e0 = n0 - part * D;
          if (n0 + 16 <= 3 * D && (n0 + 15) / D == part && (part == 0 || (e0 % dh) + 16 <= dh)) {
            if (part == 0) st16(qrow, e0, D, v);
            else {
              if (to_ring) st16(ring_at(part - 1, e0), 0, 16, v);
              if (lin) st16(lin + (part - 1) * D, e0, D, v);
            }
          } else {
            for (int j = 0; j < 16; ++j) {
              const int n = n0 + j;
              if (n >= 3 * D) break;
              const int p = n / D, e = n - p * D;
              if (p == 0) qrow[e] = v[j];
              else {
                if (to_ring) *ring_at(p - 1, e) = v[j];
                if (lin) lin[(p - 1) * D + e] = v[j];
              }
            }
          }
        }
      });
      trace_point(a, tp++);
    }

    // ---- final RMSNorm (the head's input) ----
    if (a.final_norm) {
      norm_phase(a.nsteps == 0 && !a.has_attn ? (a.embed_first ? 1 : (a.residual ? 2 : 0)) : 0, a.final_gain, a.fnorm,
                 D, bars->rowmax_n, a.fnorm_rowmax, false);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tmem_dealloc(tmem, 512);
}

}  // namespace eng
}  // namespace mc
