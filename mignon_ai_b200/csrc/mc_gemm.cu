// Isolated INT8 GEMMs on the 5th-generation tensor core (tcgen05 kind::i8).
//
// Two entry points share one structure (a 128-row M tile per CTA, K streamed through a ring of
// shared-memory stages, accumulators in TMEM, an epilogue by four row-owning warps):
//
//  * gemm_i8_kernel: int8 activations A[M x K] and weights W[N x K], both loaded by TMA. The s32
//    accumulators are exact; the epilogue writes them and/or y = acc * row_scale * col_scale + bias.
//    This is the config-5 sweep (per-channel weight scales, per-row activation scales).
//
//  * gemm_f32a_kernel: float32 activations, the reference's INT8 product (MatVecInt8,
//    internal/kernels/int8.go:31-41: y = (x . w) * scale + bias with x in float32). Each
//    activation row is sliced into three int8 digit planes (mc_sm100.cuh: slice3) by the
//    row-owning warps while the weights stream in by TMA; three MMAs per K step accumulate the
//    planes into three exact s32 accumulators that the epilogue recombines.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>

#include "mc_host.h"
#include "mc_sm100.cuh"

namespace mc {
namespace gemm {

constexpr int kBM = 128;   // rows per CTA (TMEM lanes)
constexpr int kBK = 128;   // K bytes per stage (one 128-byte swizzle row)

// ------------------------------------------------------------------------------------------------
// int8 x int8
// ------------------------------------------------------------------------------------------------
constexpr int kI8BN = 256;
constexpr int kI8Stages = 4;
constexpr int kI8StageA = kBM * kBK;     // 16 KB
constexpr int kI8StageB = kI8BN * kBK;   // 32 KB
constexpr int kI8EpiWarps = 8;
constexpr int kI8Staging = kI8EpiWarps * 32 * 128;  // per epilogue warp: 32 rows x 128 bytes, 16-byte chunks swizzled
constexpr int kI8Smem = kI8Stages * (kI8StageA + kI8StageB) + kI8Staging + 1024 + 256;  // ring, staging, barriers

struct I8Args {
  int M, N, K;
  const float* row_scale;  // [M] or null (1)
  const float* col_scale;  // [N] or null (1)
  const float* bias;       // [N] or null
  int32_t* c_i32;          // [M x N] or null
  float* y;                // [M x N] or null
};

// The epilogue of one 128-row x 256-column accumulator for one epilogue warp: TMEM lanes
// quad*32..+31 (output rows r0..r0+31), columns half*128..+127 of the accumulator at column
// acc_col. 32 columns at a time, each thread (= row) writes its 128-byte row into the warp's
// staging tile with the 16-byte chunks XOR-swizzled by row (conflict-free), then 8 lanes per row
// store whole 128-byte lines (4 rows per instruction).
__device__ __forceinline__ void i8_drain_tile(const I8Args& args, uint32_t tmem, int acc_col, int r0, int n0, int half,
                                              int lane, uint32_t* st) {
  const int quad = (r0 / 32) & 3;
  const int row = r0 + lane;
  const float rs = (args.row_scale && row < args.M) ? args.row_scale[row] : 1.0f;
  for (int pass = 0; pass < 2; ++pass) {
    int32_t* out = pass == 0 ? args.c_i32 : reinterpret_cast<int32_t*>(args.y);
    if (!out) continue;
    for (int c = half * 128; c < half * 128 + 128; c += 32) {
      uint32_t r[32];
      tmem_ld32(tmem_addr(tmem, quad * 32, acc_col + c), r);
      tmem_wait_ld();
      const int n = n0 + c;
      if (pass == 1) {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float cs = args.col_scale ? args.col_scale[n + e] : 1.0f;
          // Separately rounded multiplies and add (never contracted into an FMA).
          float tv = __fmul_rn((float)(int)r[e], rs);
          tv = __fmul_rn(tv, cs);
          if (args.bias) tv = __fadd_rn(tv, args.bias[n + e]);
          r[e] = __float_as_uint(tv);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<uint4*>(st + lane * 32 + 4 * (j ^ (lane & 7))) =
            make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int piece = lane + 32 * i;  // 32 rows x 8 chunks of 16 bytes
        const int rr = piece >> 3, ch = piece & 7;
        const int grow = r0 + rr;
        const uint4 v = *reinterpret_cast<const uint4*>(st + rr * 32 + 4 * (ch ^ (rr & 7)));
        if (grow < args.M) *reinterpret_cast<uint4*>(out + (size_t)grow * args.N + n + 4 * ch) = v;
      }
      __syncwarp();
    }
  }
}

// Persistent: one CTA per SM walks the 128 x 256 output tiles (N-tiles fastest, so neighbouring
// CTAs share the A tile in L2). Warp 0 issues the TMA loads through a 4-stage ring, warp 1 the
// MMAs into one of two TMEM accumulators (2 x 256 columns), and eight epilogue warps drain the
// other accumulator (warp w: TMEM lanes 32*(w%4), columns 128*((w-2)/4)) while the next tile's
// MMAs run, so output stores overlap the tensor core.
constexpr int kI8Threads = 64 + 32 * kI8EpiWarps;

__global__ void __launch_bounds__(kI8Threads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w, I8Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + kI8Stages * kI8StageA;
  uint32_t* stg = reinterpret_cast<uint32_t*>(sb + kI8Stages * kI8StageB);  // [warp][32 rows][32 words]
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + kI8Stages * kI8StageB + kI8Staging);
  uint64_t* empty = full + kI8Stages;
  uint64_t* acc_full = empty + kI8Stages;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int ktiles = (args.K + kBK - 1) / kBK;
  const int ntn = args.N / kI8BN, ntm = (args.M + kBM - 1) / kBM;
  const int ntiles = ntn * ntm;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kI8Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kI8EpiWarps);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // TMA producer: every tile's K tiles through the ring
    if (lane == 0) {
      prefetch_tensormap(&map_a);
      prefetch_tensormap(&map_w);
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int m0 = (t / ntn) * kBM, n0 = (t % ntn) * kI8BN;
        for (int kt = 0; kt < ktiles; ++kt, ++it) {
          const int s = it % kI8Stages;
          if (it >= kI8Stages && !mbar_wait_or_abort(&empty[s], ((it / kI8Stages) - 1) & 1, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], kI8StageA + kI8StageB);
          tma_load_2d(sa + s * kI8StageA, &map_a, kt * kBK, m0, &full[s]);
          tma_load_2d(sb + s * kI8StageB, &map_w, kt * kBK, n0, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // MMA issuer: tile i accumulates into TMEM buffer i % 2 once the epilogue has drained it
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(kBM, kI8BN);
      uint32_t it = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++i) {
        const int b = i & 1;
        if (i >= 2 && !mbar_wait_or_abort(&acc_empty[b], ((i / 2) - 1) & 1, kErrWaitAccFree)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * kI8BN;
        for (int kt = 0; kt < ktiles; ++kt, ++it) {
          const int s = it % kI8Stages;
          if (!mbar_wait_or_abort(&full[s], (it / kI8Stages) & 1, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_sw128(sa + s * kI8StageA);
          const uint64_t db = smem_desc_sw128(sb + s * kI8StageB);
          const int ksteps = min(4, (args.K - kt * kBK + 31) / 32);
          for (int kk = 0; kk < ksteps; ++kk)
            mma_i8(acc, da + 2 * kk, db + 2 * kk, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[b]);
      }
    }
  } else {
    // Epilogue warps: warp w reads TMEM lanes 32*(w%4)..+31 (rows) and columns 128*((w-2)/4)..+127
    const int quad = warp % 4, half = (warp - 2) / 4;
    uint32_t i = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
      const int b = i & 1;
      const int m0 = (t / ntn) * kBM, n0 = (t % ntn) * kI8BN;
      // TMEM loads are warp-collective: the whole warp takes the same branch.
      if (!__all_sync(0xffffffffu, mbar_wait_or_abort(&acc_full[b], (i / 2) & 1, kErrWaitAcc))) break;
      tc_fence_after();
      i8_drain_tile(args, tmem, b * kI8BN, m0 + quad * 32, n0, half, lane, stg + (size_t)(warp - 2) * 32 * 32);
      // the accumulator is read: the MMA warp may reuse it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------------------------------------
// int8 x int8 on CTA pairs (cta_group::2)
// ------------------------------------------------------------------------------------------------
// The same persistent structure over 256 x 256 output tiles, one per cluster of two CTAs on two
// SMs. Each CTA loads its own 128 rows of A and its own 128 rows of W (output channels) per K
// stage; the first CTA's MMA thread issues M = 256, N = 256 MMAs that read both CTAs' stages, and
// each CTA's TMEM receives its 128 output rows over all 256 columns. Per SM and per 128 x 256
// output tile that is A 128 x K + W 128 x K bytes through L2 instead of A 128 x K + W 256 x K,
// the operand traffic the single-CTA kernel waits on.
//
// Barriers: both CTAs' loads complete on the first CTA's full[s] (the first CTA expects the
// pair's bytes); the MMA thread's commits arrive on empty[s] and acc_full[b] in both CTAs; both
// CTAs' epilogue warps arrive on the first CTA's acc_empty[b]. No load uses cluster multicast.
constexpr int kPStages = 6;
constexpr int kPStageA = kBM * kBK;  // 16 KB: this CTA's 128 rows of A
constexpr int kPStageB = 128 * kBK;  // 16 KB: this CTA's 128 rows of W
constexpr int kPSmem = kPStages * (kPStageA + kPStageB) + kI8Staging + 1024 + 256;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kI8Threads, 1)
    gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                        I8Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + kPStages * kPStageA;
  uint32_t* stg = reinterpret_cast<uint32_t*>(sb + kPStages * kPStageB);
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + kPStages * kPStageB + kI8Staging);
  uint64_t* empty = full + kPStages;
  uint64_t* acc_full = empty + kPStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs
  const int pair = blockIdx.x / 2, npairs = gridDim.x / 2;
  const int ktiles = (args.K + kBK - 1) / kBK;
  const int ntn = args.N / 256, ntm = (args.M + 255) / 256;
  const int ntiles = ntn * ntm;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kI8EpiWarps);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before any load or commit reaches them
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&map_a);
      prefetch_tensormap(&map_w);
      const uint32_t full0 = cluster_map_shared(full, 0);  // the first CTA's full[0]
      uint32_t it = 0;
      bool ok = true;
      for (int t = pair; t < ntiles && ok; t += npairs) {
        const int m0 = (t / ntn) * 256 + (int)rank * 128, n0 = (t % ntn) * 256 + (int)rank * 128;
        for (int kt = 0; kt < ktiles; ++kt, ++it) {
          const int s = it % kPStages;
          if (it >= kPStages && !mbar_wait_or_abort(&empty[s], ((it / kPStages) - 1) & 1, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (kPStageA + kPStageB));
          tma_load_2d_pair(sa + s * kPStageA, &map_a, kt * kBK, m0, full0 + 8u * s);
          tma_load_2d_pair(sb + s * kPStageB, &map_w, kt * kBK, n0, full0 + 8u * s);
        }
      }
      // Until the MMAs have read every stage this CTA filled, the peer's MMA thread still reads
      // its shared memory: wait for each stage's last release before leaving.
      if (ok) {
        for (uint32_t j = it > kPStages ? it - kPStages : 0; j < it; ++j)
          if (!mbar_wait_or_abort(&empty[j % kPStages], (j / kPStages) & 1, kErrWaitEmpty)) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = idesc_i8(256, 256);
      uint32_t it = 0, i = 0;
      bool ok = true;
      for (int t = pair; t < ntiles && ok; t += npairs, ++i) {
        const int b = i & 1;
        if (i >= 2 && !mbar_wait_or_abort(&acc_empty[b], ((i / 2) - 1) & 1, kErrWaitAccFree)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * 256;
        for (int kt = 0; kt < ktiles; ++kt, ++it) {
          const int s = it % kPStages;
          if (!mbar_wait_or_abort(&full[s], (it / kPStages) & 1, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_sw128(sa + s * kPStageA);
          const uint64_t db = smem_desc_sw128(sb + s * kPStageB);
          const int ksteps = min(4, (args.K - kt * kBK + 31) / 32);
          for (int kk = 0; kk < ksteps; ++kk)
            mma_i8_pair(acc, da + 2 * kk, db + 2 * kk, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
          mma_commit_pair(&empty[s], 0x3);
        }
        if (ok) mma_commit_pair(&acc_full[b], 0x3);
      }
    }
  } else {
    const int quad = warp % 4, half = (warp - 2) / 4;
    const uint32_t acc_empty0 = cluster_map_shared(acc_empty, 0);
    uint32_t i = 0;
    for (int t = pair; t < ntiles; t += npairs, ++i) {
      const int b = i & 1;
      const int m0 = (t / ntn) * 256 + (int)rank * 128, n0 = (t % ntn) * 256;
      if (!__all_sync(0xffffffffu, mbar_wait_or_abort(&acc_full[b], (i / 2) & 1, kErrWaitAcc))) break;
      tc_fence_after();
      i8_drain_tile(args, tmem, b * 256, m0 + quad * 32, n0, half, lane, stg + (size_t)(warp - 2) * 32 * 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8u * b);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other may still reach its shared memory or TMEM
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, 512);
}

// ------------------------------------------------------------------------------------------------
// float32 activations (three digit planes) x int8 weights
// ------------------------------------------------------------------------------------------------
constexpr int kFBN = 128;
constexpr int kFStages = 3;
constexpr int kFTile = kBM * kBK;              // one 128 x 128 int8 tile
constexpr int kFStage = 3 * kFTile + kFTile;   // three digit planes + the weight tile
constexpr int kFSmem = kFStages * kFStage + 1024 + 256;

struct F32Args {
  int M, N, K;
  const float* a;          // [M x K] float32
  const float* row_max;    // [M] max |a_row|
  float w_scale;           // per-tensor weight scale (MatVecInt8's scale)
  const float* bias;       // [N] or null
  float* y;                // [M x N]
  int32_t* slices;         // [3 x M x N] or null: the exact per-plane accumulators
};

__global__ void row_absmax_kernel(const float* a, int M, int K, float* out) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= M) return;
  float m = 0.f;
  for (int k = lane; k < K; k += 32) m = fmaxf(m, fabsf(a[(size_t)row * K + k]));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) out[row] = m;
}

__global__ void __launch_bounds__(160, 1)
    gemm_f32a_kernel(const __grid_constant__ CUtensorMap map_w, F32Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kFStages * kFStage);
  uint64_t* empty = full + kFStages;
  uint64_t* accfull = empty + kFStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accfull + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kFBN;
  const int ktiles = (args.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFStages; ++s) {
      mbar_init(&full[s], 128 + 1);  // 128 slicing threads + the weight-tile expect_tx arrival
      mbar_init(&empty[s], 1);
    }
    mbar_init(accfull, 1);
    fence_barrier_init();
  }
  if (warp == 4) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    // Producers: thread t slices row m0 + t of each K tile into the three digit planes.
    const int t = threadIdx.x;
    const int row = m0 + t;
    const bool valid = row < args.M;
    const float inv = valid ? row_inv_step(args.row_max[row]) : 0.f;
    const float* arow = args.a + (size_t)(valid ? row : 0) * args.K;
    bool ok = true;
    for (int kt = 0; kt < ktiles; ++kt) {
      const int s = kt % kFStages;
      if (kt >= kFStages && !mbar_wait_or_abort(&empty[s], ((kt / kFStages) - 1) & 1, kErrWaitEmpty)) {
        ok = false;
        break;
      }
      uint8_t* st = smem + s * kFStage;
      if (t == 0) {
        mbar_arrive_expect_tx(&full[s], kFTile);
        tma_load_2d(st + 3 * kFTile, &map_w, kt * kBK, n0, &full[s]);
      }
      const int k0 = kt * kBK;
#pragma unroll 2
      for (int c = 0; c < 8; ++c) {
        uint32_t p1[4], p2[4], p3[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float x[4];
          const int k = k0 + c * 16 + q * 4;
          if (valid && k + 3 < args.K) {
            float4 v = *reinterpret_cast<const float4*>(arow + k);
            x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) x[e] = (valid && k + e < args.K) ? arow[k + e] : 0.f;
          }
          Digits3 d[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) d[e] = slice3(x[e], inv);
          p1[q] = pack4(d[0].d1, d[1].d1, d[2].d1, d[3].d1);
          p2[q] = pack4(d[0].d2, d[1].d2, d[2].d2, d[3].d2);
          p3[q] = pack4(d[0].d3, d[1].d3, d[2].d3, d[3].d3);
        }
        const uint32_t off = sw128_offset(t, c);
        *reinterpret_cast<uint4*>(st + off) = make_uint4(p1[0], p1[1], p1[2], p1[3]);
        *reinterpret_cast<uint4*>(st + kFTile + off) = make_uint4(p2[0], p2[1], p2[2], p2[3]);
        *reinterpret_cast<uint4*>(st + 2 * kFTile + off) = make_uint4(p3[0], p3[1], p3[2], p3[3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&full[s]);
    }
    // Epilogue (warp-uniform branch: TMEM loads are warp-collective).
    if (__all_sync(0xffffffffu, ok && mbar_wait_or_abort(accfull, 0, kErrWaitAcc))) {
      tc_fence_after();
      const int quad = warp;  // warps 0..3 own TMEM lanes 32*warp..
      const float step = valid ? row_step(args.row_max[row]) : 0.f;
      for (int c = 0; c < kFBN; c += 32) {
        uint32_t r1[32], r2[32], r3[32];
        tmem_ld32(tmem_addr(tmem, quad * 32, c), r1);
        tmem_ld32(tmem_addr(tmem, quad * 32, kFBN + c), r2);
        tmem_ld32(tmem_addr(tmem, quad * 32, 2 * kFBN + c), r3);
        tmem_wait_ld();
        if (!valid) continue;
        const int n = n0 + c;
        float* yrow = args.y + (size_t)row * args.N + n;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const double acc = combine3((int)r1[j + e], (int)r2[j + e], (int)r3[j + e]);
            const float dot = (float)(acc * (double)step);
            // MatVecInt8: y = dot * scale, then y += bias, each rounded (int8.go:37-40).
            float t2 = __fmul_rn(dot, args.w_scale);
            if (args.bias) t2 = __fadd_rn(t2, args.bias[n + j + e]);
            v[e] = t2;
          }
          *reinterpret_cast<float4*>(yrow + j) = make_float4(v[0], v[1], v[2], v[3]);
        }
        if (args.slices) {
          const size_t plane = (size_t)args.M * args.N;
          int32_t* o = args.slices + (size_t)row * args.N + n;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            o[j] = (int)r1[j];
            o[plane + j] = (int)r2[j];
            o[2 * plane + j] = (int)r3[j];
          }
        }
      }
    }
  } else if (warp == 4 && lane == 0) {
    const uint32_t idesc = idesc_i8(kBM, kFBN);
    bool ok = true;
    for (int kt = 0; kt < ktiles && ok; ++kt) {
      const int s = kt % kFStages;
      if (!mbar_wait_or_abort(&full[s], (kt / kFStages) & 1, kErrWaitFull)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint8_t* st = smem + s * kFStage;
      const uint64_t db = smem_desc_sw128(st + 3 * kFTile);
      const int ksteps = min(4, (args.K - kt * kBK + 31) / 32);
#pragma unroll
      for (int p = 0; p < 3; ++p) {
        const uint64_t da = smem_desc_sw128(st + p * kFTile);
        for (int kk = 0; kk < ksteps; ++kk)
          mma_i8(tmem + p * kFBN, da + 2 * kk, db + 2 * kk, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
      }
      mma_commit(&empty[s]);
    }
    if (ok) mma_commit(accfull);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------------------------------------
// float32 activations with the weights on the MMA's M side (K up to 1536)
// ------------------------------------------------------------------------------------------------
// A persistent CTA takes blocks of kWR activation rows. It slices a block's rows once into the
// three digit planes, which stay in shared memory for the whole block, stacked along the MMA's N
// (plane p's rows follow plane p-1's: N = 3 kWR), and streams every 128-row tile of W past them
// (TMA loads through a kWStages ring): D[weight row][plane, activation row] accumulates the three
// plane products of 128 output columns x kWR rows in one MMA chain, into one of two TMEM
// accumulators, so one tile's epilogue overlaps the next tile's MMAs. An epilogue thread owns one
// output column (its TMEM lane); a warp stores 32 consecutive columns of a row at a time. The
// arithmetic is gemm_f32a_kernel's: the same digits, exact plane accumulators, the same epilogue.
constexpr int kWR = 32;                  // activation rows per block
constexpr int kWN = 3 * kWR;             // MMA N: the three planes stacked
constexpr int kWStages = 4;              // weight-tile ring (deeper rings measured no faster)
constexpr int kWMaxKT = 12;              // K tiles whose planes stay resident (K <= 1536)
constexpr int kWPlaneTile = kWN * kBK;   // one K tile of the block's three planes (12 KB)
constexpr int kWThreads = 192;           // 4 slicing / epilogue warps, the MMA warp, the producer warp
constexpr size_t kWSmemMax = 1024 + (size_t)kWMaxKT * kWPlaneTile + (size_t)kWStages * kFTile + 256;

inline size_t gemm_f32a_wm_smem(int kt) { return 1024 + (size_t)kt * kWPlaneTile + (size_t)kWStages * kFTile + 256; }

__global__ void __launch_bounds__(kWThreads, 1)
    gemm_f32a_wm_kernel(const __grid_constant__ CUtensorMap map_w, F32Args args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ float s_step[kWR];  // the slicing step of each row of the current block
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int KT = (args.K + kBK - 1) / kBK;
  uint8_t* sP = smem;                                        // [KT][3 kWR rows x 128 B] digit planes
  uint8_t* sW = smem + (size_t)KT * kWPlaneTile;             // [kWStages][128 x 128 B] weight tiles
  uint64_t* w_full = reinterpret_cast<uint64_t*>(sW + (size_t)kWStages * kFTile);  // [kWStages]
  uint64_t* w_empty = w_full + kWStages;
  uint64_t* acc_full = w_empty + kWStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint64_t* p_full = acc_empty + 2;         // the current block's planes are written
  uint64_t* p_empty = p_full + 1;           // the current block's MMAs are done with them
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(p_empty + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nblocks = (args.M + kWR - 1) / kWR, ntiles = args.N / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);  // one arrival per epilogue warp
    }
    mbar_init(p_full, 128);
    mbar_init(p_empty, 1);
    fence_barrier_init();
  }
  if (warp == 4) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 5) {
    // ---------------- weight tiles by TMA, in the MMA warp's order ----------------
    if (lane == 0) {
      uint32_t widx = 0;
      bool ok = true;
      for (int b = blockIdx.x; b < nblocks && ok; b += gridDim.x)
        for (int j = 0; j < ntiles && ok; ++j)
          for (int kt = 0; kt < KT; ++kt, ++widx) {
            const int s = widx % kWStages;
            if (widx >= kWStages && !mbar_wait_or_abort(&w_empty[s], ((widx / kWStages) - 1) & 1, kErrWaitEmpty)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&w_full[s], kFTile);
            tma_load_2d(sW + (size_t)s * kFTile, &map_w, kt * kBK, j * 128, &w_full[s]);
          }
    }
  } else if (warp == 4) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(128, kWN);
      const uint64_t dw0 = smem_desc_sw128(sW), dp0 = smem_desc_sw128(sP);
      uint32_t widx = 0, tidx = 0, nb = 0;
      bool ok = true;
      for (int b = blockIdx.x; b < nblocks && ok; b += gridDim.x, ++nb) {
        if (!mbar_wait_or_abort(p_full, nb & 1, kErrWaitFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int j = 0; j < ntiles && ok; ++j, ++tidx) {
          const int slot = tidx & 1;
          if (tidx >= 2 && !mbar_wait_or_abort(&acc_empty[slot], ((tidx / 2) - 1) & 1, kErrWaitAccFree)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t dt = tmem + (uint32_t)slot * 128;
          for (int kt = 0; kt < KT; ++kt, ++widx) {
            const int s = widx % kWStages;
            if (!mbar_wait_or_abort(&w_full[s], (widx / kWStages) & 1, kErrWaitFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            // descriptors advance by their encoded start address (bytes / 16)
            const uint64_t da = dw0 + (uint64_t)(s * (kFTile >> 4));
            const uint64_t db = dp0 + (uint64_t)(kt * (kWPlaneTile >> 4));
            const int ksteps = min(4, (args.K - kt * kBK + 31) / 32);
            for (int kk = 0; kk < ksteps; ++kk) mma_i8(dt, da + 2 * kk, db + 2 * kk, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
            mma_commit(&w_empty[s]);
          }
          if (!ok) break;
          mma_commit(&acc_full[slot]);
        }
        if (!ok) break;
        mma_commit(p_empty);  // arrives once every MMA of the block has read its planes
      }
    }
  } else {
    // ---------------- slicing (per block) and epilogues (per weight tile) ----------------
    uint32_t tidx = 0, nb = 0;
    bool ok = true;
    for (int b = blockIdx.x; b < nblocks; b += gridDim.x, ++nb) {
      const int m0 = b * kWR;
      if (nb > 0) ok = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(p_empty, (nb - 1) & 1, kErrWaitEmpty));
      if (ok) {
        // warp w slices rows w, w + 4, ...; lane l the K values 4l..4l+3 of every K tile (a warp
        // reads 512 consecutive bytes of the row per tile, all tiles' loads in flight together)
        for (int r = warp; r < kWR; r += 4) {
          const int m = m0 + r;
          const bool valid = m < args.M;
          const float rm = valid ? args.row_max[m] : 0.f;
          const float inv = row_inv_step(rm);
          if (lane == 0) s_step[r] = row_step(rm);
          const float* arow = args.a + (size_t)(valid ? m : 0) * args.K;
          float4 v[kWMaxKT];
#pragma unroll
          for (int kt = 0; kt < kWMaxKT; ++kt) {
            const int k = kt * kBK + 4 * lane;
            v[kt] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (kt < KT && valid && k < args.K) {
              if (k + 4 <= args.K) {
                v[kt] = *reinterpret_cast<const float4*>(arow + k);
              } else {
                v[kt].x = arow[k];
                if (k + 1 < args.K) v[kt].y = arow[k + 1];
                if (k + 2 < args.K) v[kt].z = arow[k + 2];
              }
            }
          }
#pragma unroll
          for (int kt = 0; kt < kWMaxKT; ++kt) {
            if (kt >= KT) break;
            const float x[4] = {v[kt].x, v[kt].y, v[kt].z, v[kt].w};
            Digits3 d[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) d[e] = slice3(x[e], inv);
            uint8_t* tile = sP + (size_t)kt * kWPlaneTile;
            const int chunk = lane >> 2, byte = (4 * lane) & 15;
            *reinterpret_cast<uint32_t*>(tile + sw128_offset(r, chunk) + byte) = pack4(d[0].d1, d[1].d1, d[2].d1, d[3].d1);
            *reinterpret_cast<uint32_t*>(tile + sw128_offset(kWR + r, chunk) + byte) =
                pack4(d[0].d2, d[1].d2, d[2].d2, d[3].d2);
            *reinterpret_cast<uint32_t*>(tile + sw128_offset(2 * kWR + r, chunk) + byte) =
                pack4(d[0].d3, d[1].d3, d[2].d3, d[3].d3);
          }
        }
        fence_proxy_async_smem();  // the planes, read by the MMAs (async proxy)
      }
      mbar_arrive(p_full);
      asm volatile("bar.sync 1, 128;" ::: "memory");  // s_step of every row of the block
      for (int j = 0; j < ntiles; ++j, ++tidx) {
        const int slot = tidx & 1;
        const bool got = __all_sync(0xffffffffu, ok && mbar_wait_or_abort(&acc_full[slot], (tidx / 2) & 1, kErrWaitAcc));
        if (!got) ok = false;
        uint32_t r1[32], r2[32], r3[32];
        if (ok) {
          tc_fence_after();
          const uint32_t base = tmem_addr(tmem, 32 * warp, (uint32_t)slot * 128);
          tmem_ld32(base, r1);
          tmem_ld32(base + kWR, r2);
          tmem_ld32(base + 2 * kWR, r3);
          tmem_wait_ld();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[slot]);
        if (!ok) continue;
        const int n = j * 128 + 32 * warp + lane;
        const float bn = args.bias ? args.bias[n] : 0.f;
#pragma unroll 4
        for (int r = 0; r < kWR; ++r) {
          const int m = m0 + r;
          if (m >= args.M) break;
          const double acc = combine3((int)r1[r], (int)r2[r], (int)r3[r]);
          const float dot = (float)(acc * (double)s_step[r]);
          // MatVecInt8: y = dot * scale, then y += bias, each rounded (int8.go:37-40).
          float y = __fmul_rn(dot, args.w_scale);
          if (args.bias) y = __fadd_rn(y, bn);
          args.y[(size_t)m * args.N + n] = y;
          if (args.slices) {
            const size_t plane = (size_t)args.M * args.N, o = (size_t)m * args.N + n;
            args.slices[o] = (int)r1[r];
            args.slices[plane + o] = (int)r2[r];
            args.slices[2 * plane + o] = (int)r3[r];
          }
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");  // s_step is rewritten by the next block's slicing
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) tmem_dealloc(tmem, 256);
}

}  // namespace gemm

// ------------------------------------------------------------------------------------------------
// Host launchers
// ------------------------------------------------------------------------------------------------
// Per-device set-up of the GEMM kernels, done once per device under a lock: the shared-memory
// size attribute of a kernel is a setting of the device that is current when it is made, and the
// multiprocessor count (the persistent grid) can differ between devices.
static int gemm_device_setup(int* n_sm, int* n_pairs = nullptr) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static int sms[kMaxDevices] = {0};    // 0: not set up yet
  static int pairs[kMaxDevices] = {0};  // CTA pairs of gemm_i8_pair_kernel resident at once
  int dev = 0;
  MC_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(kUnsupported, "gemm: device ordinal above 63");
  std::lock_guard<std::mutex> lk(mu);
  if (sms[dev] == 0) {
    MC_CUDA(cudaFuncSetAttribute(gemm::gemm_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm::kI8Smem));
    MC_CUDA(cudaFuncSetAttribute(gemm::gemm_i8_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 gemm::kPSmem));
    {
      // SMs pair up within a GPC, so the resident pairs can be fewer than half the SMs
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2, 1, 1);
      cfg.blockDim = dim3(gemm::kI8Threads, 1, 1);
      cfg.dynamicSmemBytes = gemm::kPSmem;
      int nc = 0;
      if (cudaOccupancyMaxActiveClusters(&nc, gemm::gemm_i8_pair_kernel, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();  // no pairs: the single-CTA kernel runs
        nc = 0;
      }
      pairs[dev] = nc;
    }
    MC_CUDA(cudaFuncSetAttribute(gemm::gemm_f32a_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm::kFSmem));
    MC_CUDA(cudaFuncSetAttribute(gemm::gemm_f32a_wm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)gemm::kWSmemMax));
    int n = 0;
    MC_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    sms[dev] = std::max(n, 1);
  }
  *n_sm = sms[dev];
  if (n_pairs) *n_pairs = pairs[dev];
  return kOk;
}

int gemm_i8_launch(const int8_t* a, const int8_t* w, int M, int N, int K, const float* row_scale,
                   const float* col_scale, const float* bias, int32_t* c_i32, float* y, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || N % gemm::kI8BN != 0 || K % 16 != 0)
    return set_error(kInvalidArgument, "gemm_i8: need M,N,K > 0, N % 256 == 0 and K % 16 == 0");
  if (!c_i32 && !y) return set_error(kInvalidArgument, "gemm_i8: no output");
  int n_sm = 0, n_pairs = 0;
  const int st = gemm_device_setup(&n_sm, &n_pairs);
  if (st != kOk) return st;
  gemm::I8Args args{M, N, K, row_scale, col_scale, bias, c_i32, y};
  // CTA pairs (cta_group::2) unless MC_GEMM_I8_SINGLE is set or no pair fits on the device
  const bool pair = n_pairs > 0 && !getenv("MC_GEMM_I8_SINGLE");
  CUtensorMap ma, mw;
  if (!make_tmap_i8(&ma, a, M, K, K, gemm::kBK, gemm::kBM)) return kCudaError;
  if (!make_tmap_i8(&mw, w, N, K, K, gemm::kBK, pair ? 128 : gemm::kI8BN)) return kCudaError;
  if (pair) {
    const int tiles = (N / 256) * ((M + 255) / 256);
    gemm::gemm_i8_pair_kernel<<<2 * std::min(tiles, n_pairs), gemm::kI8Threads, gemm::kPSmem, stream>>>(ma, mw, args);
  } else {
    const int tiles = (N / gemm::kI8BN) * ((M + gemm::kBM - 1) / gemm::kBM);
    gemm::gemm_i8_kernel<<<std::min(tiles, n_sm), gemm::kI8Threads, gemm::kI8Smem, stream>>>(ma, mw, args);
  }
  MC_CUDA(cudaGetLastError());
  return kOk;
}

int gemm_f32a_launch(const float* a, const int8_t* w, int M, int N, int K, float w_scale, const float* bias,
                     float* y, int32_t* slices, float* row_max_scratch, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || N % gemm::kFBN != 0 || K % 16 != 0)
    return set_error(kInvalidArgument, "gemm_f32a: need M,N,K > 0, N % 128 == 0 and K % 16 == 0");
  CUtensorMap mw;
  if (!make_tmap_i8(&mw, w, N, K, K, gemm::kBK, gemm::kFBN)) return kCudaError;
  int n_sm = 0;
  const int st = gemm_device_setup(&n_sm);
  if (st != kOk) return st;
  gemm::row_absmax_kernel<<<(M + 7) / 8, 256, 0, stream>>>(a, M, K, row_max_scratch);
  gemm::F32Args args{M, N, K, a, row_max_scratch, w_scale, bias, y, slices};
  const int kt = (K + gemm::kBK - 1) / gemm::kBK;
  const char* old_kernel = getenv("MC_GEMM_F32A_TILED");  // the one-tile-per-CTA kernel, for comparison
  if (kt <= gemm::kWMaxKT && !old_kernel) {
    // weights on M: each CTA slices 32 activation rows once and runs every weight tile past them
    const int nblocks = (M + gemm::kWR - 1) / gemm::kWR;
    gemm::gemm_f32a_wm_kernel<<<std::min(nblocks, n_sm), gemm::kWThreads, gemm::gemm_f32a_wm_smem(kt), stream>>>(mw, args);
  } else {
    dim3 grid(N / gemm::kFBN, (M + gemm::kBM - 1) / gemm::kBM);
    gemm::gemm_f32a_kernel<<<grid, 160, gemm::kFSmem, stream>>>(mw, args);
  }
  MC_CUDA(cudaGetLastError());
  return kOk;
}

// ------------------------------------------------------------------------------------------------
// Allocation-free form of the float32-activation GEMM
// ------------------------------------------------------------------------------------------------
// Some callers cannot allocate device memory: a host runtime that may only pass buffers it
// registered in advance, or a service whose GPU memory is budgeted once at start-up. For them, the one
// scratch buffer this GEMM needs, the largest magnitude of every activation row (one float per
// row), lives in this fixed device array. Every GPU that loads the library holds it (256 KB)
// until the process exits.
constexpr int kNoAllocMaxRows = 65536;
static __device__ __align__(256) float g_noalloc_row_max[kNoAllocMaxRows];

// Device address of the array on the current device. Host code may not pass the array's name to
// a kernel (on the host it is only a stand-in), so the address is looked up once per device with
// that device current, and cached.
static int noalloc_row_max(float** out) {
  static std::mutex mu;
  static float* addr[64] = {nullptr};
  int dev = 0;
  MC_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(kUnsupported, "device ordinal above 63");
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_row_max);
    if (e != cudaSuccess)
      return set_error(kCudaError, std::string("cudaGetSymbolAddress(g_noalloc_row_max): ") + cudaGetErrorString(e));
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return kOk;
}

// The float32-activation GEMM with its row-maximum scratch in g_noalloc_row_max: allocates
// nothing. Rows above kNoAllocMaxRows are rejected. All calls share the array, which keeps the
// last call's values; each call rewrites every entry it reads before reading it, so nothing needs
// clearing, but calls that overlap on the GPU race on it and must be serialized by the caller.
int gemm_f32a_noalloc_launch(const float* a, const int8_t* w, int M, int N, int K, float w_scale, const float* bias,
                             float* y, cudaStream_t stream) {
  if (M > kNoAllocMaxRows)
    return set_error(kInvalidArgument, "gemm_f32a_noalloc: m = " + std::to_string(M) + " is above the fixed maximum of " +
                                           std::to_string(kNoAllocMaxRows) + " rows");
  // every shape check before the first CUDA call, so a rejected call has no side effects
  if (M <= 0 || N <= 0 || K <= 0 || N % gemm::kFBN != 0 || K % 16 != 0)
    return set_error(kInvalidArgument, "gemm_f32a_noalloc: need M,N,K > 0, N % 128 == 0 and K % 16 == 0");
  float* row_max = nullptr;
  const int st = noalloc_row_max(&row_max);
  if (st != kOk) return st;
  return gemm_f32a_launch(a, w, M, N, K, w_scale, bias, y, nullptr, row_max, stream);
}

}  // namespace mc
