// Blackwell (sm_100a) building blocks: mbarriers with bounded waits, TMA loads, the 5th-generation
// tensor core (tcgen05: TMEM allocation, kind::i8 MMA, commit, TMEM loads) and the shared-memory
// operand layout the MMA reads.
//
// Every wait is bounded: after kWaitLimitNs of polling it records an error code in the device
// error word and returns false, so a kernel never spins forever on a barrier that will not
// complete. Callers then skip the rest of their work and still free their TMEM.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace mc {

// Error word written by device code (0 = ok). Read and cleared by the host after each call. The
// library is one translation unit, so this is its only definition.
__device__ int g_device_error = 0;

enum DeviceError : int {
  kErrNone = 0,
  kErrWaitFull = 1,     // a consumer timed out waiting for operands
  kErrWaitEmpty = 2,    // a producer timed out waiting for a free stage
  kErrWaitAcc = 3,      // the epilogue timed out waiting for the accumulator
  kErrWaitAccFree = 4,  // the MMA issuer timed out waiting for the epilogue
  kErrBadToken = 5,     // reserved: token ids are clamped, never rejected
  kErrBounds = 6,       // an index check failed (the access was skipped)
};

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_device_error, 0, code); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase with the given parity to complete; false (and an error record) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int err_code) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(a, parity)) return true;
    if ((i & 255u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) {
      record_error(err_code);
      return false;
    }
  }
}

// A wait that gives up immediately once any thread of the grid has recorded an error, so one
// failure does not cost every waiter its full time limit.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, int err_code) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(a, parity)) return true;
    if ((i & 255u) == 0) {
      if (*((volatile int*)&g_device_error) != 0) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        record_error(err_code);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Async-proxy fences and TMA
// ---------------------------------------------------------------------------------------------
// Makes this thread's generic-proxy global-memory writes visible to later async-proxy reads
// (bulk copies) by threads that synchronize with it afterwards.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Makes this thread's generic-proxy shared-memory writes visible to the async proxy (TMA, MMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2-D tiled TMA load (no multicast) completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Untiled bulk copy global -> shared (no multicast); both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// L2 cache policies for bulk copies (per-instruction hints; no device setting changes):
// evict_first for data read once (the key/value rings streamed by attention), evict_last for
// data every CTA reads again (weight tiles), so streaming reads do not push the weights out of L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// bulk_load with an L2 cache policy.
__device__ __forceinline__ void bulk_load_hint(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------------------------------------
// Clusters of two CTAs (a CTA pair running one cta_group::2 MMA)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the variable at p in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t cluster_map_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// Every thread of every CTA of the cluster; orders prior writes (barrier inits included) before
// what the other CTAs do after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrives on an mbarrier given by its shared::cluster address (this CTA's or a peer's), with the
// default CTA-scope release: it hands over TMEM (ordered by the tcgen05 fences around it), not
// global memory, so it need not wait for this thread's global stores to become visible to the
// cluster (a cluster-scope release did, and held each epilogue warp until its stores drained).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 2-D tiled TMA load (no multicast) into this CTA's shared memory, completing on an mbarrier that
// may sit in the peer CTA of the pair (shared::cluster address): the pair's operand halves all
// complete on the barrier of the CTA that issues the MMA.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar_cluster_addr) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------------------------
// tcgen05: TMEM and MMA
// ---------------------------------------------------------------------------------------------
// Allocates ncols (power of two >= 32) TMEM columns; one full warp executes it. The TMEM address
// is written to *smem_dst.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Instruction descriptor of tcgen05.mma kind::i8: signed 8-bit A and B, both K-major, s32
// accumulator, M x N tile (bit layout of the PTX ISA instruction-descriptor table).
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4)                       // D format: s32
         | (1u << 7)                     // A format: signed 8-bit
         | (1u << 10)                    // B format: signed 8-bit
         | ((uint32_t)(n >> 3) << 17)    // N / 8
         | ((uint32_t)(m >> 4) << 24);   // M / 16
}

// Shared-memory matrix descriptor of a K-major operand in the 128-byte swizzled layout: rows of
// 128 bytes (128 int8 K-values), 8-row groups 1024 bytes apart; the tile base is 1024-aligned.
// Advancing K by 32 bytes within the swizzle row adds 2 to the encoded start address.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* tile) {
  const uint32_t addr = smem_u32(tile);
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);        // start address
  d |= (uint64_t)1u << 16;                        // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024u >> 4) << 32;              // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1u << 46;                        // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                        // layout: 128-byte swizzle
  return d;
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread. No memory clobber: the operands are
// ordered by the (volatile, clobbering) mbarrier waits and fences around it, and volatile asm
// statements keep their order.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Arrives on the mbarrier once all previously issued MMAs of this thread have completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// TMEM of a CTA pair: one warp of each CTA (the same warp index in both) allocates the same
// columns in both CTAs' TMEM; the pair MMA writes rows 0-127 of its M = 256 tile to the first
// CTA's lanes and rows 128-255 to the second's.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D (+)= A * B^T over a CTA pair, issued by one thread of the pair's first CTA: A's rows 0-127
// and B's rows 0-127 are read from its shared memory, A's rows 128-255 and B's rows 128-255 from
// the same addresses in the peer CTA.
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Arrives on the mbarrier at this address in each CTA of cta_mask once the pair MMAs issued so far
// by this thread have completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane (warp w reads lanes 32*(w%4)..+31).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// TMEM address of (lane, column) relative to an allocation base.
__device__ __forceinline__ uint32_t tmem_addr(uint32_t base, uint32_t lane, uint32_t col) {
  return base + (lane << 16) + col;
}

// ---------------------------------------------------------------------------------------------
// Swizzled operand tiles written by threads
// ---------------------------------------------------------------------------------------------
// Byte offset of (row, 16-byte chunk) in a 128-row x 128-byte tile in the 128-byte swizzled
// K-major layout (the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B and the MMA reads).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return (row >> 3) * 1024u + (row & 7u) * 128u + ((chunk ^ (row & 7u)) << 4);
}

// ---------------------------------------------------------------------------------------------
// Activation slicing: float32 rows as three signed 8-bit digit planes
// ---------------------------------------------------------------------------------------------
// A row x with m = max|x| is written as x ~= (m/127) * (d1 + d2/254 + d3/254^2), each digit an
// integer in [-127, 127]: q = x*127/m, d1 = rint(q), d2 = rint((q-d1)*254), d3 = rint(...).
// The residual is at most 0.5/254^2 of one step of q, i.e. below 6.1e-8 * m: the three digit
// planes carry about 24 bits of each activation, the resolution of float32.
constexpr float kDigitBase = 254.0f;
constexpr double kInvDigitBase = 1.0 / 254.0;

struct Digits3 {
  int d1, d2, d3;
};

__device__ __forceinline__ Digits3 slice3(float x, float inv_step) {
  const float q = x * inv_step;
  const float d1 = rintf(q);
  const float t2 = (q - d1) * kDigitBase;
  const float d2 = rintf(t2);
  const float t3 = (t2 - d2) * kDigitBase;
  const float d3 = rintf(t3);
  return {(int)d1, (int)d2, (int)d3};
}

// The step of the first digit plane for a row whose largest magnitude is m, and its inverse.
// slice3 with the digits left in the low byte of float bit patterns, ready to pack: adding
// 1.5 * 2^23 to |v| < 2^22 rounds v to the nearest integer (ties to even, as rintf) and leaves it,
// two's complement, in the low mantissa bits. Same digits as slice3.
__device__ __forceinline__ void slice3_bits(float x, float inv, uint32_t& u1, uint32_t& u2, uint32_t& u3) {
  const float M = 12582912.0f;
  const float q = __fmul_rn(x, inv);
  const float s1 = __fadd_rn(q, M);
  const float t2 = __fmul_rn(__fsub_rn(q, __fsub_rn(s1, M)), kDigitBase);
  const float s2 = __fadd_rn(t2, M);
  const float t3 = __fmul_rn(__fsub_rn(t2, __fsub_rn(s2, M)), kDigitBase);
  const float s3 = __fadd_rn(t3, M);
  u1 = __float_as_uint(s1);
  u2 = __float_as_uint(s2);
  u3 = __float_as_uint(s3);
}

// Packs the low bytes of a, b, c, d into one word (a in the lowest byte).
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Rows whose largest magnitude is below 1e-30 are treated as zero rows (their inverse step would
// overflow float32).
__device__ __forceinline__ float row_step(float m) { return m >= 1e-30f ? m * (1.0f / 127.0f) : 0.f; }
__device__ __forceinline__ float row_inv_step(float m) { return m >= 1e-30f ? 127.0f / m : 0.f; }

// Combines the three slice accumulators into the dot product of the sliced row with the weights.
__device__ __forceinline__ double combine3(int32_t a1, int32_t a2, int32_t a3) {
  return (double)a1 + ((double)a2 + (double)a3 * kInvDigitBase) * kInvDigitBase;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) | ((uint32_t)(d & 0xFF) << 24);
}

}  // namespace mc
