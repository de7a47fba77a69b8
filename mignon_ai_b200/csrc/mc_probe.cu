// The int8 rate of the tensor pipe, measured: the denominator of every INT8 roofline fraction.
//
// One CTA per multiprocessor; one thread issues back-to-back tcgen05.mma kind::i8 instructions of
// the largest single-CTA shape (M = 128, N = 256, K = 32) whose operands stay resident in shared
// memory, alternating between two TMEM accumulators, with no loads and no epilogue: the kernel
// does nothing but tensor-pipe work. The operands hold a pseudo-random byte pattern, because the
// power the tensor core draws (and so the clock it keeps under the power cap) depends on the
// operand bits; zero operands would overstate the rate a real GEMM can sustain.

namespace mc {
namespace probe {

constexpr int kThreads = 128;
constexpr int kTileA = 128 * 128;  // 128 rows x 128 K bytes
constexpr int kTileB = 256 * 128;  // 256 rows x 128 K bytes
constexpr int kSmem = kTileA + kTileB + 1024 /*align*/ + 64 /*barrier, TMEM address*/;

__global__ void __launch_bounds__(kThreads, 1) mma_i8_rate_kernel(int iters, uint32_t seed) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + kTileA;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sb + kTileB);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int warp = threadIdx.x / 32;

  // operands: a multiplicative hash of the word index (any bytes are valid int8 values)
  uint32_t* w = reinterpret_cast<uint32_t*>(smem);
  for (int i = threadIdx.x; i < (kTileA + kTileB) / 4; i += kThreads) {
    uint32_t h = (uint32_t)i * 2654435761u + seed;
    h ^= h >> 15;
    h *= 2246822519u;
    h ^= h >> 13;
    w[i] = h;
  }
  fence_proxy_async_smem();  // the generic-proxy writes above, seen by the MMA's async-proxy reads
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (threadIdx.x == 0) {
    const uint32_t idesc = idesc_i8(128, 256);
    const uint64_t da = smem_desc_sw128(sa), db = smem_desc_sw128(sb);
    for (int it = 0; it < iters; ++it) {
      const uint32_t acc = tmem + (uint32_t)(it & 1) * 256;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) mma_i8(acc, da + 2 * kk, db + 2 * kk, idesc, kk > 0 ? 1u : 0u);
    }
    mma_commit(bar);
    mbar_wait(bar, 0, kErrWaitAcc);  // bounded: records an error and returns if it runs out
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

}  // namespace probe
}  // namespace mc

extern "C" int mc_probe_mma_i8(int device, int iters, int launches, double* tops, double* ms) {
  using namespace mc;
  clear_error();
  DeviceRestore restore_device;
  if (!tops || !ms || iters < 1 || iters > (1 << 22) || launches < 1)
    return set_error(kInvalidArgument, "mc_probe_mma_i8: iters in [1, 2^22], launches >= 1, non-null outputs");
  MC_CUDA(cudaSetDevice(device));
  int n_sm = 0;
  MC_CUDA(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, device));
  MC_CUDA(cudaFuncSetAttribute(probe::mma_i8_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, probe::kSmem));
  cudaStream_t s;
  MC_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  cudaEvent_t e0, e1;
  MC_CUDA(cudaEventCreate(&e0));
  MC_CUDA(cudaEventCreate(&e1));
  probe::mma_i8_rate_kernel<<<n_sm, probe::kThreads, probe::kSmem, s>>>(iters, 1u);  // warm-up
  MC_CUDA(cudaEventRecord(e0, s));
  for (int l = 0; l < launches; ++l) probe::mma_i8_rate_kernel<<<n_sm, probe::kThreads, probe::kSmem, s>>>(iters, 2u + l);
  MC_CUDA(cudaEventRecord(e1, s));
  MC_CUDA(cudaGetLastError());
  int st = check_device_error(s);
  float t = 0.f;
  if (st == kOk) MC_CUDA(cudaEventElapsedTime(&t, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaStreamDestroy(s);
  if (st != kOk) return st;
  *ms = (double)t / launches;
  const double ops = 2.0 * 128 * 256 * 128 * (double)iters * n_sm;  // per launch: iters x (128 x 256 x 128) MACs per SM
  *tops = ops / (*ms * 1e-3) / 1e12;
  return kOk;
}
