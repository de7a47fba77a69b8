// The device-error path of the bounded waits, exercised without a fault: one thread waits on an
// mbarrier that nothing arrives on, gives up after the wait limit (2 s), records the error word
// and returns; the host reads MC_DEVICE_TIMEOUT and the context stays usable.

namespace mc {
namespace eng {

__global__ void selftest_wait_kernel(int* gave_up) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_barrier_init();
  *gave_up = mbar_wait(&bar, 0, kErrWaitFull) ? 0 : 1;  // phase 0 never completes
}

}  // namespace eng
}  // namespace mc

extern "C" int mc_selftest_wait_timeout(int device) {
  clear_error();
  DeviceRestore restore_device;
  MC_CUDA(cudaSetDevice(device));
  DevBuf flag;
  if (cudaMalloc(&flag.p, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return set_error(kOutOfMemory, "mc_selftest_wait_timeout: cudaMalloc failed");
  }
  MC_CUDA(cudaMemset(flag.p, 0, sizeof(int)));
  eng::selftest_wait_kernel<<<1, 32>>>(static_cast<int*>(flag.p));
  MC_CUDA(cudaGetLastError());
  int gave_up = 0;
  MC_CUDA(cudaMemcpy(&gave_up, flag.p, sizeof(int), cudaMemcpyDeviceToHost));
  const int st = check_device_error(0);
  if (st == kOk || !gave_up) return set_error(kCudaError, "mc_selftest_wait_timeout: the wait did not give up");
  return st;  // MC_DEVICE_TIMEOUT, with the device's message
}
