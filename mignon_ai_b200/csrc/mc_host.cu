// Host-side helpers of libmignoncuda (see mc_host.h).
#include <cudaTypedefs.h>

#include <mutex>

#include "mc_host.h"
#include "mc_sm100.cuh"

namespace mc {

static thread_local std::string t_last_error;

int set_error(int status, const std::string& msg) {
  t_last_error = msg;
  return status;
}

void clear_error() { t_last_error.clear(); }

const char* last_error_cstr() { return t_last_error.c_str(); }

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_tmap_i8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch,
                  uint32_t box_cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) {
    set_error(kCudaError, "cuTensorMapEncodeTiled is not available from the driver");
    return false;
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(kCudaError, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
    return false;
  }
  return true;
}

int check_device_error(cudaStream_t stream) {
  int code = 0;
  MC_CUDA(cudaMemcpyFromSymbolAsync(&code, g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream));
  MC_CUDA(cudaStreamSynchronize(stream));
  if (code != 0) {
    int zero = 0;
    MC_CUDA(cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream));
    MC_CUDA(cudaStreamSynchronize(stream));
    return set_error(kDeviceTimeout, "device wait gave up (code " + std::to_string(code) +
                                         "); the kernel returned without finishing its work");
  }
  return kOk;
}

}  // namespace mc
