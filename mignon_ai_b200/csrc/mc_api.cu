// C-ABI entry points of libmignoncuda (include/mignon_cuda.h).
#include <cstring>
#include <vector>

#include "../../include/mignon_cuda.h"
#include "mc_host.h"

namespace mc {
const char* last_error_cstr();
int gemm_i8_launch(const int8_t* a, const int8_t* w, int M, int N, int K, const float* row_scale,
                   const float* col_scale, const float* bias, int32_t* c_i32, float* y, cudaStream_t stream);
int gemm_f32a_launch(const float* a, const int8_t* w, int M, int N, int K, float w_scale, const float* bias,
                     float* y, int32_t* slices, float* row_max_scratch, cudaStream_t stream);

// Device buffer released when the scope ends.
struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};
}  // namespace mc

using namespace mc;

extern "C" {

const char* mc_last_error(void) { return last_error_cstr(); }

int mc_version(void) { return 100; }

int mc_gemm_i8_dev(const int8_t* a, const int8_t* w, int m, int n, int k, const float* row_scale,
                   const float* col_scale, const float* bias, int32_t* c_i32, float* y, void* stream) {
  clear_error();
  if (!a || !w) return set_error(kInvalidArgument, "mc_gemm_i8_dev: null operand");
  return gemm_i8_launch(a, w, m, n, k, row_scale, col_scale, bias, c_i32, y, (cudaStream_t)stream);
}

int mc_gemm_f32a_dev(const float* x, const int8_t* w, int m, int n, int k, float w_scale, const float* bias,
                     float* y, int32_t* slices, float* row_max_scratch, void* stream) {
  clear_error();
  if (!x || !w || !y || !row_max_scratch) return set_error(kInvalidArgument, "mc_gemm_f32a_dev: null pointer");
  return gemm_f32a_launch(x, w, m, n, k, w_scale, bias, y, slices, row_max_scratch, (cudaStream_t)stream);
}

int mc_gemm_i8(int device, const int8_t* a, const int8_t* w, int m, int n, int k, const float* row_scale,
               const float* col_scale, const float* bias, int32_t* c_i32, float* y) {
  clear_error();
  if (!a || !w || m <= 0 || n <= 0 || k <= 0) return set_error(kInvalidArgument, "mc_gemm_i8: bad arguments");
  MC_CUDA(cudaSetDevice(device));
  DevBuf da, dw, drs, dcs, db, dc, dy;
  const size_t mk = (size_t)m * k, nk = (size_t)n * k, mn = (size_t)m * n;
  MC_CUDA(cudaMalloc(&da.p, mk));
  MC_CUDA(cudaMalloc(&dw.p, nk));
  MC_CUDA(cudaMemcpy(da.p, a, mk, cudaMemcpyHostToDevice));
  MC_CUDA(cudaMemcpy(dw.p, w, nk, cudaMemcpyHostToDevice));
  if (row_scale) {
    MC_CUDA(cudaMalloc(&drs.p, 4 * (size_t)m));
    MC_CUDA(cudaMemcpy(drs.p, row_scale, 4 * (size_t)m, cudaMemcpyHostToDevice));
  }
  if (col_scale) {
    MC_CUDA(cudaMalloc(&dcs.p, 4 * (size_t)n));
    MC_CUDA(cudaMemcpy(dcs.p, col_scale, 4 * (size_t)n, cudaMemcpyHostToDevice));
  }
  if (bias) {
    MC_CUDA(cudaMalloc(&db.p, 4 * (size_t)n));
    MC_CUDA(cudaMemcpy(db.p, bias, 4 * (size_t)n, cudaMemcpyHostToDevice));
  }
  if (c_i32) MC_CUDA(cudaMalloc(&dc.p, 4 * mn));
  if (y) MC_CUDA(cudaMalloc(&dy.p, 4 * mn));
  int st = gemm_i8_launch((const int8_t*)da.p, (const int8_t*)dw.p, m, n, k, (const float*)drs.p,
                          (const float*)dcs.p, (const float*)db.p, (int32_t*)dc.p, (float*)dy.p, 0);
  if (st != kOk) return st;
  st = check_device_error(0);
  if (st != kOk) return st;
  if (c_i32) MC_CUDA(cudaMemcpy(c_i32, dc.p, 4 * mn, cudaMemcpyDeviceToHost));
  if (y) MC_CUDA(cudaMemcpy(y, dy.p, 4 * mn, cudaMemcpyDeviceToHost));
  return kOk;
}

}  // extern "C"
