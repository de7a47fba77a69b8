/*
 * libmignoncuda — C-ABI of the B200 (sm_100a) engine for mignon-ai's INT8 inference path.
 *
 * Plain C types only: pointers, sizes, status codes. Every function returns an mc_status
 * (0 = MC_OK); mc_last_error() returns a thread-local message for the last failure. The caller
 * owns host buffers; the library owns device memory it allocates. Functions whose names end in
 * _dev take device pointers and a CUDA stream (cudaStream_t passed as void*) and do not
 * synchronize; all others take host pointers and return when their results are in host memory.
 *
 * Each entry point names the reference interface it replaces (paths relative to the
 * mignon-ai repository).
 */
#ifndef MIGNON_CUDA_H
#define MIGNON_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  MC_OK = 0,
  MC_INVALID_ARGUMENT = 1,
  MC_CUDA_ERROR = 2,
  MC_BAD_MODEL = 3,
  MC_OUT_OF_MEMORY = 4,
  MC_DEVICE_TIMEOUT = 5,
  MC_UNSUPPORTED = 6
} mc_status;

/* Message of the last failed call on this thread ("" after a success). */
const char* mc_last_error(void);

/* Library version: major*10000 + minor*100 + patch. */
int mc_version(void);

/* ---------------------------------------------------------------------------------------------
 * Isolated INT8 GEMMs (the INT8 product kernels.MatVecInt8, internal/kernels/int8.go:31-41,
 * batched over rows; the config-5 sweep entry point).
 * ------------------------------------------------------------------------------------------- */

/* C[m,n] = sum_k A[m,k] * W[n,k] with int8 A [M x K] and W [N x K] (row-major, K contiguous),
 * exact s32 accumulators. Writes c_i32 [M x N] if non-null and
 * y[m,n] = ((float)C[m,n] * row_scale[m]) * col_scale[n] + bias[n] if y is non-null (null scales
 * count as 1, a null bias as 0). Requires N % 256 == 0, K % 16 == 0. Device pointers. */
int mc_gemm_i8_dev(const int8_t* a, const int8_t* w, int m, int n, int k, const float* row_scale,
                   const float* col_scale, const float* bias, int32_t* c_i32, float* y, void* stream);

/* y[m,n] = dot(x[m,:], W[n,:]) * w_scale + bias[n] with float32 activations x [M x K], as
 * MatVecInt8 (int8.go:33-41) computes it per row. Each row is sliced into three int8 digit
 * planes; if slices is non-null the three exact s32 plane accumulators are written to it
 * ([3 x M x N]). row_max_scratch: device float[M]. Requires N % 128 == 0, K % 16 == 0. */
int mc_gemm_f32a_dev(const float* x, const int8_t* w, int m, int n, int k, float w_scale, const float* bias,
                     float* y, int32_t* slices, float* row_max_scratch, void* stream);

/* Host-pointer form of mc_gemm_i8_dev: copies in, runs on `device`, copies out. */
int mc_gemm_i8(int device, const int8_t* a, const int8_t* w, int m, int n, int k, const float* row_scale,
               const float* col_scale, const float* bias, int32_t* c_i32, float* y);

#ifdef __cplusplus
}
#endif
#endif /* MIGNON_CUDA_H */
