// Single translation unit of libmignoncuda.so: every kernel and the C-ABI are compiled together so
// device globals (the error word) need no separate device linking.
#include "mc_host.cu"
#include "mc_gemm.cu"
#include "mc_api.cu"
