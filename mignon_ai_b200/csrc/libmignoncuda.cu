// Single translation unit of libmignoncuda.so: every kernel and the C-ABI are compiled together so
// device globals (the error word) and shared device helpers need no separate device linking.
#include "mc_host.cu"
#include "mc_gemm.cu"
#include "mc_modelfile.cu"
#include "mc_block.cu"
#include "mc_block_decode.cu"
#include "mc_attn.cu"
#include "mc_head.cu"
#include "mc_policy.cu"
#include "mc_engine_host.cu"
#include "mc_api.cu"
#include "mc_sched.cu"
#include "mc_convert.cu"
