// sfb200.cu — single translation unit of libsfb200.so (sm_100a).
#include "common.cuh"
#include "attn_tc.cu"
#include "attn_simt.cu"
#include "dequant.cu"
#include "w8a16_gemm.cu"
#include "rdt_ops.cu"
#include "rdt1b.cu"
#include "capi.cu"
