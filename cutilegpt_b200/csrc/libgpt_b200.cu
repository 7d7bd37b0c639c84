// Single translation unit of libgpt_b200.so (see build.py).
#include "capi.cu"
#include "elementwise.cu"
#include "gemm_tc.cu"
#include "gemm_skinny.cu"
#include "gemm_simt.cu"
#include "attention.cu"
#include "decode.cu"
#include "decode_noalloc.cu"
