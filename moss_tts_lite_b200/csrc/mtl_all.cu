// Single translation unit for libmtl_b200.so (device globals such as the
// error word are shared by every kernel without relocatable device code).
#include "w4_gemv.cu"
#include "w4_tc.cu"
#include "w4_tcb.cu"
#include "step_kernels.cu"
#include "attn_decode.cu"
#include "w4_gemm.cu"
#include "w4_chain.cu"
#include "w4_chainb.cu"
#include "attn_prefill.cu"
#include "sampling.cu"
#include "capi.cu"
#include "noalloc.cu"
