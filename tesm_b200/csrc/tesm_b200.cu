// Unity build of libtesm_b200.so: one translation unit so that device globals shared
// between kernels need no relocatable device code.
#include "capi.cu"
#include "quant.cu"
#include "gemv.cu"
#include "gemm_tc.cu"
#include "scan.cu"
#include "siso.cu"
#include "global_tc.cu"
#include "mimo.cu"
#include "decode.cu"
#include "model.cu"
#include "noalloc.cu"
