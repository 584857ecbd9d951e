// Single translation unit of libindecis_b200.so: the kernels share device
// globals (the error flag) without relocatable device code.
#include "gemm_i8.cu"
#include "gemm_persist.cu"
#include "rows_fast.cu"
#include "rows.cu"
#include "rows_ln.cu"
#include "attention.cu"
#include "attention_tc.cu"
#include "attention_short.cu"
#include "siglip.cu"
#include "capi.cu"
#include "siglip_capi.cu"
#include "noalloc.cu"
