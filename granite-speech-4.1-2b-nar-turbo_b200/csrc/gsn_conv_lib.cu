// Single translation unit of libgsn_conv.so: the device status word (gsn_ptx.cuh) must have exactly one
// definition visible to every kernel without relocatable device code.
#include "layernorm.cu"
#include "dwconv.cu"
#include "dwconv_mma_sm100.cu"
#include "gemm_sm100.cu"
#include "quant_rows.cu"
#include "gemm_glu_dw_sm100.cu"
#include "attention_sm100.cu"
#include "ctc_head.cu"
#include "capi.cu"
