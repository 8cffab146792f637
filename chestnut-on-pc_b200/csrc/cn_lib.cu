// Single translation unit of libchestnut.so: device globals (the device error
// word) are then shared by every kernel without relocatable device code.
#include "cn_gemm.cu"
#include "cn_gemm_noalloc.cu"
#include "cn_reduce.cu"
#include "cn_ops.cu"
#include "cn_attn.cu"
#include "cn_trunk.cu"
#include "cn_stem.cu"
#include "cn_decode.cu"
#include "cn_engine.cu"
#include "cn_warp.cu"
