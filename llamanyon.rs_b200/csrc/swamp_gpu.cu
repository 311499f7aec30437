// swamp_gpu.cu -- unity translation unit for libswamp_gpu.so.
//
// The library is compiled as one translation unit so that device globals
// (the per-device error flag) have exactly one definition without relocatable
// device code.
#include "sg_layout.cu"
#include "sg_gemv_mma.cu"
#include "sg_gemv_q6k.cu"
#include "sg_gemm.cu"
#include "sg_api.cu"
#include "sg_synth.cu"
#include "sg_ops.cu"
#include "sg_noalloc.cu"
#include "sg_gguf.cu"
