// libreax_howu.so -- the linear-attention layer kernels (conv + SiLU + L2 norm, chunked KKT inverse, chunked gated
// delta rule with and without the fused gated RMSNorm, reduce + residual + RMSNorm) and the attention forward
// entry points the reference also exports from this library, sm_100a.
// ABI: libreax_howu/reax_howu.cu:363-376, reax_kkt.cu:263-272, reax_howu_norm_v3.cu:431-435,
// reax_rarn_final.cu:98-106, reax_conv_v2.cu:164-189, reax_fmha_v8.cu:435-450.
#include "conv.cuh"
#include "fmha.cuh"
#include "howu_tc.cuh"
#include "kkt.cuh"
#include "rarn.cuh"

REAX_DEFINE_STATUS_EXPORT()
REAX_DEFINE_FMHA_EXPORTS()
REAX_DEFINE_RARN_EXPORT()
REAX_DEFINE_CONV_EXPORTS()
REAX_DEFINE_KKT_EXPORTS()
REAX_DEFINE_HOWU_EXPORTS()
