// libreax_fmha_post.so -- attention forward (bias / qpos modes) and the qpos mode with the fused attn_post
// (sigmoid gate + row scatter) epilogue, sm_100a.  ABI: libreax_fmha_post/reax_fmha_v11.cu:565-590, plus the
// head-dimension extensions declared in include/reax_abi.h.
#include "fmha.cuh"

REAX_DEFINE_STATUS_EXPORT()
REAX_DEFINE_FMHA_EXPORTS()
REAX_DEFINE_FMHA_QP_EXPORT()
