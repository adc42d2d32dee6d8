// libreax_plain.so -- plain GEMM D = X W^T with bf16 output, sm_100a (tcgen05 + TMA).
// ABI: libreax_plain/gemm_plain2.cu:31-57 (reax_gemm_ncfg, reax_gemm_cfgname, reax_gemm).
#include "gemm_sm100.cuh"

REAX_DEFINE_STATUS_EXPORT()

namespace {
// Configuration names are ABI data (kept verbatim); each index selects an sm_100a tile variant by its N extent
// (256 / 128 / 64).  All variants give identical bits.
const char* const kNames[15] = {"128x256x32 w64x64 s3", "256x128x32 w64x64 s3", "128x128x32 w64x64 s4",
                                "128x256x32 w64x64 s4", "128x256x32 w64x64 s2", "192x128x32 w48x64 s3",
                                "192x128x32 w48x64 s4", "64x256x32 w64x64 s4",  "64x256x32 w32x64 s4",
                                "128x128x32 w64x64 s3", "128x128x32 w64x32 s4", "256x128x32 w64x64 s4",
                                "256x64x32 w64x64 s4",  "128x64x32 w64x64 s4",  "64x128x32 w64x64 s4"};
const int kTileN[15] = {256, 128, 128, 256, 256, 128, 128, 256, 256, 128, 128, 128, 64, 64, 128};
}  // namespace

REAX_API int reax_gemm_ncfg() { return 15; }
REAX_API const char* reax_gemm_cfgname(int c) { return (c >= 0 && c < 15) ? kNames[c] : "?"; }

// X [M, K] (ld K), W [N, K] (ld K), D [M, N] with leading dimension ldd; fp32 accumulation, bf16 output.
// Not implementable (1): K, ldd not multiples of 8 or operands not 16-byte aligned (the reference's alignment-8
// CUTLASS kernels reject the same cases).
REAX_API int reax_gemm(int cfg, const void* x, const void* w, void* d, int M, int N, int K, int ldd, void* stream) {
  if (cfg < 0 || cfg >= 15) return 9;
  if (M < 0 || N < 0 || K < 0 || K % 8 || ldd % 8 || ldd < N) return 1;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(d)) & 15) return 1;
  cudaStream_t st = (cudaStream_t)stream;
  if (M == 0 || N == 0) return 0;
  if (K == 0)
    return cudaMemset2DAsync(d, (size_t)ldd * 2, 0, (size_t)N * 2, (size_t)M, st) == cudaSuccess ? 0 : 4;
  reax_host::GemmProblem pr;
  pr.a = x;
  pr.b = w;
  pr.out = d;
  pr.M = M;
  pr.Nacc = N;
  pr.K = K;
  pr.Kseg = K;
  pr.S = 1;
  pr.ld_out = ldd;
  pr.batch_out = 0;
  pr.out_cols = N;
  if (M <= 64) return reax_host::launch_gemm_swapped<reax::EPI_BF16_T>(pr, st, 4);
  switch (kTileN[cfg]) {
    case 256: return reax_host::launch_gemm<256, 4, reax::EPI_BF16>(pr, st, 4);
    case 128: return reax_host::launch_gemm<128, 6, reax::EPI_BF16>(pr, st, 4);
    default: return reax_host::launch_gemm<64, 8, reax::EPI_BF16>(pr, st, 4);
  }
}
