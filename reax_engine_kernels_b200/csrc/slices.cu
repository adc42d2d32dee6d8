// libreax_slices.so -- split-K partials as one batched GEMM, sm_100a (tcgen05 + TMA).
// ABI: libreax_slices/gemm_slices_v2.cu:55-84 (reax_slices_ncfg, reax_slices_cfgname, reax_slices).
//
// Slice s reads columns [s*kps, (s+1)*kps) of X and W through a 3-D tensor map (kps, S, rows) whose innermost
// extent is kps, so a K tile that runs past the end of a slice is zero-filled by the copy engine instead of
// reading the next slice.  Every configuration index runs the same K-reduction order, so all 16 indices give
// bitwise identical partials.
#include "gemm_sm100.cuh"

REAX_DEFINE_STATUS_EXPORT()

namespace {
// The SLICE_CFGS table (libreax_slices/gemm_slices_v2.cu:37-53): names kept verbatim as ABI data.  The tile N of
// each entry selects the sm_100a variant (256 / 128 / 64 columns per tcgen05 tile).
const char* const kNames[16] = {"128x256x32 w64x64 s3", "256x128x32 w64x64 s3", "128x128x32 w64x64 s4",
                                "64x256x32 w64x64 s4",  "128x128x32 w64x64 s3", "256x128x32 w64x64 s4",
                                "128x256x32 w64x64 s4", "64x128x32 w64x64 s4",  "128x64x32 w64x64 s4",
                                "64x256x32 w64x64 s3",  "64x128x32 w32x64 s4",  "256x64x32 w64x64 s3",
                                "128x128x32 w64x64 s5", "128x128x32 w64x64 s6", "64x128x32 w32x64 s6",
                                "256x128x32 w64x64 s5"};
const int kTileN[16] = {256, 128, 128, 256, 128, 128, 256, 128, 64, 256, 128, 64, 128, 128, 128, 128};

template <int KIND>
int run(int tn, const reax_host::GemmProblem& pr, cudaStream_t st) {
  switch (tn) {
    case 256: return reax_host::launch_gemm<256, 4, KIND>(pr, st, 4);
    case 128: return reax_host::launch_gemm<128, 6, KIND>(pr, st, 4);
    default: return reax_host::launch_gemm<64, 8, KIND>(pr, st, 4);
  }
}
}  // namespace

REAX_API int reax_slices_ncfg() { return 16; }
REAX_API const char* reax_slices_cfgname(int c) { return (c >= 0 && c < 16) ? kNames[c] : "?"; }

// P[s] = X[:, s*kps:(s+1)*kps] @ W[:, s*kps:(s+1)*kps]^T, P[s] at p + s*M*N (ld N), fp32 or bf16.
// Not implementable (1): K or kps not multiples of 8, S*kps > K, operands not 16-byte aligned.
REAX_API int reax_slices(int cfg, int part_fp32, const void* x, const void* w, void* p, int M, int N, int kps, int S,
                           int K, void* stream) {
  if (cfg < 0 || cfg >= 16) return 9;
  if (M < 0 || N < 0 || K < 0 || kps < 0 || S < 0) return 1;
  if (K % 8 || kps % 8 || (long long)S * kps > K) return 1;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(p)) & 15) return 1;
  cudaStream_t st = (cudaStream_t)stream;
  if (M == 0 || N == 0 || S == 0) return 0;
  const size_t esz = part_fp32 ? 4 : 2;
  if (kps == 0)
    return cudaMemsetAsync(p, 0, (size_t)S * M * N * esz, st) == cudaSuccess ? 0 : 4;
  reax_host::GemmProblem pr;
  pr.a = x;
  pr.b = w;
  pr.out = p;
  pr.M = M;
  pr.Nacc = N;
  pr.K = K;
  pr.Kseg = kps;
  pr.S = S;
  pr.ld_out = N;
  pr.batch_out = (long long)M * N;
  pr.out_cols = N;
  if (M <= 64)
    return part_fp32 ? reax_host::launch_gemm_swapped<reax::EPI_F32_T>(pr, st, 4)
                     : reax_host::launch_gemm_swapped<reax::EPI_BF16_T>(pr, st, 4);
  return part_fp32 ? run<reax::EPI_F32>(kTileN[cfg], pr, st) : run<reax::EPI_BF16>(kTileN[cfg], pr, st);
}
