// libreax_gv.so -- gate/up GEMM with the fused SiLU*mul epilogue, sm_100a (tcgen05 + TMA).
// ABI: libreax_gv/gateup_vis2.cu:171-208 (reax_gv_ncfg, reax_gv_cfgname, reax_gv).
#include "gemm_sm100.cuh"

REAX_DEFINE_STATUS_EXPORT()

namespace {
// Configuration names are part of the ABI (the engine records and selects configs by index and name); the
// table is kept verbatim.  In this build every index selects an sm_100a tile variant by its N extent:
// N >= 192 -> 128x256 tcgen05 tiles (4-stage ring), otherwise 128x128 tiles (6-stage ring).  All variants give
// identical bits (the K-reduction order never depends on the tile).
const char* const kNames[20] = {"128x256x32 w64x64 s3",     "256x128x32 w64x64 s3",     "128x128x32 w64x64 s4",
                                "128x256x32 w64x64 s4",     "128x256x64 w64x64x64 s2",  "256x128x64 w64x64x64 s2",
                                "128x128x64 w64x64x64 s3",  "128x128x64 w64x64x64 s2",  "64x256x64 w64x64x64 s2",
                                "128x256x32 w64x64 s2",     "128x192x32 w64x48 s3",     "128x192x32 w64x48 s4",
                                "192x128x32 w48x64 s3",     "192x128x32 w48x64 s4",     "64x256x32 w64x64 s4",
                                "64x256x32 w32x64 s4",      "192x192x32 w96x48 s3",     "128x128x32 w64x64 s3",
                                "128x128x32 w64x32 s4",     "256x128x32 w64x64 s4"};
const int kTileN[20] = {256, 128, 128, 256, 256, 128, 128, 128, 256, 256, 192, 192, 128, 128, 256, 256, 192, 128, 128, 128};
}  // namespace

// bf16(silu(g)) for every bf16 bit pattern of the gate g, as the epilogue computes it (expf and IEEE division,
// silu_exact); filled once per device by silu_table_kernel.  128 KB of device memory per GPU that loads the library.
__device__ uint16_t g_silu_tab[65536];

__global__ void silu_table_kernel(uint16_t* tab) {
  const unsigned int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 65536u) tab[i] = __bfloat16_as_ushort(__float2bfloat16_rn(reax::silu_exact(__uint_as_float(i << 16))));
}

// The table's device address on the current device, filling it on the first call there: the fill runs on `st` and
// the call waits for it, so every later launch on any stream sees a complete table (the first call on a device is
// therefore not one to capture in a CUDA graph).  nullptr on a CUDA error.
static const uint16_t* silu_table(cudaStream_t st) {
  static std::mutex mu;
  static std::map<int, const uint16_t*> ready;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  auto it = ready.find(dev);
  if (it != ready.end()) return it->second;
  void* tab = nullptr;
  if (cudaGetSymbolAddress(&tab, g_silu_tab) != cudaSuccess) return nullptr;
  silu_table_kernel<<<256, 256, 0, st>>>(static_cast<uint16_t*>(tab));
  if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess) return nullptr;
  ready[dev] = static_cast<const uint16_t*>(tab);
  return static_cast<const uint16_t*>(tab);
}

REAX_API int reax_gv_ncfg() { return 20; }
REAX_API const char* reax_gv_cfgname(int c) { return (c >= 0 && c < 20) ? kNames[c] : "?"; }

// x [M, K] row-major, w_g4 [2*N2, K] row-major (gate/up rows interleaved in groups of 4), out [M, N2] row-major
REAX_API int reax_gv(int cfg, const void* x, const void* w, void* out, int M, int N2, int K, void* stream) {
  if (cfg < 0 || cfg >= 20) return 9;
  if (K % 8 || N2 % 4) return 1;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) return 1;
  cudaStream_t st = (cudaStream_t)stream;
  if (M <= 0 || N2 <= 0) return 0;
  if (K == 0)  // empty reduction: g = u = 0 -> silu(0) * 0 = +0
    return cudaMemsetAsync(out, 0, (size_t)M * (size_t)N2 * 2, st) == cudaSuccess ? 0 : 3;
  reax_host::GemmProblem pr;
  pr.a = x;
  pr.b = w;
  pr.out = out;
  pr.M = M;
  pr.Nacc = 2 * N2;
  pr.K = K;
  pr.Kseg = K;
  pr.S = 1;
  pr.ld_out = N2;
  pr.batch_out = 0;
  pr.out_cols = N2;
  pr.silu_tab = silu_table(st);
  if (pr.silu_tab == nullptr) return 2;
  if (kTileN[cfg] >= 192) return reax_host::launch_gemm<256, 4, reax::EPI_GV>(pr, st, 3);
  return reax_host::launch_gemm<128, 6, reax::EPI_GV>(pr, st, 3);
}
