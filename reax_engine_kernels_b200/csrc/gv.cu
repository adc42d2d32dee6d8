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

// ------------------------------------------------------------------------------------------------
// reax_gv_noalloc: reax_gv for callers that cannot allocate device memory
// ------------------------------------------------------------------------------------------------
// reax_gv allocates, on its first split launches on a device, the scratch memory that the split-last-waves kernel
// passes partial accumulators through (cudaMalloc; a pool of up to four 18.9 MB blocks per device).  Some callers cannot let a library do that: an inference engine
// that reserves all of the GPU's memory up front for its own arena (weights, KV cache) and hands out nothing else,
// or a serving loop for which a cudaMalloc -- which may wait for the whole device -- in the middle of a step is not
// acceptable.  This entry point computes exactly what reax_gv computes (same kernels, same bits) with that scratch
// in the static array below instead, which is part of the library's image: every GPU that loads libreax_gv holds it
// (about 20 MiB) until the process exits.  It allocates nothing: no cudaMalloc, cudaFree or allocating routine.
//
// Limits and sharing:
//   * The array holds partial accumulators for up to kNoAllocMaxCtas CTAs, i.e. GPUs with at most 160 SMs (a B200
//     has 148); on a GPU with more SMs the call returns 5 and launches nothing.  Problem sizes are not limited by it.
//   * Every call, on every stream, uses the same array.  Calls that overlap on the GPU (launched on different
//     streams without ordering between them) race on it and may produce wrong results; order them on one stream or
//     with events.
//   * The array keeps the last call's contents.  Nothing in it has to start at zero: each call tags its hand-over
//     flags with a new epoch, so a flag left by an earlier call never matches, and every partial slot is written by
//     its call before it is read.
//   * The first call on each device does the set-up with that device current: it looks up the array's device
//     address (cudaGetSymbolAddress -- in host code the array's name is only a stand-in) and fills the SiLU table,
//     waiting on `stream` for the fill.  Make that first call before any stream capture.
constexpr int kNoAllocMaxCtas = 160;
constexpr size_t kNoAllocFlagBytes =
    ((size_t)reax::kSplitFlagsPerCta * kNoAllocMaxCtas * sizeof(unsigned int) + 255) & ~(size_t)255;
constexpr size_t kNoAllocScratchBytes =
    kNoAllocFlagBytes + (size_t)kNoAllocMaxCtas * 128 * reax::kSplitSlotCols * sizeof(float);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// per device: the array's device address and the epoch of the last call
static bool noalloc_scratch(int dev, reax_host::SplitScratch& out) {
  struct Dev {
    unsigned char* base = nullptr;
    unsigned int epoch = 0;
  };
  static std::mutex mu;
  static std::map<int, Dev> devs;
  std::lock_guard<std::mutex> lk(mu);
  Dev& d = devs[dev];
  if (d.base == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      devs.erase(dev);
      return false;
    }
    d.base = static_cast<unsigned char*>(p);
  }
  if (++d.epoch == 0) d.epoch = 1;
  out.flag = reinterpret_cast<unsigned int*>(d.base);
  out.part = reinterpret_cast<float*>(d.base + kNoAllocFlagBytes);
  out.epoch = d.epoch;
  return true;
}

REAX_API int reax_gv_noalloc(int cfg, const void* x, const void* w, void* out, int M, int N2, int K, void* stream) {
  if (cfg < 0 || cfg >= 20) return 9;
  if (K % 8 || N2 % 4) return 1;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) return 1;
  cudaStream_t st = (cudaStream_t)stream;
  if (M <= 0 || N2 <= 0) return 0;
  if (K == 0)  // empty reduction: g = u = 0 -> silu(0) * 0 = +0
    return cudaMemsetAsync(out, 0, (size_t)M * (size_t)N2 * 2, st) == cudaSuccess ? 0 : 3;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 2;
  if (reax_host::device_sms(dev) > kNoAllocMaxCtas) return 5;  // more CTAs than the static scratch has slots for
  reax_host::SplitScratch sc;
  if (!noalloc_scratch(dev, sc)) return 2;
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
  if (kTileN[cfg] >= 192) return reax_host::launch_gemm<256, 4, reax::EPI_GV>(pr, st, 3, &sc);
  return reax_host::launch_gemm<128, 6, reax::EPI_GV>(pr, st, 3, &sc);
}
