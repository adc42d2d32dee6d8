// The gate table of libreax_howu: silu(z) = z / (1 + expf(-z)) in fp32, with expf and IEEE division (silu_exact),
// for every bf16 bit pattern of z -- the exact value, so a kernel whose gate input is a bf16 number reads it instead of
// computing it.  256 KB of static device memory, filled once per device by gate_table_kernel on the first call that
// needs it.
#pragma once
#include "common.cuh"

namespace reax {
__device__ float g_gate_tab[65536];
__global__ void gate_table_kernel(float* tab) {
  const unsigned int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 65536u) tab[i] = silu_exact(__uint_as_float(i << 16));
}
}  // namespace reax

namespace reax_host {
// The table's device address on the current device, filling it on the first call there (a kernel on `st`, waited for,
// so launches on every stream see a complete table; the first call on a device is not one to capture in a CUDA
// graph).  nullptr on a CUDA error.
inline const float* gate_table(cudaStream_t st) {
  static std::mutex mu;
  static std::map<int, const float*> ready;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  auto it = ready.find(dev);
  if (it != ready.end()) return it->second;
  void* tab = nullptr;
  if (cudaGetSymbolAddress(&tab, reax::g_gate_tab) != cudaSuccess) return nullptr;
  reax::gate_table_kernel<<<256, 256, 0, st>>>(static_cast<float*>(tab));
  if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess) return nullptr;
  ready[dev] = static_cast<const float*>(tab);
  return static_cast<const float*>(tab);
}
}  // namespace reax_host
