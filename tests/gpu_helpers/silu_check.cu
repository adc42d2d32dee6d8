// Test helper: the delta-rule norm's gate silu_gate (Markstein quotient) against silu_exact (expf + IEEE division) for
// every bf16 bit pattern.  Built by tests/test_silu_gpu.py from the package's own header.
#include "howu_tc.cuh"

// one thread per bf16 pattern: mismatches (fp32 bit patterns differ, NaN == NaN) counted in *bad, the first recorded
__global__ void silu_check_kernel(unsigned int* bad, unsigned int* first) {
  const unsigned int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 65536u) return;
  const float z = __uint_as_float(i << 16);
  const float a = reax::silu_gate(z), b = reax::silu_exact(z);
  const bool same = __float_as_uint(a) == __float_as_uint(b) || (a != a && b != b);
  if (!same) {
    if (atomicAdd(bad, 1u) == 0u) *first = i;
  }
}

extern "C" int run_silu_check(unsigned int* host_out) {
  unsigned int* d = nullptr;
  if (cudaMalloc(&d, 2 * sizeof(unsigned int)) != cudaSuccess) return -1;
  cudaMemset(d, 0, 2 * sizeof(unsigned int));
  silu_check_kernel<<<256, 256>>>(d, d + 1);
  const cudaError_t e = cudaMemcpy(host_out, d, 2 * sizeof(unsigned int), cudaMemcpyDeviceToHost);
  cudaFree(d);
  return e == cudaSuccess ? 0 : (int)e;
}
