// Test helper: the bounded mbarrier wait of the package's kernels, run against a barrier nothing ever arrives on.
// Built by tests/test_bounded_wait_gpu.py with a short REAX_WAIT_LIMIT so the wait gives up within milliseconds.
#include "common.cuh"

REAX_DEFINE_STATUS_EXPORT()

// One CTA of 64 threads: thread 0 initialises an mbarrier expecting one arrival that never comes; every thread waits
// on it with the warp-uniform bounded wait.  result[0] = number of threads whose wait returned false (all 64 when the
// limit works), result[1] = 1 if the shared abort flag was raised.
__global__ void stuck_wait_kernel(int* result) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    reax::mbar_init(reax::smem_u32(&bar), 1);
    abort_flag = 0;
    reax::fence_mbar_init();
  }
  __syncthreads();
  const bool ok = reax::mbar_wait_warp(reax::smem_u32(&bar), 0, &abort_flag, reax::ST_TIMEOUT_ATTN);
  if (!ok) atomicAdd(&result[0], 1);
  __syncthreads();
  if (threadIdx.x == 0) result[1] = abort_flag;
}

// an ordinary kernel afterwards: the context must still work
__global__ void add_one_kernel(int* x) { x[threadIdx.x] += 1; }

extern "C" int run_stuck_wait(int* host_result) {
  int* d = nullptr;
  if (cudaMalloc(&d, 2 * sizeof(int)) != cudaSuccess) return -1;
  cudaMemset(d, 0, 2 * sizeof(int));
  stuck_wait_kernel<<<1, 64>>>(d);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(host_result, d, 2 * sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(d);
  return (int)e;
}

extern "C" int run_after(int* host_value) {
  int* d = nullptr;
  if (cudaMalloc(&d, 32 * sizeof(int)) != cudaSuccess) return -1;
  cudaMemset(d, 0, 32 * sizeof(int));
  add_one_kernel<<<1, 32>>>(d);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(host_value, d, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(d);
  return (int)e;
}
