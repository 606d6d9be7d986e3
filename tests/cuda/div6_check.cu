// Test helper: the writer's division by 6 (nvqsa::div6_rn) against CUDA's IEEE
// division __fdiv_rn(x, 6.0f) for every one of the 2^32 fp32 bit patterns.
// Built with nvcc by tests/test_gpu_writer.py; NaN results compare as NaN.
#include "common.cuh"

namespace {
__global__ void div6_check_kernel(unsigned long long* bad, unsigned int* first) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (1ull << 32); i += stride) {
    const float x = __uint_as_float((uint32_t)i);
    const float a = nvqsa::div6_rn(x);
    const float b = __fdiv_rn(x, 6.0f);
    const bool same = (a != a) ? (b != b) : (__float_as_uint(a) == __float_as_uint(b));
    if (!same) {
      const unsigned long long k = atomicAdd(bad, 1ull);
      if (k < 8) first[k] = (uint32_t)i;
    }
  }
}
}  // namespace

extern "C" int div6_check(unsigned long long* mismatches, unsigned int* first8) {
  unsigned long long* d_bad = nullptr;
  unsigned int* d_first = nullptr;
  if (cudaMalloc(&d_bad, sizeof(unsigned long long)) != cudaSuccess) return 1;
  if (cudaMalloc(&d_first, 8 * sizeof(unsigned int)) != cudaSuccess) return 1;
  cudaMemset(d_bad, 0, sizeof(unsigned long long));
  cudaMemset(d_first, 0xff, 8 * sizeof(unsigned int));
  div6_check_kernel<<<148 * 8, 256>>>(d_bad, d_first);
  int rc = cudaDeviceSynchronize() == cudaSuccess ? 0 : 2;
  cudaMemcpy(mismatches, d_bad, sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  cudaMemcpy(first8, d_first, 8 * sizeof(unsigned int), cudaMemcpyDeviceToHost);
  cudaFree(d_bad);
  cudaFree(d_first);
  return rc;
}
