// fake_cudart.cpp — TEST INFRASTRUCTURE. Host-memory stand-ins for the CUDA
// runtime calls that the reference's tests/kernel_tests.cu makes (through
// DeviceBuffer, upload and download: include/cuda_utils.h:19-63,
// tests/kernel_tests.cu:25-34), so that the reference's own check harness runs
// on a machine without a GPU with its launch_* calls served by the CPU oracle
// (launch_on_oracle.cpp). "Device" pointers are plain host allocations.
#include <cuda_runtime_api.h>

#include <cstdlib>
#include <cstring>

extern "C" {

cudaError_t cudaMalloc(void** ptr, size_t size) {
  *ptr = std::malloc(size ? size : 1);
  return *ptr ? cudaSuccess : cudaErrorMemoryAllocation;
}

cudaError_t cudaFree(void* ptr) {
  std::free(ptr);
  return cudaSuccess;
}

cudaError_t cudaMemcpy(void* dst, const void* src, size_t count, enum cudaMemcpyKind) {
  std::memmove(dst, src, count);
  return cudaSuccess;
}

cudaError_t cudaMemset(void* dst, int value, size_t count) {
  std::memset(dst, value, count);
  return cudaSuccess;
}

cudaError_t cudaDeviceSynchronize(void) { return cudaSuccess; }

cudaError_t cudaGetLastError(void) { return cudaSuccess; }

const char* cudaGetErrorString(cudaError_t) { return "host stand-in"; }

}  // extern "C"
