// staging.cu — stream-ordered copies between page-locked host memory and
// device memory by an SM kernel, for callers that feed the decode entry points
// from host buffers (the end-to-end path: query rows in, attention rows out).
//
// The reference moves the query in and the output out around its CUDA
// attention call with synchronous cudaMemcpy (swamp-gpu/kernels/
// fused_attention.cu:313-330, gpu_alloc_and_copy_q / gpu_copy_output_to_host)
// and copies mapped host-visible buffers on its Vulkan path
// (swamp-gpu/src/lib.rs:149-157, upload / download).
// On B200 the same transfers run as kernels reading or writing mapped
// page-locked memory over PCIe: 16-byte loads, one per thread, grid-strided.
// In a CUDA graph they are kernel nodes; for the 22-layer batched decode with
// a copy in and a copy out around every layer this measured 1150 us per step
// against 1211 us with copy-engine copies on the same streams.
#include <stdint.h>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace staging {

constexpr int THREADS = 256;
constexpr int64_t MAX_CTAS = 296;

__global__ void __launch_bounds__(THREADS) copy16_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                         int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)THREADS + threadIdx.x; i < n; i += (int64_t)gridDim.x * THREADS)
    dst[i] = src[i];
}

__global__ void __launch_bounds__(THREADS) copy1_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                        int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)THREADS + threadIdx.x; i < n; i += (int64_t)gridDim.x * THREADS)
    dst[i] = src[i];
}

int64_t grid_for(int64_t n) {
  const int64_t g = (n + THREADS - 1) / THREADS;
  return g < MAX_CTAS ? g : MAX_CTAS;
}

}  // namespace staging
}  // namespace nyion

using namespace nyion;
using namespace nyion::staging;

extern "C" int32_t nyion_attn_host_map(const void* host, void** device_ptr) {
  if (!host || !device_ptr) return fail(NYION_ERR_INVALID, "host_map: null pointer argument");
  *device_ptr = nullptr;
  void* d = nullptr;
  const cudaError_t e = cudaHostGetDevicePointer(&d, const_cast<void*>(host), 0);
  if (e != cudaSuccess) {
    cudaGetLastError();   // not sticky: clear it so a later launch check does not report it
    return check_cuda(e, "host_map: cudaHostGetDevicePointer (memory not page-locked?)");
  }
  *device_ptr = d;
  return NYION_OK;
}

extern "C" int32_t nyion_attn_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return NYION_OK;
  if (!dst || !src) return fail(NYION_ERR_INVALID, "copy_async: null pointer argument");
  const uintptr_t a = reinterpret_cast<uintptr_t>(dst), b = reinterpret_cast<uintptr_t>(src);
  if (a < b + bytes && b < a + bytes) return fail(NYION_ERR_INVALID, "copy_async: overlapping ranges");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n16 = ((a | b) & 15) == 0 ? (int64_t)(bytes / 16) : 0;
  if (n16 > 0) {
    copy16_kernel<<<(unsigned)grid_for(n16), THREADS, 0, s>>>(static_cast<const uint4*>(src),
                                                              static_cast<uint4*>(dst), n16);
    const int32_t st = check_cuda(cudaGetLastError(), "copy_async launch");
    if (st) return st;
  }
  const int64_t done = n16 * 16, rest = (int64_t)bytes - done;
  if (rest > 0) {
    copy1_kernel<<<(unsigned)grid_for(rest), THREADS, 0, s>>>(static_cast<const uint8_t*>(src) + done,
                                                              static_cast<uint8_t*>(dst) + done, rest);
    return check_cuda(cudaGetLastError(), "copy_async launch");
  }
  return NYION_OK;
}
