// Host-to-device staging of a decode step's inputs by SM loads from mapped
// pinned host memory. A decode step's per-step inputs (queries, block table,
// lengths: ~132 KB at batch 8 x 32 heads x d128) are too small for the copy
// engine: on B200 a 135 KB pinned host-to-device cudaMemcpyAsync followed by
// a kernel measured 17.1 us between CUDA events, against 12.3 us for this
// kernel followed by the same kernel (an empty kernel alone: 5.5 us). Here
// every thread of a small grid reads 16-byte pieces of the host buffer over
// PCIe (all pieces in flight at once) and stores them to device memory.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/int4kv_b200.h"

namespace {

constexpr int kStageThreads = 128;
constexpr int kStageUnroll = 4;        // 16-byte pieces in flight per thread per iteration
constexpr long long kStageMaxBlocks = 1184;  // 8 per SM on a 148-SM B200; larger copies loop

// dst[i] = src[i] for i < n16 (16-byte pieces). The loads bypass every cache
// level (ld.global.cv): the host rewrites the buffer between calls, and a
// line of host memory cached on the device by an earlier call would be stale.
__global__ void __launch_bounds__(kStageThreads)
stage_host_kernel(uint4* __restrict__ dst, const uint4* src, long long n16) {
  // a kernel launched after this one with programmatic stream serialization
  // (the paged decode) may be dispatched at once; it waits for this grid's
  // completion before it reads anything
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n16;
       i += stride * kStageUnroll) {
    uint4 v[kStageUnroll];
#pragma unroll
    for (int j = 0; j < kStageUnroll; ++j) {
      const long long x = i + j * stride;
      if (x < n16) v[j] = __ldcv(src + x);
    }
#pragma unroll
    for (int j = 0; j < kStageUnroll; ++j) {
      const long long x = i + j * stride;
      if (x < n16) dst[x] = v[j];
    }
  }
}

}  // namespace

extern "C" cudaError_t int4kv_stage_inputs(void* dst, const void* src, size_t bytes,
                                           cudaStream_t stream) {
  if (!dst || !src || bytes == 0 || bytes % 16 != 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u)
    return cudaErrorInvalidValue;
  const long long n16 = (long long)(bytes / 16);
  long long blocks = (n16 + kStageThreads - 1) / kStageThreads;
  if (blocks > kStageMaxBlocks) blocks = kStageMaxBlocks;
  stage_host_kernel<<<(unsigned)blocks, kStageThreads, 0, stream>>>(
      static_cast<uint4*>(dst), static_cast<const uint4*>(src), n16);
  return cudaGetLastError();
}
