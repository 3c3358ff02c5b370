// Sequence-split exchange over NVLink peer memory, fused with the merge.
//
// Each rank decodes its token range of one long sequence into per-stream
// partial records (int4kv_paged_decode_partials). This kernel then, per chunk
// of 8 streams (one CTA):
//   1. stores the chunk's records into every rank's exchange buffer (plain
//      stores through CUDA IPC peer mappings, over NVLink),
//   2. raises this rank's flag for the chunk in every rank's buffer (release,
//      system scope),
//   3. waits -- bounded, 2 s of %globaltimer -- for every rank's flag of the
//      same chunk in its own buffer (acquire), and
//   4. merges the chunk's records of all ranks (the reference's warp merge,
//      csrc/flash_decode_int4.cu:199-220, across GPUs) into the output.
// A CTA waits only on the same chunk of other GPUs' kernels, never on another
// CTA of its own GPU. The replacement for the NCCL all-gather + merge kernel.
//
// Exchange buffer (one per rank, zero-filled once, mapped by every rank):
//   step  uint32 [chunks]                  steps completed by this rank's CTA c
//   flag  uint32 [2][kMaxRanks][chunks]    flag[parity][src][c] = step of src
//   recs  record [2][kMaxRanks][streams]   records pushed by src for the step
// Steps alternate between two parities, so a rank can push step E+1 while a
// slower peer still merges step E; it cannot get two steps ahead, because its
// CTA c merges step E+1 only after that peer's CTA c pushed step E+1.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "../../include/int4kv_b200.h"

using namespace i4kv;

namespace {

constexpr int kMaxRanks = INT4KV_EXCHANGE_MAX_RANKS;
constexpr int kChunk = 8;  // streams per CTA (one warp each)
constexpr uint64_t kPeerWaitNs = 2000000000ull;

__host__ __device__ inline size_t align128(size_t x) { return (x + 127) / 128 * 128; }
__host__ __device__ inline int chunks_of(int streams) { return (streams + kChunk - 1) / kChunk; }
__host__ __device__ inline size_t rec_bytes(int d) { return 16 + 4 * (size_t)d; }
__host__ __device__ inline size_t off_flag(int streams) { return align128((size_t)chunks_of(streams) * 4); }
__host__ __device__ inline size_t off_recs(int streams) {
  return off_flag(streams) + align128((size_t)2 * kMaxRanks * chunks_of(streams) * 4);
}
__host__ __device__ inline size_t exchange_bytes(int streams, int d) {
  return off_recs(streams) + (size_t)2 * kMaxRanks * streams * rec_bytes(d);
}

struct Peers {
  char* buf[kMaxRanks];  // rank r's exchange buffer as mapped on this GPU
};

template <int D>
__global__ void __launch_bounds__(kChunk * 32)
exchange_merge_kernel(const char* __restrict__ parts, Peers peers, int world, int rank,
                      int streams, float* __restrict__ out, uint32_t* status) {
  constexpr int DPL = D / 32;
  constexpr int REC = 16 + 4 * D;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x, nchunk = chunks_of(streams);
  char* own = peers.buf[rank];
  uint32_t* step = reinterpret_cast<uint32_t*>(own);
  __shared__ int s_ok;
  const uint32_t E = step[c] + 1u;  // this CTA's step (only CTA c touches step[c])
  const int par = (int)(E & 1u);
  const int s0 = c * kChunk, ns = min(kChunk, streams - s0);

  // 1. push this rank's records of the chunk into every rank's buffer
  const size_t chunk_bytes = (size_t)ns * REC;
  const uint4* src = reinterpret_cast<const uint4*>(parts + (size_t)s0 * REC);
  for (int p = 0; p < world; ++p) {
    uint4* dst = reinterpret_cast<uint4*>(peers.buf[p] + off_recs(streams) +
                                          (((size_t)par * kMaxRanks + rank) * streams + s0) * REC);
    for (size_t i = threadIdx.x; i < chunk_bytes / 16; i += blockDim.x) dst[i] = __ldcg(src + i);
  }
  fence_acq_rel_sys();
  __syncthreads();
  // 2. raise this rank's flag for the chunk everywhere
  if (threadIdx.x < world) {
    uint32_t* f = reinterpret_cast<uint32_t*>(peers.buf[threadIdx.x] + off_flag(streams)) +
                  ((size_t)par * kMaxRanks + rank) * nchunk + c;
    st_release_sys(f, E);
  }
  // 3. wait for every rank's flag of this chunk (bounded)
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < world) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(own + off_flag(streams)) +
                        ((size_t)par * kMaxRanks + threadIdx.x) * nchunk + c;
    bool ok = ld_acquire_sys(f) == E;
    if (!ok) {
      const uint64_t t0 = global_ns();
      while (!(ok = ld_acquire_sys(f) == E)) {
        if (global_ns() - t0 > kPeerWaitNs) break;
        __nanosleep(200);
      }
    }
    if (!ok) atomicAnd(&s_ok, 0);
  }
  __syncthreads();
  const bool ok = s_ok != 0;
  if (threadIdx.x == 0) step[c] = E;
  if (!ok && threadIdx.x == 0 && status) atomicOr(status, kStatusPeerTimeout);
  // 4. merge the chunk's records of all ranks, one warp per stream
  if (warp >= ns) return;
  const int s = s0 + warp;
  float o[DPL];
  if (!ok) {
#pragma unroll
    for (int k = 0; k < DPL; ++k) o[k] = __int_as_float(0x7fc00000);
  } else {
    const char* base = own + off_recs(streams) + ((size_t)par * kMaxRanks * streams + s) * REC;
    const size_t stride = (size_t)streams * REC;
    double M = -INFINITY;
    for (int p = 0; p < world; ++p) M = fmax(M, __ldcg(reinterpret_cast<const double*>(base + p * stride)));
    double L = 0.0, O[DPL];
#pragma unroll
    for (int k = 0; k < DPL; ++k) O[k] = 0.0;
    if (M != -INFINITY) {
      for (int p = 0; p < world; ++p) {
        const char* r = base + p * stride;
        const double m = __ldcg(reinterpret_cast<const double*>(r));
        if (m == -INFINITY) continue;
        const double e = exp(m - M);
        L = fma(__ldcg(reinterpret_cast<const double*>(r + 8)), e, L);
        float v[DPL];
        load_lane_vec_cg<D>(reinterpret_cast<const float*>(r + 16), v, lane);
#pragma unroll
        for (int k = 0; k < DPL; ++k) O[k] = fma((double)v[k], e, O[k]);
      }
    }
    const double den = fmax(L, 1e-10);
#pragma unroll
    for (int k = 0; k < DPL; ++k) o[k] = (float)(O[k] / den);
  }
  store_lane_vec<D>(out + (size_t)s * D, o, lane);
}

}  // namespace

extern "C" {

cudaError_t int4kv_exchange_bytes(int world, int streams, int head_dim, size_t* bytes) {
  if (!bytes || world <= 0 || world > kMaxRanks || streams <= 0) return cudaErrorInvalidValue;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return cudaErrorInvalidValue;
  *bytes = exchange_bytes(streams, head_dim);
  return cudaSuccess;
}

cudaError_t int4kv_exchange_merge(const void* partials, void* const* peer_bufs, int world,
                                  int rank, int streams, int head_dim, float* out,
                                  uint32_t* status, cudaStream_t stream) {
  if (!partials || !peer_bufs || !out || world <= 0 || world > kMaxRanks || rank < 0 ||
      rank >= world || streams <= 0)
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(partials) & 15u) || (reinterpret_cast<uintptr_t>(out) & 15u))
    return cudaErrorInvalidValue;
  Peers peers{};
  for (int r = 0; r < world; ++r) {
    if (!peer_bufs[r] || (reinterpret_cast<uintptr_t>(peer_bufs[r]) & 127u)) return cudaErrorInvalidValue;
    peers.buf[r] = static_cast<char*>(peer_bufs[r]);
  }
  const char* p = static_cast<const char*>(partials);
  const unsigned grid = (unsigned)chunks_of(streams);
  switch (head_dim) {
    case 64: exchange_merge_kernel<64><<<grid, kChunk * 32, 0, stream>>>(p, peers, world, rank, streams, out, status); break;
    case 128: exchange_merge_kernel<128><<<grid, kChunk * 32, 0, stream>>>(p, peers, world, rank, streams, out, status); break;
    case 256: exchange_merge_kernel<256><<<grid, kChunk * 32, 0, stream>>>(p, peers, world, rank, streams, out, status); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t int4kv_exchange_alloc(int device, size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return cudaErrorInvalidValue;
  *ptr = nullptr;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return e;
  void* p = nullptr;
  if ((e = cudaMalloc(&p, bytes)) != cudaSuccess) return e;
  if ((e = cudaMemset(p, 0, bytes)) != cudaSuccess || (e = cudaDeviceSynchronize()) != cudaSuccess) {
    cudaFree(p);
    return e;
  }
  *ptr = p;
  return cudaSuccess;
}

cudaError_t int4kv_exchange_free(void* ptr) { return ptr ? cudaFree(ptr) : cudaSuccess; }

cudaError_t int4kv_ipc_handle(const void* dev_ptr, void* handle) {
  if (!dev_ptr || !handle) return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
  if (e != cudaSuccess) return e;
  static_assert(sizeof(h) == INT4KV_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return cudaSuccess;
}

cudaError_t int4kv_ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

cudaError_t int4kv_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return cudaErrorInvalidValue;
  return cudaIpcCloseMemHandle(dev_ptr);
}

}  // extern "C"
