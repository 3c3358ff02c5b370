// Generic INT4 flash-decode over ONE shared page stream (the reference's
// cu_flash_decode_int4 contract, csrc/flash_decode_int4.cu:104-284):
// every query of [batch, heads] attends to the same list of pages, each page
// [block_size, head_dim] with one code per byte, its own per-channel
// scale/zp and a valid-row count. Any head_dim in [1, 256], any page size.
//
// B200 mapping (CUDA cores):
//   * A CTA serves a tile of QT queries, so every key/value byte it reads feeds
//     QT dot products (the shared-stream case is all-queries-one-stream).
//   * Logits: one thread per key row, QT dot products in float64 as
//     sum_d (q_d*s_d)*c_d - sum_d q_d*zp_d*s_d (exact dequantization, the
//     reference's float64 arbiter); no cross-lane reduction per token.
//   * Softmax: per-warp online state over 32-row tiles; P.V with lanes over
//     head_dim (coalesced value rows).
//   * Split-KV: the page list can be cut into `splits` contiguous ranges, one
//     CTA each, merged by a combine kernel. The drop-in entry point has no
//     workspace argument and runs with one split.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "../../include/int4kv_b200.h"

using namespace i4kv;

namespace {

constexpr int kQT = 4;        // queries per CTA
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxD = 256;
constexpr int kDPL = kMaxD / 32;
constexpr uint32_t kFull = 0xffffffffu;

struct DenseArgs {
  const float* q;
  const uint8_t* kq;
  const float* ks;
  const float* kz;
  const void* v;
  const int* lens;
  int nq, D, nb, bs, splits;
  float* out;       // final output (splits == 1)
  char* ws;         // partial records (splits > 1)
  const int* ids;   // nullable: page pg of the stream is block ids[pg] of the storage
  int num_blocks;   // storage blocks (ids outside [0, num_blocks) are skipped)
};

// Code of dim d in a key row: one code per byte, or two per byte (low
// nibble = even dim) in the packed storage of the vLLM-style block cache.
template <bool PACKED>
__device__ __forceinline__ double key_code(const uint8_t* krow, int d) {
  if constexpr (PACKED) {
    return (double)((krow[d >> 1] >> ((d & 1) << 2)) & 15);
  } else {
    return (double)krow[d];
  }
}

template <int VK>
__device__ __forceinline__ float value_at(const void* vrow, int d) {
  if constexpr (VK == 0) {
    return static_cast<const float*>(vrow)[d];
  } else if constexpr (VK == 1) {
    return __half2float(static_cast<const __half*>(vrow)[d]);
  } else {
    return __bfloat162float(static_cast<const __nv_bfloat16*>(vrow)[d]);
  }
}

// Partial record: [m f64][l f32][pad][acc D f32], padded to a multiple of 16
// bytes so every record (and its double) stays aligned for any head_dim.
__host__ __device__ inline size_t dense_rec_bytes(int D) { return 16 + 16 * (((size_t)D + 3) / 4); }

template <bool PACKED, int VK>
__global__ void __launch_bounds__(kThreads)
dense_decode_kernel(DenseArgs a) {
  __shared__ float s_q[kQT][kMaxD];
  __shared__ double s_qs[kQT][kMaxD];   // q_d * s_d of the current page (exact)
  __shared__ double s_bias[kQT];        // sum_d q_d * zp_d * s_d of the current page
  __shared__ double s_m[kWarps][kQT];
  __shared__ float s_l[kWarps][kQT];
  __shared__ float s_acc[kWarps][kQT][kMaxD];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q0 = blockIdx.x * kQT;
  const int nqt = min(kQT, a.nq - q0);
  const int D = a.D;
  const int split = blockIdx.y;
  const int pb = (int)((long long)split * a.nb / a.splits);
  const int pe = (int)((long long)(split + 1) * a.nb / a.splits);

  for (int i = threadIdx.x; i < kQT * D; i += kThreads) {
    const int qi = i / D, d = i - qi * D;
    s_q[qi][d] = qi < nqt ? a.q[(size_t)(q0 + qi) * D + d] : 0.f;
  }

  double m_w[kQT];
  float l_lane[kQT];
  float acc[kQT][kDPL];
#pragma unroll
  for (int qi = 0; qi < kQT; ++qi) {
    m_w[qi] = -INFINITY;
    l_lane[qi] = 0.f;
#pragma unroll
    for (int k = 0; k < kDPL; ++k) acc[qi][k] = 0.f;
  }

  const int row_bytes = PACKED ? (D + 1) / 2 : D;
  constexpr int VB = VK == 0 ? 4 : 2;
  for (int pi = pb; pi < pe; ++pi) {
    const int pg = a.ids ? a.ids[pi] : pi;  // storage block of the stream's page pi
    if (pg < 0 || pg >= a.num_blocks) continue;  // uniform across the CTA
    __syncthreads();  // previous page's folded constants no longer in use
    for (int i = threadIdx.x; i < kQT * D; i += kThreads) {
      const int qi = i / D, d = i - qi * D;
      s_qs[qi][d] = (double)s_q[qi][d] * (double)a.ks[(size_t)pg * D + d];
    }
    if (warp < kQT) {  // warp qi reduces sum_d q_d * zp_d * s_d for query qi
      double b = 0.0;
      for (int d = lane; d < D; d += 32)
        b = fma((double)s_q[warp][d],
                (double)a.kz[(size_t)pg * D + d] * (double)a.ks[(size_t)pg * D + d], b);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) b += __shfl_xor_sync(kFull, b, o);
      if (lane == 0) s_bias[warp] = b;
    }
    __syncthreads();
    const int blen = min(max(a.lens[pg], 0), a.bs);  // defence in depth, as the reference
    const uint8_t* kpage = a.kq + (size_t)pg * a.bs * row_bytes;
    const char* vpage = static_cast<const char*>(a.v) + (size_t)pg * a.bs * D * VB;
    for (int r0 = warp * 32; r0 < blen; r0 += kThreads) {
      const int r = r0 + lane;
      const bool valid = r < blen;
      double lg[kQT];
#pragma unroll
      for (int qi = 0; qi < kQT; ++qi) lg[qi] = 0.0;
      if (valid) {
        const uint8_t* krow = kpage + (size_t)r * row_bytes;
        for (int d = 0; d < D; ++d) {
          const double code = key_code<PACKED>(krow, d);
#pragma unroll
          for (int qi = 0; qi < kQT; ++qi) lg[qi] = fma(s_qs[qi][d], code, lg[qi]);
        }
#pragma unroll
        for (int qi = 0; qi < kQT; ++qi) lg[qi] -= s_bias[qi];
      }
      const int nrow = min(32, blen - r0);
#pragma unroll
      for (int qi = 0; qi < kQT; ++qi) {
        double l = valid ? lg[qi] : -INFINITY;
        double mx = l;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(kFull, mx, o));
        const double m_new = fmax(m_w[qi], mx);
        const float corr = expf((float)(m_w[qi] - m_new));
        const float p = expf((float)(l - m_new));
        l_lane[qi] = l_lane[qi] * corr + p;
        m_w[qi] = m_new;
#pragma unroll
        for (int k = 0; k < kDPL; ++k) acc[qi][k] *= corr;
        lg[qi] = p;  // reuse as this lane's probability
      }
      for (int j = 0; j < nrow; ++j) {
        const char* vrow = vpage + (size_t)(r0 + j) * D * VB;
        float pj[kQT];
#pragma unroll
        for (int qi = 0; qi < kQT; ++qi) pj[qi] = __shfl_sync(kFull, (float)lg[qi], j);
#pragma unroll
        for (int k = 0; k < kDPL; ++k) {
          const int d = lane + 32 * k;
          if (d < D) {
            const float vv = value_at<VK>(vrow, d);
#pragma unroll
            for (int qi = 0; qi < kQT; ++qi) acc[qi][k] = fmaf(pj[qi], vv, acc[qi][k]);
          }
        }
      }
    }
  }

  // merge the warps' states
#pragma unroll
  for (int qi = 0; qi < kQT; ++qi) {
    float l = l_lane[qi];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(kFull, l, o);
    if (lane == 0) {
      s_m[warp][qi] = m_w[qi];
      s_l[warp][qi] = l;
    }
#pragma unroll
    for (int k = 0; k < kDPL; ++k) {
      const int d = lane + 32 * k;
      if (d < D) s_acc[warp][qi][d] = acc[qi][k];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nqt * D; i += kThreads) {
    const int qi = i / D, d = i - qi * D;
    double M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmax(M, s_m[w][qi]);
    float L = 0.f, o = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        if (s_m[w][qi] == -INFINITY) continue;
        const float e = expf((float)(s_m[w][qi] - M));
        L = fmaf(s_l[w][qi], e, L);
        o = fmaf(s_acc[w][qi][d], e, o);
      }
    }
    if (a.splits == 1) {
      a.out[(size_t)(q0 + qi) * D + d] = __fdiv_rn(o, fmaxf(L, 1e-10f));
    } else {
      char* rec = a.ws + ((size_t)(q0 + qi) * a.splits + split) * dense_rec_bytes(D);
      if (d == 0) {
        *reinterpret_cast<double*>(rec) = M;
        *reinterpret_cast<float*>(rec + 8) = L;
      }
      reinterpret_cast<float*>(rec + 16)[d] = o;
    }
  }
}

__global__ void __launch_bounds__(128)
dense_combine_kernel(const char* __restrict__ ws, int nq, int D, int splits, float* __restrict__ out) {
  const int qi = blockIdx.x;
  if (qi >= nq) return;
  const size_t rb = dense_rec_bytes(D);
  const char* base = ws + (size_t)qi * splits * rb;
  double M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmax(M, *reinterpret_cast<const double*>(base + s * rb));
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.f, o = 0.f;
    if (M != -INFINITY) {
      for (int s = 0; s < splits; ++s) {
        const char* rec = base + s * rb;
        const double m = *reinterpret_cast<const double*>(rec);
        if (m == -INFINITY) continue;
        const float e = expf((float)(m - M));
        L = fmaf(*reinterpret_cast<const float*>(rec + 8), e, L);
        o = fmaf(reinterpret_cast<const float*>(rec + 16)[d], e, o);
      }
    }
    out[(size_t)qi * D + d] = __fdiv_rn(o, fmaxf(L, 1e-10f));
  }
}

int choose_splits(int nq, int nb) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = (nq + kQT - 1) / kQT;
  int splits = (2 * sms + tiles - 1) / tiles;
  if (splits > nb) splits = nb;
  if (splits > 64) splits = 64;
  return splits < 1 ? 1 : splits;
}

cudaError_t check(const float* query, const uint8_t* k_q, const float* k_scale, const float* k_zp,
                  const float* value, const int* block_lens, int batch_size, int num_heads,
                  int head_dim, int num_blocks, int block_size, const float* output) {
  if (head_dim <= 0 || head_dim > kMaxD) return cudaErrorInvalidValue;
  if (batch_size <= 0 || num_heads <= 0 || num_blocks < 0 || block_size < 0) return cudaErrorInvalidValue;
  if ((long long)batch_size * num_heads >= (1LL << 31) / kMaxD) return cudaErrorInvalidValue;
  if (!query || !output) return cudaErrorInvalidValue;
  if (num_blocks > 0 && (!k_q || !k_scale || !k_zp || !value || !block_lens)) return cudaErrorInvalidValue;
  return cudaSuccess;
}

}  // namespace

extern "C" {

cudaError_t cu_flash_decode_int4(const float* query, const uint8_t* k_q, const float* k_scale,
                                 const float* k_zp, const float* value, const int* block_lens,
                                 int batch_size, int num_heads, int head_dim, int num_blocks,
                                 int block_size, float* output, cudaStream_t stream) {
  cudaError_t e = check(query, k_q, k_scale, k_zp, value, block_lens, batch_size, num_heads,
                        head_dim, num_blocks, block_size, output);
  if (e != cudaSuccess) return e;
  const int nq = batch_size * num_heads;
  DenseArgs a{query, k_q, k_scale, k_zp, value, block_lens, nq, head_dim, num_blocks, block_size,
              1, output, nullptr, nullptr, num_blocks};
  dense_decode_kernel<false, 0><<<dim3((nq + kQT - 1) / kQT, 1), kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t int4kv_dense_decode_workspace_size(int batch_size, int num_heads, int head_dim,
                                               int num_blocks, int block_size, size_t* bytes) {
  if (!bytes || head_dim <= 0 || head_dim > kMaxD || batch_size <= 0 || num_heads <= 0 ||
      num_blocks < 0 || block_size < 0)
    return cudaErrorInvalidValue;
  const int nq = batch_size * num_heads;
  const int splits = choose_splits(nq, num_blocks);
  *bytes = splits > 1 ? (size_t)nq * splits * dense_rec_bytes(head_dim) : 16;
  return cudaSuccess;
}

cudaError_t int4kv_dense_decode(const float* query, const uint8_t* k_q, const float* k_scale,
                                const float* k_zp, const float* value, const int* block_lens,
                                int batch_size, int num_heads, int head_dim, int num_blocks,
                                int block_size, float* output, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream) {
  cudaError_t e = check(query, k_q, k_scale, k_zp, value, block_lens, batch_size, num_heads,
                        head_dim, num_blocks, block_size, output);
  if (e != cudaSuccess) return e;
  const int nq = batch_size * num_heads;
  const int splits = choose_splits(nq, num_blocks);
  if (splits > 1) {
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 15u) ||
        workspace_bytes < (size_t)nq * splits * dense_rec_bytes(head_dim))
      return cudaErrorInvalidValue;
  }
  DenseArgs a{query, k_q, k_scale, k_zp, value, block_lens, nq, head_dim, num_blocks, block_size,
              splits, output, static_cast<char*>(workspace), nullptr, num_blocks};
  dense_decode_kernel<false, 0><<<dim3((nq + kQT - 1) / kQT, splits), kThreads, 0, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess || splits == 1) return e;
  dense_combine_kernel<<<nq, 128, 0, stream>>>(static_cast<const char*>(workspace), nq, head_dim,
                                               splits, output);
  return cudaGetLastError();
}

cudaError_t int4kv_block_decode(const float* query, const uint8_t* k_packed, const float* k_scale,
                                const float* k_zp, const void* value, int value_dtype,
                                const int32_t* block_lens, const int32_t* block_ids,
                                int num_listed, int num_blocks, int batch_size, int num_heads,
                                int head_dim, int block_size, float* output, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream) {
  if ((!block_ids && num_listed > 0) || num_blocks < 0) return cudaErrorInvalidValue;
  cudaError_t e = check(query, k_packed, k_scale, k_zp, static_cast<const float*>(value),
                        block_lens, batch_size, num_heads, head_dim, num_listed, block_size,
                        output);
  if (e != cudaSuccess) return e;
  if (value_dtype != INT4KV_VALUES_F32 && value_dtype != INT4KV_VALUES_F16 &&
      value_dtype != INT4KV_VALUES_BF16)
    return cudaErrorInvalidValue;
  const int nq = batch_size * num_heads;
  const int splits = choose_splits(nq, num_listed);
  if (splits > 1) {
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 15u) ||
        workspace_bytes < (size_t)nq * splits * dense_rec_bytes(head_dim))
      return cudaErrorInvalidValue;
  }
  DenseArgs a{query, k_packed, k_scale, k_zp, value, block_lens, nq, head_dim, num_listed,
              block_size, splits, output, static_cast<char*>(workspace), block_ids, num_blocks};
  const dim3 grid((nq + kQT - 1) / kQT, splits);
  switch (value_dtype) {
    case INT4KV_VALUES_F32: dense_decode_kernel<true, 0><<<grid, kThreads, 0, stream>>>(a); break;
    case INT4KV_VALUES_F16: dense_decode_kernel<true, 1><<<grid, kThreads, 0, stream>>>(a); break;
    default: dense_decode_kernel<true, 2><<<grid, kThreads, 0, stream>>>(a); break;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess || splits == 1) return e;
  dense_combine_kernel<<<nq, 128, 0, stream>>>(static_cast<const char*>(workspace), nq, head_dim,
                                               splits, output);
  return cudaGetLastError();
}

const char* int4kv_build_info(void) {
  return "libint4kv_b200: sm_100a, IEEE float32 (no fast-math), built " __DATE__ " " __TIME__;
}

}  // extern "C"
