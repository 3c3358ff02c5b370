// INT4 key quantizers for sm_100a.
//
// Math (bit-exact with the reference's NumPy oracle, src/quantize_int4_ref.py:51-75):
//   per channel over the rows of one group:  mn = min x, mx = max x
//   scale = max(mx - mn, 1e-8) / 15,  zp = -mn / scale
//   q = clip(round_half_even((x - mn) / scale), 0, 15)
// computed with IEEE float32 operations (no fast-math, explicit _rn intrinsics).
//
// Kernels:
//   grouped_quant_kernel  -- kv[N, H*D] in groups of R <= 128 rows, one CTA per
//                            (group, 128-channel slab); every input byte is read
//                            from HBM once and held in registers between the
//                            min/max pass and the quantize pass. Output is either
//                            nibble-packed rows [N, H, D/2] + scale/zp [G, H, D]
//                            (contiguous) or written straight into the paged
//                            cache pools (paged), where the values are scattered
//                            into their pages by the same CTA.
//   grouped_quant_loop_kernel -- same contract for groups longer than 128 rows
//                            (two passes; the second pass re-reads from L2).
//   legacy_quant_kernel   -- the reference's cu_quantize_int4 contract: one group
//                            = all rows, one value per byte. A thread-block cluster
//                            splits the rows; partial min/max meet in distributed
//                            shared memory, so no global scratch is needed.
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "../../include/int4kv_b200.h"

namespace cg = cooperative_groups;
using namespace i4kv;

namespace {

constexpr int kQuantWarps = 8;
constexpr int kQuantThreads = kQuantWarps * 32;
constexpr int kSlab = 128;                    // channels per CTA (32 lanes x 4)
constexpr int kMaxRowsPerWarp = 16;           // 8 warps x 16 rows = 128-row groups
constexpr int kRegGroupMax = kQuantWarps * kMaxRowsPerWarp;

// Where the quantizer writes. Contiguous: packed[n, c/2], scale/zp[g, c].
// Paged: token n of sequence `seq` (absolute position pos0 + n) lands in page
// bt[seq, pos/P] slot pos%P; the group's scale/zp land at the group's first page.
struct OutContig {
  uint8_t* packed;   // [N, C/2]
  float* scale;      // [G, C]
  float* zp;         // [G, C]
};

struct OutPaged {
  const float* v;            // [T, C] values to scatter (may be null)
  const int32_t* tok_off;    // [B+1] row offsets of each sequence in kv / v
  const int32_t* start_pos;  // [B] absolute position of each sequence's first row (nullable)
  const int32_t* block_table;// [B, max_pages]
  int max_pages, page, num_pages, heads, head_dim;
  uint8_t* k_pool;           // [num_pages, H, page, D/2]
  float* v_pool;             // [num_pages, H, page, D]
  float* sz_pool;            // [num_pages, H, 2, D]
  uint32_t* status;          // nullable
};

__device__ __forceinline__ void minmax4(const float4& v, float4& mn, float4& mx) {
  mn.x = fminf(mn.x, v.x); mn.y = fminf(mn.y, v.y); mn.z = fminf(mn.z, v.z); mn.w = fminf(mn.w, v.w);
  mx.x = fmaxf(mx.x, v.x); mx.y = fmaxf(mx.y, v.y); mx.z = fmaxf(mx.z, v.z); mx.w = fmaxf(mx.w, v.w);
}

__device__ __forceinline__ uint16_t pack4(const float4& v, const float4& mn, const float4& sc) {
  const uint32_t a = quant_code(v.x, mn.x, sc.x);
  const uint32_t b = quant_code(v.y, mn.y, sc.y);
  const uint32_t c = quant_code(v.z, mn.z, sc.z);
  const uint32_t d = quant_code(v.w, mn.w, sc.w);
  return static_cast<uint16_t>(a | (b << 4) | (c << 8) | (d << 12));
}

// Cross-warp reduction of per-lane [4-channel] min/max into per-channel
// (min, scale) in shared memory; also emits scale/zp through `emit(ch, s, z)`.
template <class Emit>
__device__ __forceinline__ void reduce_params(float4 mn, float4 mx, float* s_min, float* s_max,
                                              float* s_lo, float* s_sc, int slab_c0, int C,
                                              Emit emit) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  reinterpret_cast<float4*>(s_min)[warp * 32 + lane] = mn;
  reinterpret_cast<float4*>(s_max)[warp * 32 + lane] = mx;
  __syncthreads();
  if (threadIdx.x < kSlab) {
    const int ch = threadIdx.x;
    float lo = s_min[ch], hi = s_max[ch];
#pragma unroll
    for (int w = 1; w < kQuantWarps; ++w) {
      lo = fminf(lo, s_min[w * kSlab + ch]);
      hi = fmaxf(hi, s_max[w * kSlab + ch]);
    }
    float s, z;
    channel_params(lo, hi, &s, &z);
    s_lo[ch] = lo;
    s_sc[ch] = s;
    if (slab_c0 + ch < C) emit(slab_c0 + ch, s, z);
  }
  __syncthreads();
}

template <bool kPaged>
__global__ void __launch_bounds__(kQuantThreads)
grouped_quant_kernel(const float* __restrict__ kv, int N, int C, int R, OutContig oc, OutPaged op) {
  __shared__ __align__(16) float s_min[kQuantWarps * kSlab];
  __shared__ __align__(16) float s_max[kQuantWarps * kSlab];
  __shared__ __align__(16) float s_lo[kSlab];
  __shared__ __align__(16) float s_sc[kSlab];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slab_c0 = blockIdx.x * kSlab;
  const int c0 = slab_c0 + lane * 4;
  const int g = blockIdx.y;
  int seq = 0, row_base = 0, n_rows = N, pos0 = 0;
  if constexpr (kPaged) {
    seq = blockIdx.z;
    row_base = op.tok_off[seq];
    n_rows = op.tok_off[seq + 1] - row_base;
    pos0 = op.start_pos ? op.start_pos[seq] : 0;
    // Groups must start on a group boundary of the sequence, and the launch
    // must cover every row; anything else is malformed metadata.
    const bool bad = pos0 < 0 || (pos0 % R) != 0 || n_rows < 0 || n_rows > N;
    if (bad) {
      if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && op.status)
        atomicOr(op.status, kStatusBadLength);
      return;
    }
  }
  const int r0 = g * R;
  if (r0 >= n_rows) return;
  const int rows = min(R, n_rows - r0);
  const bool lane_ok = c0 < C;

  float4 vals[kMaxRowsPerWarp];
  float4 mn = make_float4(INFINITY, INFINITY, INFINITY, INFINITY);
  float4 mx = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
#pragma unroll
  for (int i = 0; i < kMaxRowsPerWarp; ++i) {
    const int r = warp + i * kQuantWarps;
    if (lane_ok && r < rows) {
      vals[i] = __ldg(reinterpret_cast<const float4*>(kv + (size_t)(row_base + r0 + r) * C + c0));
      minmax4(vals[i], mn, mx);
    }
  }

  if constexpr (!kPaged) {
    reduce_params(mn, mx, s_min, s_max, s_lo, s_sc, slab_c0, C, [&](int ch, float s, float z) {
      oc.scale[(size_t)g * C + ch] = s;
      oc.zp[(size_t)g * C + ch] = z;
    });
  } else {
    const int gpos = pos0 + r0;  // absolute position of the group's first token
    const int gpage = gpos / op.page;
    int slot = (gpage < op.max_pages) ? op.block_table[(size_t)seq * op.max_pages + gpage] : -1;
    if (slot < 0 || slot >= op.num_pages) slot = -1;
    reduce_params(mn, mx, s_min, s_max, s_lo, s_sc, slab_c0, C, [&](int ch, float s, float z) {
      if (slot < 0) return;
      const int h = ch / op.head_dim, d = ch - h * op.head_dim;
      float* dst = op.sz_pool + ((size_t)slot * op.heads + h) * 2 * op.head_dim;
      dst[d] = s;
      dst[op.head_dim + d] = z;
    });
    if (slot < 0 && threadIdx.x == 0 && op.status) atomicOr(op.status, kStatusBadPage);
  }
  if (!lane_ok) return;

  const float4 lo = reinterpret_cast<const float4*>(s_lo)[lane];
  const float4 sc = reinterpret_cast<const float4*>(s_sc)[lane];
#pragma unroll
  for (int i = 0; i < kMaxRowsPerWarp; ++i) {
    const int r = warp + i * kQuantWarps;
    if (r < rows) {
      const uint16_t code = pack4(vals[i], lo, sc);
      if constexpr (!kPaged) {
        *reinterpret_cast<uint16_t*>(oc.packed + ((size_t)(r0 + r) * C + c0) / 2) = code;
      } else {
        const int pos = pos0 + r0 + r;
        const int p = pos / op.page, t = pos - p * op.page;
        const int phys = (p < op.max_pages) ? op.block_table[(size_t)seq * op.max_pages + p] : -1;
        if (phys < 0 || phys >= op.num_pages) {
          if (op.status) atomicOr(op.status, kStatusBadPage);
          continue;
        }
        const int h = c0 / op.head_dim, d = c0 - h * op.head_dim;
        const size_t ph = ((size_t)phys * op.heads + h) * op.page + t;
        *reinterpret_cast<uint16_t*>(op.k_pool + ph * (op.head_dim / 2) + d / 2) = code;
        if (op.v) {
          const float4 vv =
              __ldg(reinterpret_cast<const float4*>(op.v + (size_t)(row_base + r0 + r) * C + c0));
          *reinterpret_cast<float4*>(op.v_pool + ph * op.head_dim + d) = vv;
        }
      }
    }
  }
}

// Groups longer than 128 rows: pass 1 min/max, pass 2 quantize (re-read, L2-resident).
__global__ void __launch_bounds__(kQuantThreads)
grouped_quant_loop_kernel(const float* __restrict__ kv, int N, int C, int R, OutContig oc) {
  __shared__ __align__(16) float s_min[kQuantWarps * kSlab];
  __shared__ __align__(16) float s_max[kQuantWarps * kSlab];
  __shared__ __align__(16) float s_lo[kSlab];
  __shared__ __align__(16) float s_sc[kSlab];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slab_c0 = blockIdx.x * kSlab;
  const int c0 = slab_c0 + lane * 4;
  const int g = blockIdx.y;
  const int r0 = g * R;
  if (r0 >= N) return;
  const int rows = min(R, N - r0);
  const bool lane_ok = c0 < C;
  float4 mn = make_float4(INFINITY, INFINITY, INFINITY, INFINITY);
  float4 mx = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  if (lane_ok) {
    for (int r = warp; r < rows; r += kQuantWarps) {
      minmax4(__ldg(reinterpret_cast<const float4*>(kv + (size_t)(r0 + r) * C + c0)), mn, mx);
    }
  }
  reduce_params(mn, mx, s_min, s_max, s_lo, s_sc, slab_c0, C, [&](int ch, float s, float z) {
    oc.scale[(size_t)g * C + ch] = s;
    oc.zp[(size_t)g * C + ch] = z;
  });
  if (!lane_ok) return;
  const float4 lo = reinterpret_cast<const float4*>(s_lo)[lane];
  const float4 sc = reinterpret_cast<const float4*>(s_sc)[lane];
  for (int r = warp; r < rows; r += kQuantWarps) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(kv + (size_t)(r0 + r) * C + c0));
    *reinterpret_cast<uint16_t*>(oc.packed + ((size_t)(r0 + r) * C + c0) / 2) = pack4(v, lo, sc);
  }
}

// Reference contract (csrc/flash_decode_int4.cu:27-83 of the reference): one
// group = all rows, one code per byte. Grid: x = 32-channel slabs, y = cluster
// of `cl` CTAs splitting the rows. Partial min/max are exchanged through
// distributed shared memory.
constexpr int kLegacyWarps = 8;
__global__ void __launch_bounds__(kLegacyWarps * 32)
legacy_quant_kernel(const float* __restrict__ kv, int rows, int C, uint8_t* __restrict__ q_out,
                    float* __restrict__ scale_out, float* __restrict__ zp_out) {
  __shared__ float s_wmin[kLegacyWarps][32];
  __shared__ float s_wmax[kLegacyWarps][32];
  __shared__ float s_pmin[32];
  __shared__ float s_pmax[32];
  __shared__ float s_lo[32];
  __shared__ float s_sc[32];
  cg::cluster_group cluster = cg::this_cluster();
  const int cl = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const bool ok = c < C;
  const int chunk = (rows + cl - 1) / cl;
  const int rb = rank * chunk;
  const int re = min(rows, rb + chunk);

  float lo = INFINITY, hi = -INFINITY;
  if (ok) {
    int r = rb + warp;
    for (; r + 3 * kLegacyWarps < re; r += 4 * kLegacyWarps) {
      const float a = __ldg(kv + (size_t)r * C + c);
      const float b = __ldg(kv + (size_t)(r + kLegacyWarps) * C + c);
      const float d = __ldg(kv + (size_t)(r + 2 * kLegacyWarps) * C + c);
      const float e = __ldg(kv + (size_t)(r + 3 * kLegacyWarps) * C + c);
      lo = fminf(fminf(lo, a), fminf(b, fminf(d, e)));
      hi = fmaxf(fmaxf(hi, a), fmaxf(b, fmaxf(d, e)));
    }
    for (; r < re; r += kLegacyWarps) {
      const float a = __ldg(kv + (size_t)r * C + c);
      lo = fminf(lo, a);
      hi = fmaxf(hi, a);
    }
  }
  s_wmin[warp][lane] = lo;
  s_wmax[warp][lane] = hi;
  __syncthreads();
  if (warp == 0) {
    for (int w = 1; w < kLegacyWarps; ++w) {
      lo = fminf(lo, s_wmin[w][lane]);
      hi = fmaxf(hi, s_wmax[w][lane]);
    }
    s_pmin[lane] = lo;
    s_pmax[lane] = hi;
  }
  cluster.sync();
  if (warp == 0) {
    float glo = INFINITY, ghi = -INFINITY;
    for (int k = 0; k < cl; ++k) {
      const float* pmin = cluster.map_shared_rank(s_pmin, k);
      const float* pmax = cluster.map_shared_rank(s_pmax, k);
      glo = fminf(glo, pmin[lane]);
      ghi = fmaxf(ghi, pmax[lane]);
    }
    float s, z;
    channel_params(glo, ghi, &s, &z);
    s_lo[lane] = glo;
    s_sc[lane] = s;
    if (rank == 0 && ok) {
      scale_out[c] = s;
      zp_out[c] = z;
    }
  }
  cluster.sync();  // peers are done reading this CTA's partials; s_lo/s_sc visible
  if (!ok) return;
  const float mn = s_lo[lane], sc = s_sc[lane];
  for (int r = rb + warp; r < re; r += kLegacyWarps) {
    q_out[(size_t)r * C + c] = static_cast<uint8_t>(quant_code(__ldg(kv + (size_t)r * C + c), mn, sc));
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

cudaError_t cu_quantize_int4(const float* kv, int num_rows, int num_channels, uint8_t* q_out,
                             float* scale_out, float* zp_out, cudaStream_t stream) {
  if (num_rows <= 0 || num_channels <= 0) return cudaErrorInvalidValue;
  if (!kv || !q_out || !scale_out || !zp_out) return cudaErrorInvalidValue;
  const int cl = num_rows >= 8 * 256 ? 8 : (num_rows + 255) / 256;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((num_channels + 31) / 32, cl, 1);
  cfg.blockDim = dim3(kLegacyWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = cl;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, legacy_quant_kernel, kv, num_rows, num_channels, q_out,
                                       scale_out, zp_out);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

cudaError_t int4kv_quantize_grouped(const float* kv, int num_tokens, int num_heads, int head_dim,
                                    int group_tokens, uint8_t* packed_out, float* scale_out,
                                    float* zp_out, cudaStream_t stream) {
  if (num_tokens <= 0 || num_heads <= 0 || head_dim <= 0 || group_tokens <= 0)
    return cudaErrorInvalidValue;
  if (head_dim % 4 != 0) return cudaErrorInvalidValue;
  if (!kv || !packed_out || !scale_out || !zp_out || !aligned16(kv)) return cudaErrorInvalidValue;
  const long long C = (long long)num_heads * head_dim;
  if (C > (1 << 30)) return cudaErrorInvalidValue;
  const int groups = (num_tokens + group_tokens - 1) / group_tokens;
  if (groups > 65535) return cudaErrorInvalidValue;
  dim3 grid((unsigned)((C + kSlab - 1) / kSlab), groups, 1);
  OutContig oc{packed_out, scale_out, zp_out};
  if (group_tokens <= kRegGroupMax) {
    grouped_quant_kernel<false><<<grid, kQuantThreads, 0, stream>>>(kv, num_tokens, (int)C,
                                                                     group_tokens, oc, OutPaged{});
  } else {
    grouped_quant_loop_kernel<<<grid, kQuantThreads, 0, stream>>>(kv, num_tokens, (int)C,
                                                                  group_tokens, oc);
  }
  return cudaGetLastError();
}

cudaError_t int4kv_cache_write(const float* k, const float* v, const int32_t* tok_offsets,
                               const int32_t* start_pos, int batch, int max_rows_per_seq,
                               int num_heads, int head_dim, int group_tokens, int page_tokens,
                               const int32_t* block_table, int max_pages, int num_pages,
                               uint8_t* k_pool, float* v_pool, float* sz_pool, uint32_t* status,
                               cudaStream_t stream) {
  if (batch <= 0 || max_rows_per_seq < 0 || num_heads <= 0 || head_dim <= 0) return cudaErrorInvalidValue;
  if (head_dim % 4 != 0 || page_tokens <= 0 || group_tokens <= 0) return cudaErrorInvalidValue;
  if (group_tokens % page_tokens != 0 || group_tokens > kRegGroupMax) return cudaErrorInvalidValue;
  if (!k || !tok_offsets || !block_table || !k_pool || !sz_pool || !aligned16(k)) return cudaErrorInvalidValue;
  if (v && (!v_pool || !aligned16(v) || !aligned16(v_pool))) return cudaErrorInvalidValue;
  if (max_pages <= 0 || num_pages <= 0 || batch > 65535) return cudaErrorInvalidValue;
  if (max_rows_per_seq == 0) return cudaSuccess;
  const long long C = (long long)num_heads * head_dim;
  if (C > (1 << 30)) return cudaErrorInvalidValue;
  const int groups = (max_rows_per_seq + group_tokens - 1) / group_tokens;
  if (groups > 65535) return cudaErrorInvalidValue;
  dim3 grid((unsigned)((C + kSlab - 1) / kSlab), groups, batch);
  OutPaged op{v, tok_offsets, start_pos, block_table, max_pages, page_tokens, num_pages,
              num_heads, head_dim, k_pool, v_pool, sz_pool, status};
  grouped_quant_kernel<true><<<grid, kQuantThreads, 0, stream>>>(k, max_rows_per_seq, (int)C,
                                                                  group_tokens, OutContig{}, op);
  return cudaGetLastError();
}

}  // extern "C"
