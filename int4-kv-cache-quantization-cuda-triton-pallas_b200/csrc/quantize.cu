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
//   legacy_*_kernel       -- the reference's cu_quantize_int4 contract: one group
//                            = all rows, one value per byte. Four launches chained
//                            by programmatic dependent launch, no scratch beyond the
//                            outputs: the scale / zp outputs first hold the running
//                            per-channel max / min as order-preserving integer keys
//                            (atomic max / min from every row chunk), then the
//                            codes are written from them, then they are replaced by
//                            the final scale / zp.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "../../include/int4kv_b200.h"

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
  void* v_pool;              // [num_pages, H, page, D] of value kind `vk`
  int vk;                    // INT4KV_VALUES_*
  float* sz_pool;            // [num_pages, H, 2, D]
  uint32_t* status;          // nullable
};

__device__ __forceinline__ void minmax4(const float4& v, float4& mn, float4& mx) {
  mn.x = fminf(mn.x, v.x); mn.y = fminf(mn.y, v.y); mn.z = fminf(mn.z, v.z); mn.w = fminf(mn.w, v.w);
  mx.x = fmaxf(mx.x, v.x); mx.y = fmaxf(mx.y, v.y); mx.z = fmaxf(mx.z, v.z); mx.w = fmaxf(mx.w, v.w);
}

__device__ __forceinline__ uint16_t pack4(const float4& v, const float4& mn, const float4& sc,
                                           const float4& rc) {
  return static_cast<uint16_t>(pack4_rcp(v, mn, sc, rc));
}

// Cross-warp reduction of per-lane [4-channel] min/max into per-channel
// (min, scale, 1/scale) in shared memory; also emits scale/zp through
// `emit(ch, s, z)`.
template <class Emit>
__device__ __forceinline__ void reduce_params(float4 mn, float4 mx, float* s_min, float* s_max,
                                              float* s_lo, float* s_sc, float* s_rc, int slab_c0,
                                              int C, Emit emit) {
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
    s_rc[ch] = __frcp_rn(s);
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
  __shared__ __align__(16) float s_rc[kSlab];

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
    reduce_params(mn, mx, s_min, s_max, s_lo, s_sc, s_rc, slab_c0, C, [&](int ch, float s, float z) {
      oc.scale[(size_t)g * C + ch] = s;
      oc.zp[(size_t)g * C + ch] = z;
    });
  } else {
    const int gpos = pos0 + r0;  // absolute position of the group's first token
    const int gpage = gpos / op.page;
    int slot = (gpage < op.max_pages) ? op.block_table[(size_t)seq * op.max_pages + gpage] : -1;
    if (slot < 0 || slot >= op.num_pages) slot = -1;
    reduce_params(mn, mx, s_min, s_max, s_lo, s_sc, s_rc, slab_c0, C, [&](int ch, float s, float z) {
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
  const float4 rc = reinterpret_cast<const float4*>(s_rc)[lane];
#pragma unroll
  for (int i = 0; i < kMaxRowsPerWarp; ++i) {
    const int r = warp + i * kQuantWarps;
    if (r < rows) {
      const uint16_t code = pack4(vals[i], lo, sc, rc);
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
          const size_t vi = ph * op.head_dim + d;
          if (op.vk == INT4KV_VALUES_F32) {
            *reinterpret_cast<float4*>(static_cast<float*>(op.v_pool) + vi) = vv;
          } else if (op.vk == INT4KV_VALUES_F16) {
            const __half2 a = __floats2half2_rn(vv.x, vv.y), b = __floats2half2_rn(vv.z, vv.w);
            uint2 w;
            w.x = *reinterpret_cast<const uint32_t*>(&a);
            w.y = *reinterpret_cast<const uint32_t*>(&b);
            *reinterpret_cast<uint2*>(static_cast<__half*>(op.v_pool) + vi) = w;
          } else {
            const __nv_bfloat162 a = __floats2bfloat162_rn(vv.x, vv.y), b = __floats2bfloat162_rn(vv.z, vv.w);
            uint2 w;
            w.x = *reinterpret_cast<const uint32_t*>(&a);
            w.y = *reinterpret_cast<const uint32_t*>(&b);
            *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(op.v_pool) + vi) = w;
          }
        }
      }
    }
  }
}

// Persistent, TMA-pipelined form of grouped_quant_kernel for the contiguous
// output (groups of R <= 128 rows, C % SLAB == 0). CTAs walk tiles (group g,
// SLAB-channel slab) t = blockIdx.x, + gridDim.x, ...; the TMA engine moves
// each tile (R rows x 4 SLAB bytes, one 2-D tensor copy) into a ring of
// kTmaStages shared-memory stages, so later tiles stream in while the current
// one is reduced and quantized. Thread (row group q = tid / (SLAB/4), channel
// quad c = tid % (SLAB/4)) owns channels [4c, 4c+4) of rows q, q + 512/(SLAB/4),
// ..., held in registers between the min/max pass and the quantize pass; the
// threads of a row store its SLAB/2 code bytes together (whole sectors).
// Thread 0 alone waits on a stage's barrier (bounded) and the CTA learns the
// outcome through shared memory, so every thread takes the same path; after a
// timeout the CTA drains its copies (bounded), writes NaN into the scale/zp
// of every tile it did not finish, and exits.
//
// Two widths. SLAB = 128 (one CTA per SM, 64 KB stages) reads each token row
// in 512-byte pieces and is used whenever C % 128 == 0; SLAB = 64 (two CTAs
// per SM, 32 KB stages, 256-byte pieces) serves the other widths. Measured on
// B200 at 32 heads x d128 (C = 4096, rows 16 KB apart): 459 us (128) vs 508
// us (64) at 131072 tokens, 123 vs 135 at 32768, 38.6 vs 41.0 at 8192, the
// same ~20 us at 2048 -- the wider pieces stream better from HBM, though the
// 64-wide form overlaps one CTA's barriers with the other CTA's streaming.
constexpr int kTmaStages = 3;
constexpr int kTmaThreads = 512;
constexpr int kTileRows = kRegGroupMax;                     // 128
constexpr int kTmaWarps = kTmaThreads / 32;
constexpr uint64_t kQuantWaitNs = 2000000000ull;            // 2 s

template <int SLAB>
struct TmaShape {
  static constexpr int kQuads = SLAB / 4;                          // threads per row
  static constexpr int kRowGroups = kTmaThreads / kQuads;
  static constexpr int kRowsPerThread = kTileRows / kRowGroups;    // 4 (64) or 8 (128)
  static constexpr int kCtasPerSm = SLAB == 64 ? 2 : 1;
};

template <int SLAB>
struct TmaSmem {
  float stage[kTmaStages][kTileRows * SLAB];
  float4 s_min[kTmaWarps * (SLAB / 4)];   // [warp][channel quad] partials (SLAB 64: 2 row groups folded)
  float4 s_max[kTmaWarps * (SLAB / 4)];
  float s_lo[SLAB];
  float s_sc[SLAB];
  float s_rc[SLAB];
  uint64_t bar[kTmaStages];
  int ok;
};

// Load tile `tile` into `dst`: one 2-D tensor copy for a full group; the
// short last group (rows < R) instead takes one 1-D bulk copy per row, so no
// box ever reaches past the tensor and the byte count is exact.
template <int SLAB>
__device__ __forceinline__ void tma_issue_tile(const CUtensorMap* tmap, const float* kv, int N,
                                               int C, int R, int S, long long tile, float* dst,
                                               uint64_t* bar) {
  const int g = (int)(tile / S), slab = (int)(tile - (long long)g * S);
  const int r0 = g * R, rows = min(R, N - r0);
  fence_proxy_async_smem();
  mbar_arrive_expect_tx(bar, (uint32_t)(rows * SLAB * 4));
  if (rows == R) {
    tma_load_2d(dst, tmap, slab * SLAB, r0, bar);
  } else {
    for (int r = 0; r < rows; ++r)
      bulk_g2s(dst + r * SLAB, kv + (size_t)(r0 + r) * C + slab * SLAB, SLAB * 4, bar);
  }
}

template <int SLAB>
__global__ void __launch_bounds__(kTmaThreads, TmaShape<SLAB>::kCtasPerSm)
grouped_quant_tma_kernel(const __grid_constant__ CUtensorMap tmap, const float* __restrict__ kv,
                         int N, int C, int R, OutContig oc) {
  extern __shared__ __align__(128) char smem_raw[];
  using Sh = TmaShape<SLAB>;
  constexpr int kTmaSlab = SLAB, kTmaQuads = Sh::kQuads, kTmaRowGroups = Sh::kRowGroups,
                kTmaRowsPerThread = Sh::kRowsPerThread;
  TmaSmem<SLAB>& sm = *reinterpret_cast<TmaSmem<SLAB>*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cq = tid % kTmaQuads, rg = tid / kTmaQuads;
  const int S = C / kTmaSlab;  // C % kTmaSlab == 0 (launcher)
  const long long total = (long long)((N + R - 1) / R) * S;
  const long long first = blockIdx.x, step = gridDim.x;
  if (first >= total) return;
  if (tid == 0) {
    for (int i = 0; i < kTmaStages; ++i) mbar_init(&sm.bar[i], 1);
    fence_barrier_init();
    for (int i = 0; i < kTmaStages; ++i) {
      const long long t = first + i * step;
      if (t < total) tma_issue_tile<SLAB>(&tmap, kv, N, C, R, S, t, sm.stage[i], &sm.bar[i]);
    }
  }
  __syncthreads();
  // tile t = g * S + slab, walked incrementally (no division per tile)
  const int step_g = (int)(step / S), step_s = (int)(step - (long long)step_g * S);
  int g = (int)(first / S), slab = (int)(first - (long long)g * S);
  int st = 0;
  uint32_t parity = 0;
  long long i = 0;
  for (long long t = first; t < total; t += step, ++i) {
    if (tid == 0) sm.ok = mbar_wait_bounded(&sm.bar[st], parity, kQuantWaitNs) ? 1 : 0;
    __syncthreads();
    if (!sm.ok) {
      // drain the copies still in flight (bounded), poison what was not done
      if (tid == 0) {
        for (long long k = 0; k < kTmaStages && t + k * step < total; ++k)
          (void)mbar_wait_bounded(&sm.bar[(i + k) % kTmaStages],
                                  (uint32_t)(((i + k) / kTmaStages) & 1), kQuantWaitNs);
      }
      for (long long u = t; u < total; u += step) {
        const int g = (int)(u / S), c0 = (int)(u - (long long)g * S) * kTmaSlab;
        for (int c = tid; c < kTmaSlab; c += blockDim.x) {
          oc.scale[(size_t)g * C + c0 + c] = __int_as_float(0x7fc00000);
          oc.zp[(size_t)g * C + c0 + c] = __int_as_float(0x7fc00000);
        }
      }
      return;
    }
    (void)mbar_try_wait(&sm.bar[st], parity);  // completed: acquire for this thread too
    const int r0 = g * R, rows = min(R, N - r0);
    const int slab_c0 = slab * kTmaSlab;
    const float* tile = sm.stage[st];

    float4 vals[kTmaRowsPerThread];
    float4 mn, mx;
    if (rows == kTileRows) {  // full tile: three-input min / max over the thread's rows
#pragma unroll
      for (int k = 0; k < kTmaRowsPerThread; ++k)
        vals[k] = reinterpret_cast<const float4*>(tile + (rg + k * kTmaRowGroups) * kTmaSlab)[cq];
      if constexpr (kTmaRowsPerThread == 4) {
        mn.x = fmin3f(fmin3f(vals[0].x, vals[1].x, vals[2].x), vals[3].x, INFINITY);
        mn.y = fmin3f(fmin3f(vals[0].y, vals[1].y, vals[2].y), vals[3].y, INFINITY);
        mn.z = fmin3f(fmin3f(vals[0].z, vals[1].z, vals[2].z), vals[3].z, INFINITY);
        mn.w = fmin3f(fmin3f(vals[0].w, vals[1].w, vals[2].w), vals[3].w, INFINITY);
        mx.x = fmax3f(fmax3f(vals[0].x, vals[1].x, vals[2].x), vals[3].x, -INFINITY);
        mx.y = fmax3f(fmax3f(vals[0].y, vals[1].y, vals[2].y), vals[3].y, -INFINITY);
        mx.z = fmax3f(fmax3f(vals[0].z, vals[1].z, vals[2].z), vals[3].z, -INFINITY);
        mx.w = fmax3f(fmax3f(vals[0].w, vals[1].w, vals[2].w), vals[3].w, -INFINITY);
      } else {
        static_assert(kTmaRowsPerThread == 8, "min3/max3 chains for 4 or 8 rows");
#define I4KV_CHAIN3(f3, f2, c) \
  f2(f3(f3(f3(vals[0].c, vals[1].c, vals[2].c), vals[3].c, vals[4].c), vals[5].c, vals[6].c), vals[7].c)
        mn.x = I4KV_CHAIN3(fmin3f, fminf, x); mn.y = I4KV_CHAIN3(fmin3f, fminf, y);
        mn.z = I4KV_CHAIN3(fmin3f, fminf, z); mn.w = I4KV_CHAIN3(fmin3f, fminf, w);
        mx.x = I4KV_CHAIN3(fmax3f, fmaxf, x); mx.y = I4KV_CHAIN3(fmax3f, fmaxf, y);
        mx.z = I4KV_CHAIN3(fmax3f, fmaxf, z); mx.w = I4KV_CHAIN3(fmax3f, fmaxf, w);
#undef I4KV_CHAIN3
      }
    } else {
      mn = make_float4(INFINITY, INFINITY, INFINITY, INFINITY);
      mx = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
#pragma unroll
      for (int k = 0; k < kTmaRowsPerThread; ++k) {
        const int r = rg + k * kTmaRowGroups;
        if (r < rows) {
          vals[k] = reinterpret_cast<const float4*>(tile + r * kTmaSlab)[cq];
          minmax4(vals[k], mn, mx);
        }
      }
    }
    // fold the warp's two row groups (lanes l and l ^ 16 hold the same quad)
    if constexpr (kTmaQuads == 16) {
      float4 o;
      o.x = __shfl_xor_sync(0xffffffffu, mn.x, 16); o.y = __shfl_xor_sync(0xffffffffu, mn.y, 16);
      o.z = __shfl_xor_sync(0xffffffffu, mn.z, 16); o.w = __shfl_xor_sync(0xffffffffu, mn.w, 16);
      float4 p;
      p.x = __shfl_xor_sync(0xffffffffu, mx.x, 16); p.y = __shfl_xor_sync(0xffffffffu, mx.y, 16);
      p.z = __shfl_xor_sync(0xffffffffu, mx.z, 16); p.w = __shfl_xor_sync(0xffffffffu, mx.w, 16);
      mn.x = fminf(mn.x, o.x); mn.y = fminf(mn.y, o.y); mn.z = fminf(mn.z, o.z); mn.w = fminf(mn.w, o.w);
      mx.x = fmaxf(mx.x, p.x); mx.y = fmaxf(mx.y, p.y); mx.z = fmaxf(mx.z, p.z); mx.w = fmaxf(mx.w, p.w);
    }
    if (lane < kTmaQuads) {
      sm.s_min[warp * kTmaQuads + lane] = mn;
      sm.s_max[warp * kTmaQuads + lane] = mx;
    }
    __syncthreads();  // stage st fully read: refill it; partial min/max visible
    if (tid == 0 && t + kTmaStages * step < total)
      tma_issue_tile<SLAB>(&tmap, kv, N, C, R, S, t + kTmaStages * step, sm.stage[st], &sm.bar[st]);
    if (tid < kTmaSlab) {
      // consecutive threads read consecutive channels of each warp's partials
      const float* pmin = reinterpret_cast<const float*>(sm.s_min);
      const float* pmax = reinterpret_cast<const float*>(sm.s_max);
      const int ch = tid;
      float lo = pmin[ch], hi = pmax[ch];
#pragma unroll
      for (int w = 1; w < kTmaWarps; ++w) {
        lo = fminf(lo, pmin[w * kTmaSlab + ch]);
        hi = fmaxf(hi, pmax[w * kTmaSlab + ch]);
      }
      float sc, zp;
      channel_params(lo, hi, &sc, &zp);
      sm.s_lo[ch] = lo;
      sm.s_sc[ch] = sc;
      sm.s_rc[ch] = __frcp_rn(sc);
      oc.scale[(size_t)g * C + slab_c0 + ch] = sc;
      oc.zp[(size_t)g * C + slab_c0 + ch] = zp;
    }
    __syncthreads();
    {
      const float4 lo = reinterpret_cast<const float4*>(sm.s_lo)[cq];
      const float4 sc = reinterpret_cast<const float4*>(sm.s_sc)[cq];
      const float4 rc = reinterpret_cast<const float4*>(sm.s_rc)[cq];
      // the 16 threads of a row write its 32 code bytes: one full sector
#pragma unroll
      for (int k = 0; k < kTmaRowsPerThread; ++k) {
        const int r = rg + k * kTmaRowGroups;
        if (r < rows)
          *reinterpret_cast<uint16_t*>(oc.packed + ((size_t)(r0 + r) * C + slab_c0) / 2 + cq * 2) =
              pack4(vals[k], lo, sc, rc);
      }
    }
    g += step_g;
    slab += step_s;
    if (slab >= S) { slab -= S; ++g; }
    if (++st == kTmaStages) { st = 0; parity ^= 1u; }
  }
}

// Token append for decode steps: sequence b adds one token at position
// pos_b; its group (the R tokens starting at pos_b - pos_b % R) is still open,
// so the whole group is quantized again over its valid rows only -- the
// reference's rule for a partial group (min / max over the rows it holds) --
// and after the last append of a group the cache equals a bulk write of the
// same tokens bit for bit. The float32 keys of the open group live in a
// staging slot [R, C] per sequence: rows 0 .. pos%R-1 from earlier appends
// (or the prefill), row pos%R is the new token, written into the slot here.
// Grid: x = 128-channel slabs, y = sequences; codes, the group's scale/zp and
// the new value row land in the pools like grouped_quant_kernel<true>.
struct AppendArgs {
  const float* k_new;        // [B, C]
  const float* v_new;        // [B, C] (nullable)
  const int32_t* pos;        // [B] position of the new token
  const int32_t* slot;       // [B] staging slot of each sequence
  float* stage;              // [slots, R, C]
  int num_slots;
  // Rotary position embedding of the new token's key and of the step's query
  // (nullable: no rotation). cos/sin [rope_positions, head_dim / 2] float32.
  const float* rope_cos;
  const float* rope_sin;
  int rope_positions;
  const float* q_in;         // [B, q_heads * head_dim] (nullable)
  float* q_out;              // [B, q_heads * head_dim]
  int q_heads;
};

// Rotary embedding (the rotate-half form of Llama,
// transformers.models.llama.modeling_llama.apply_rotary_pos_emb) of the four
// channels d .. d+3 of one head row `x` (head_dim hd, d % 4 == 0) at table row
// `cs`/`sn`: out_i = x_i c_i - x_{i+hd/2} s_i below hd/2, x_i c_i + x_{i-hd/2} s_i
// above, each product and the sum rounded to float32 (no contraction), as the
// reference model computes (q * cos) + (rotate_half(q) * sin).
__device__ __forceinline__ float4 rope4(const float* x, int d, int hd, const float* cs,
                                        const float* sn) {
  const int half = hd >> 1;
  const bool low = d < half;
  const int f = low ? d : d - half;
  const float4 a = __ldg(reinterpret_cast<const float4*>(x + d));
  const float4 b = __ldg(reinterpret_cast<const float4*>(x + (low ? d + half : d - half)));
  const float4 c = __ldg(reinterpret_cast<const float4*>(cs + f));
  const float4 s = __ldg(reinterpret_cast<const float4*>(sn + f));
  float4 o;
  if (low) {
    o.x = __fsub_rn(__fmul_rn(a.x, c.x), __fmul_rn(b.x, s.x));
    o.y = __fsub_rn(__fmul_rn(a.y, c.y), __fmul_rn(b.y, s.y));
    o.z = __fsub_rn(__fmul_rn(a.z, c.z), __fmul_rn(b.z, s.z));
    o.w = __fsub_rn(__fmul_rn(a.w, c.w), __fmul_rn(b.w, s.w));
  } else {
    o.x = __fadd_rn(__fmul_rn(a.x, c.x), __fmul_rn(b.x, s.x));
    o.y = __fadd_rn(__fmul_rn(a.y, c.y), __fmul_rn(b.y, s.y));
    o.z = __fadd_rn(__fmul_rn(a.z, c.z), __fmul_rn(b.z, s.z));
    o.w = __fadd_rn(__fmul_rn(a.w, c.w), __fmul_rn(b.w, s.w));
  }
  return o;
}

__global__ void __launch_bounds__(kQuantThreads)
append_quant_kernel(AppendArgs ap, int C, int R, OutPaged op) {
  __shared__ __align__(16) float s_min[kQuantWarps * kSlab];
  __shared__ __align__(16) float s_max[kQuantWarps * kSlab];
  __shared__ __align__(16) float s_lo[kSlab];
  __shared__ __align__(16) float s_sc[kSlab];
  __shared__ __align__(16) float s_rc[kSlab];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slab_c0 = blockIdx.x * kSlab;
  const int c0 = slab_c0 + lane * 4;
  const int b = blockIdx.y;
  const int pos = ap.pos[b], sl = ap.slot[b];
  if (pos < 0 || sl < 0 || sl >= ap.num_slots || pos / op.page >= op.max_pages ||
      (ap.rope_cos && pos >= ap.rope_positions)) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && op.status) atomicOr(op.status, kStatusBadLength);
    return;
  }
  const int half = op.head_dim >> 1;
  const float* rcos = ap.rope_cos ? ap.rope_cos + (size_t)pos * half : nullptr;
  const float* rsin = ap.rope_cos ? ap.rope_sin + (size_t)pos * half : nullptr;
  if (ap.q_in) {  // the step's query, rotated at the same position (spread over the slab CTAs)
    const long long cq = (long long)ap.q_heads * op.head_dim;
    const float* qrow = ap.q_in + (size_t)b * cq;
    for (long long c = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4; c < cq;
         c += (long long)gridDim.x * blockDim.x * 4) {
      const int hq = (int)(c / op.head_dim), d = (int)(c - (long long)hq * op.head_dim);
      const float* x = qrow + (size_t)hq * op.head_dim;
      *reinterpret_cast<float4*>(ap.q_out + (size_t)b * cq + c) =
          rcos ? rope4(x, d, op.head_dim, rcos, rsin) : __ldg(reinterpret_cast<const float4*>(x + d));
    }
  }
  const int rows = pos % R + 1, gpos = pos - (rows - 1);
  const bool lane_ok = c0 < C;
  float* stage = ap.stage + (size_t)sl * R * C;

  float4 vals[kMaxRowsPerWarp];
  float4 mn = make_float4(INFINITY, INFINITY, INFINITY, INFINITY);
  float4 mx = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
#pragma unroll
  for (int i = 0; i < kMaxRowsPerWarp; ++i) {
    const int r = warp + i * kQuantWarps;
    if (lane_ok && r < rows) {
      if (r == rows - 1) {  // the new token: from the input (rotated), and into the slot
        if (rcos) {
          const int hk = c0 / op.head_dim;
          vals[i] = rope4(ap.k_new + (size_t)b * C + (size_t)hk * op.head_dim, c0 - hk * op.head_dim,
                          op.head_dim, rcos, rsin);
        } else {
          vals[i] = __ldg(reinterpret_cast<const float4*>(ap.k_new + (size_t)b * C + c0));
        }
        *reinterpret_cast<float4*>(stage + (size_t)r * C + c0) = vals[i];
      } else {
        vals[i] = *reinterpret_cast<const float4*>(stage + (size_t)r * C + c0);
      }
      minmax4(vals[i], mn, mx);
    }
  }
  const int gpage = gpos / op.page;
  const int32_t* row_bt = op.block_table + (size_t)b * op.max_pages;
  int gslot = row_bt[gpage];
  if (gslot < 0 || gslot >= op.num_pages) gslot = -1;
  reduce_params(mn, mx, s_min, s_max, s_lo, s_sc, s_rc, slab_c0, C, [&](int ch, float sc, float zp) {
    if (gslot < 0) return;
    const int h = ch / op.head_dim, d = ch - h * op.head_dim;
    float* dst = op.sz_pool + ((size_t)gslot * op.heads + h) * 2 * op.head_dim;
    dst[d] = sc;
    dst[op.head_dim + d] = zp;
  });
  if (gslot < 0 && threadIdx.x == 0 && op.status) atomicOr(op.status, kStatusBadPage);
  if (!lane_ok) return;
  const float4 lo = reinterpret_cast<const float4*>(s_lo)[lane];
  const float4 sc = reinterpret_cast<const float4*>(s_sc)[lane];
  const float4 rc = reinterpret_cast<const float4*>(s_rc)[lane];
  const int h = c0 / op.head_dim, d = c0 - h * op.head_dim;
#pragma unroll
  for (int i = 0; i < kMaxRowsPerWarp; ++i) {
    const int r = warp + i * kQuantWarps;
    if (r < rows) {
      const int p = gpos + r;
      const int pg = p / op.page, t = p - pg * op.page;
      const int phys = row_bt[pg];
      if (phys < 0 || phys >= op.num_pages) {
        if (op.status) atomicOr(op.status, kStatusBadPage);
        continue;
      }
      const size_t ph = ((size_t)phys * op.heads + h) * op.page + t;
      *reinterpret_cast<uint16_t*>(op.k_pool + ph * (op.head_dim / 2) + d / 2) = pack4(vals[i], lo, sc, rc);
      if (r == rows - 1 && ap.v_new) {
        const float4 vv = __ldg(reinterpret_cast<const float4*>(ap.v_new + (size_t)b * C + c0));
        const size_t vi = ph * op.head_dim + d;
        if (op.vk == INT4KV_VALUES_F32) {
          *reinterpret_cast<float4*>(static_cast<float*>(op.v_pool) + vi) = vv;
        } else if (op.vk == INT4KV_VALUES_F16) {
          const __half2 x = __floats2half2_rn(vv.x, vv.y), y = __floats2half2_rn(vv.z, vv.w);
          uint2 w;
          w.x = *reinterpret_cast<const uint32_t*>(&x);
          w.y = *reinterpret_cast<const uint32_t*>(&y);
          *reinterpret_cast<uint2*>(static_cast<__half*>(op.v_pool) + vi) = w;
        } else {
          const __nv_bfloat162 x = __floats2bfloat162_rn(vv.x, vv.y), y = __floats2bfloat162_rn(vv.z, vv.w);
          uint2 w;
          w.x = *reinterpret_cast<const uint32_t*>(&x);
          w.y = *reinterpret_cast<const uint32_t*>(&y);
          *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(op.v_pool) + vi) = w;
        }
      }
    }
  }
}

// Rotary embedding of rows x[rows, heads, head_dim] at positions[rows] into
// out (a separate buffer: each channel reads its partner channel of x): the
// prefill's keys before they are quantized, with the arithmetic of rope4.
// One thread per four channels; a position outside the table gives NaN and
// INT4KV_STATUS_BAD_LENGTH.
__global__ void __launch_bounds__(256)
rope_rows_kernel(const float* __restrict__ x, const int32_t* __restrict__ positions, int rows,
                 int heads, int hd, const float* __restrict__ cs, const float* __restrict__ sn,
                 int rope_positions, float* out, uint32_t* status) {
  const long long row_ch = (long long)heads * hd;
  const long long total4 = (long long)rows * row_ch / 4;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total4;
       i += (long long)gridDim.x * blockDim.x) {
    const long long c = i * 4;
    const long long r = c / row_ch;
    const int ch = (int)(c - r * row_ch);
    const int h = ch / hd, d = ch - h * hd;
    const int pos = positions[r];
    float4 o;
    if (pos < 0 || pos >= rope_positions) {
      if (status) atomicOr(status, kStatusBadLength);
      o = make_float4(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000),
                      __int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
    } else {
      o = rope4(x + r * row_ch + (long long)h * hd, d, hd, cs + (size_t)pos * (hd / 2),
                sn + (size_t)pos * (hd / 2));
    }
    *reinterpret_cast<float4*>(out + c) = o;
  }
}

// Groups longer than 128 rows: pass 1 min/max, pass 2 quantize (re-read, L2-resident).
__global__ void __launch_bounds__(kQuantThreads)
grouped_quant_loop_kernel(const float* __restrict__ kv, int N, int C, int R, OutContig oc) {
  __shared__ __align__(16) float s_min[kQuantWarps * kSlab];
  __shared__ __align__(16) float s_max[kQuantWarps * kSlab];
  __shared__ __align__(16) float s_lo[kSlab];
  __shared__ __align__(16) float s_sc[kSlab];
  __shared__ __align__(16) float s_rc[kSlab];
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
  reduce_params(mn, mx, s_min, s_max, s_lo, s_sc, s_rc, slab_c0, C, [&](int ch, float s, float z) {
    oc.scale[(size_t)g * C + ch] = s;
    oc.zp[(size_t)g * C + ch] = z;
  });
  if (!lane_ok) return;
  const float4 lo = reinterpret_cast<const float4*>(s_lo)[lane];
  const float4 sc = reinterpret_cast<const float4*>(s_sc)[lane];
  const float4 rc = reinterpret_cast<const float4*>(s_rc)[lane];
  for (int r = warp; r < rows; r += kQuantWarps) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(kv + (size_t)(r0 + r) * C + c0));
    *reinterpret_cast<uint16_t*>(oc.packed + ((size_t)(r0 + r) * C + c0) / 2) = pack4(v, lo, sc, rc);
  }
}

// Reference contract (csrc/flash_decode_int4.cu:27-83 of the reference): one
// group = all rows, one code per byte. The min / max over all rows is a
// reduction across the whole grid, and the reference's launcher takes no
// scratch buffer, so it is split at the one point where every CTA must have
// contributed: kernel boundaries, whose launch gaps programmatic dependent
// launch hides. Each CTA owns a chunk of rows of one 128-channel tile; a warp
// reads whole 512-byte row pieces (float4 per lane) when the rows allow it.
//   1. legacy_keys_init   : scale_out / zp_out <- the keys of -inf / +inf
//   2. legacy_minmax      : per-CTA min / max of its chunk, then one atomicMax /
//                           atomicMin of the order-preserving key per channel
//   3. legacy_codes       : codes of the chunk from the final min / max (the
//                           chunk is read again, from L2 when it fits there)
//   4. legacy_params      : scale_out / zp_out <- scale, zp of each channel
// Steps 2-4 call grid_dependency_wait() before they touch what the step before
// wrote, so starting early never changes a result. Step 1 is launched the same
// way and waits first for whatever kernel precedes it on the stream (a
// previous call's step 4 writes the same outputs); step 4 lets the next
// call's step 1 be dispatched while it runs.
constexpr int kLegWarps = 8;
constexpr int kLegTile = 128;  // channels per CTA (32 lanes x 4)

__global__ void __launch_bounds__(256)
legacy_keys_init(float* __restrict__ scale_out, float* __restrict__ zp_out, int C) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  grid_dependency_wait();  // the previous kernel on the stream is done with the outputs
  if (c < C) {
    reinterpret_cast<uint32_t*>(scale_out)[c] = 0u;           // below the key of any float
    reinterpret_cast<uint32_t*>(zp_out)[c] = 0xffffffffu;     // above the key of any float
  }
  allow_dependent_launch();
}

constexpr int kLegRes = 16;  // rows per warp held in registers (all loads in flight at once)

template <bool VEC>
__global__ void __launch_bounds__(kLegWarps * 32)
legacy_minmax(const float* __restrict__ kv, int rows, int C, int chunk,
              float* __restrict__ scale_out, float* __restrict__ zp_out) {
  __shared__ float s_lo[kLegWarps][kLegTile];
  __shared__ float s_hi[kLegWarps][kLegTile];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = blockIdx.y * kLegTile;
  const int r0 = blockIdx.x * chunk;
  const int r1 = min(rows, r0 + chunk);
  float lo[4], hi[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) lo[k] = INFINITY, hi[k] = -INFINITY;
  if constexpr (VEC) {
    const int c = c0 + 4 * lane;
    if (c < C) {
      const float* p = kv + (size_t)r0 * C + c;
      for (int rb = r0 + warp; rb < r1; rb += kLegRes * kLegWarps) {
        float4 v[kLegRes];  // up to kLegRes rows of this warp requested before any is used
#pragma unroll
        for (int k = 0; k < kLegRes; ++k) {
          const int r = rb + k * kLegWarps;
          if (r < r1) v[k] = __ldg(reinterpret_cast<const float4*>(p + (size_t)(r - r0) * C));
        }
#pragma unroll
        for (int k = 0; k < kLegRes; ++k) {
          if (rb + k * kLegWarps < r1) {
            lo[0] = fminf(lo[0], v[k].x); hi[0] = fmaxf(hi[0], v[k].x);
            lo[1] = fminf(lo[1], v[k].y); hi[1] = fmaxf(hi[1], v[k].y);
            lo[2] = fminf(lo[2], v[k].z); hi[2] = fmaxf(hi[2], v[k].z);
            lo[3] = fminf(lo[3], v[k].w); hi[3] = fmaxf(hi[3], v[k].w);
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      s_lo[warp][4 * lane + k] = lo[k];
      s_hi[warp][4 * lane + k] = hi[k];
    }
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = c0 + lane + 32 * k;
      if (c < C) {
        for (int r = r0 + warp; r < r1; r += kLegWarps) {
          const float a = __ldg(kv + (size_t)r * C + c);
          lo[k] = fminf(lo[k], a);
          hi[k] = fmaxf(hi[k], a);
        }
      }
      s_lo[warp][lane + 32 * k] = lo[k];
      s_hi[warp][lane + 32 * k] = hi[k];
    }
  }
  allow_dependent_launch();
  __syncthreads();
  const int t = threadIdx.x;
  if (t < kLegTile && c0 + t < C) {
    float l = s_lo[0][t], h = s_hi[0][t];
#pragma unroll
    for (int w = 1; w < kLegWarps; ++w) {
      l = fminf(l, s_lo[w][t]);
      h = fmaxf(h, s_hi[w][t]);
    }
    grid_dependency_wait();  // the keys were initialised by the previous launch
    if (h >= l) {            // a chunk with no rows (or only NaN) leaves the keys alone
      atomicMax(reinterpret_cast<unsigned int*>(scale_out) + c0 + t, ordered_key(h));
      atomicMin(reinterpret_cast<unsigned int*>(zp_out) + c0 + t, ordered_key(l));
    }
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kLegWarps * 32)
legacy_codes(const float* __restrict__ kv, int rows, int C, int chunk,
             const float* __restrict__ max_keys, const float* __restrict__ min_keys,
             uint8_t* __restrict__ q_out) {
  __shared__ __align__(16) float s_mn[kLegTile];
  __shared__ __align__(16) float s_sc[kLegTile];
  __shared__ __align__(16) float s_rc[kLegTile];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = blockIdx.y * kLegTile;
  const int r0 = blockIdx.x * chunk;
  const int r1 = min(rows, r0 + chunk);
  const int t = threadIdx.x;
  const int cv = c0 + 4 * lane;
  // The input does not depend on the previous launch: a chunk that fits in
  // registers is requested before waiting for the keys, so its loads overlap
  // the min / max step's tail.
  const bool resident = VEC && chunk <= kLegRes * kLegWarps;
  float4 v[kLegRes];
  if (resident && cv < C) {
#pragma unroll
    for (int k = 0; k < kLegRes; ++k) {
      const int r = r0 + warp + k * kLegWarps;
      if (r < r1) v[k] = __ldg(reinterpret_cast<const float4*>(kv + (size_t)r * C + cv));
    }
  }
  grid_dependency_wait();  // every chunk's min / max has landed in the keys
  if (t < kLegTile) {
    float mn = 0.f, sc = 1.f;
    if (c0 + t < C) {
      mn = from_ordered_key(reinterpret_cast<const uint32_t*>(min_keys)[c0 + t]);
      const float mx = from_ordered_key(reinterpret_cast<const uint32_t*>(max_keys)[c0 + t]);
      float zp;
      channel_params(mn, mx, &sc, &zp);
    }
    s_mn[t] = mn;
    s_sc[t] = sc;
    s_rc[t] = __frcp_rn(sc);
  }
  __syncthreads();
  allow_dependent_launch();
  if constexpr (VEC) {
    if (cv >= C) return;
    const float4 mn = reinterpret_cast<const float4*>(s_mn)[lane];
    const float4 sc = reinterpret_cast<const float4*>(s_sc)[lane];
    const float4 rc = reinterpret_cast<const float4*>(s_rc)[lane];
    if (resident) {
#pragma unroll
      for (int k = 0; k < kLegRes; ++k) {
        const int r = r0 + warp + k * kLegWarps;
        if (r < r1)
          *reinterpret_cast<uint32_t*>(q_out + (size_t)r * C + cv) = codes4_rcp(v[k], mn, sc, rc);
      }
    } else {
      for (int r = r0 + warp; r < r1; r += kLegWarps) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(kv + (size_t)r * C + cv));
        *reinterpret_cast<uint32_t*>(q_out + (size_t)r * C + cv) = codes4_rcp(x, mn, sc, rc);
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = c0 + lane + 32 * k;
      if (c >= C) continue;
      const float mn = s_mn[lane + 32 * k], sc = s_sc[lane + 32 * k], rc = s_rc[lane + 32 * k];
      for (int r = r0 + warp; r < r1; r += kLegWarps)
        q_out[(size_t)r * C + c] =
            static_cast<uint8_t>(quant_code_rcp(__ldg(kv + (size_t)r * C + c), mn, sc, rc));
    }
  }
}

__global__ void __launch_bounds__(256)
legacy_params(float* __restrict__ scale_out, float* __restrict__ zp_out, int C) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  grid_dependency_wait();  // every CTA of the codes step has read the keys
  allow_dependent_launch();
  if (c < C) {
    const float mx = from_ordered_key(reinterpret_cast<const uint32_t*>(scale_out)[c]);
    const float mn = from_ordered_key(reinterpret_cast<const uint32_t*>(zp_out)[c]);
    float s, z;
    channel_params(mn, mx, &s, &z);
    scale_out[c] = s;
    zp_out[c] = z;
  }
}

int device_sms() {
  static std::mutex mu;
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if (!sms[dev] && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    sms[dev] = 148;
  return sms[dev];
}

// Launch `kern` with the programmatic-serialization attribute: it may begin
// while the previous kernel on `stream` is still running (it waits for that
// kernel's results with grid_dependency_wait()).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// SM count and the persistent kernel's shared-memory opt-in, once per device.
cudaError_t tma_quant_setup(int* sms_out) {
  static std::mutex mu;
  static int sms[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(mu);
  if (!sms[dev]) {
    e = cudaFuncSetAttribute(grouped_quant_tma_kernel<64>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(TmaSmem<64>));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(grouped_quant_tma_kernel<128>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(TmaSmem<128>));
    if (e != cudaSuccess) return e;
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    sms[dev] = n;
  }
  *sms_out = sms[dev];
  return cudaSuccess;
}

// 2-D tensor map over a row-major float32 matrix [rows, cols]: boxes of
// box_rows x box_cols (the driver's encoder, reached through the runtime so
// the library does not link libcuda itself).
cudaError_t encode_rows_map(CUtensorMap* map, const float* base, int rows, int cols, int box_cols,
                            int box_rows) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!encode) {
      cudaDriverEntryPointQueryResult qr;
      void* fn = nullptr;
      const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr);
      if (e != cudaSuccess) return e;
      if (qr != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * sizeof(float)};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims,
                            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

extern "C" {

cudaError_t cu_quantize_int4(const float* kv, int num_rows, int num_channels, uint8_t* q_out,
                             float* scale_out, float* zp_out, cudaStream_t stream) {
  if (num_rows <= 0 || num_channels <= 0) return cudaErrorInvalidValue;
  if (!kv || !q_out || !scale_out || !zp_out) return cudaErrorInvalidValue;
  const int C = num_channels;
  const int tiles = (C + kLegTile - 1) / kLegTile;
  // about two CTAs per SM in all, more when that keeps every chunk within the
  // rows the warps hold in registers; at least 8 rows (one per warp) per chunk
  int chunks = (2 * device_sms() + tiles - 1) / tiles;
  chunks = max(chunks, (num_rows + kLegRes * kLegWarps - 1) / (kLegRes * kLegWarps));
  chunks = min(chunks, (num_rows + kLegWarps - 1) / kLegWarps);
  chunks = max(chunks, 1);
  const int chunk = (num_rows + chunks - 1) / chunks;
  chunks = (num_rows + chunk - 1) / chunk;
  const bool vec = C % 4 == 0 && aligned16(kv) && (reinterpret_cast<uintptr_t>(q_out) & 3u) == 0;
  const dim3 grid(chunks, tiles), block(kLegWarps * 32);
  const dim3 pgrid((C + 255) / 256), pblock(256);
  cudaError_t e = launch_pdl(legacy_keys_init, pgrid, pblock, stream, scale_out, zp_out, C);
  if (e != cudaSuccess) return e;
  e = vec ? launch_pdl(legacy_minmax<true>, grid, block, stream, kv, num_rows, C, chunk,
                       scale_out, zp_out)
          : launch_pdl(legacy_minmax<false>, grid, block, stream, kv, num_rows, C, chunk,
                       scale_out, zp_out);
  if (e != cudaSuccess) return e;
  e = vec ? launch_pdl(legacy_codes<true>, grid, block, stream, kv, num_rows, C, chunk,
                       static_cast<const float*>(scale_out), static_cast<const float*>(zp_out),
                       q_out)
          : launch_pdl(legacy_codes<false>, grid, block, stream, kv, num_rows, C, chunk,
                       static_cast<const float*>(scale_out), static_cast<const float*>(zp_out),
                       q_out);
  if (e != cudaSuccess) return e;
  e = launch_pdl(legacy_params, pgrid, pblock, stream, scale_out, zp_out, C);
  if (e != cudaSuccess) return e;
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
  cudaError_t e = cudaSuccess;
  int sms = 0;
  CUtensorMap tmap;
  // 128-channel slabs (512-byte row pieces) wherever the width allows
  const int slab = C % 128 == 0 ? 128 : 64;
  if (group_tokens <= kRegGroupMax && C % slab == 0 && aligned16(packed_out) &&
      (e = tma_quant_setup(&sms)) == cudaSuccess &&
      (e = encode_rows_map(&tmap, kv, num_tokens, (int)C, slab, group_tokens)) == cudaSuccess) {
    const long long tiles = (long long)groups * (C / slab);
    const long long slots = (long long)sms * (slab == 64 ? TmaShape<64>::kCtasPerSm
                                                         : TmaShape<128>::kCtasPerSm);
    const unsigned pgrid = (unsigned)(tiles < slots ? tiles : slots);
    if (slab == 128)
      grouped_quant_tma_kernel<128><<<pgrid, kTmaThreads, sizeof(TmaSmem<128>), stream>>>(
          tmap, kv, num_tokens, (int)C, group_tokens, oc);
    else
      grouped_quant_tma_kernel<64><<<pgrid, kTmaThreads, sizeof(TmaSmem<64>), stream>>>(
          tmap, kv, num_tokens, (int)C, group_tokens, oc);
  } else if (e != cudaSuccess) {
    return e;
  } else if (group_tokens <= kRegGroupMax) {
    grouped_quant_kernel<false><<<grid, kQuantThreads, 0, stream>>>(kv, num_tokens, (int)C,
                                                                     group_tokens, oc, OutPaged{});
  } else {
    grouped_quant_loop_kernel<<<grid, kQuantThreads, 0, stream>>>(kv, num_tokens, (int)C,
                                                                  group_tokens, oc);
  }
  return cudaGetLastError();
}

cudaError_t int4kv_cache_write_ex(const float* k, const float* v, const int32_t* tok_offsets,
                                  const int32_t* start_pos, int batch, int max_rows_per_seq,
                                  int num_heads, int head_dim, int group_tokens, int page_tokens,
                                  const int32_t* block_table, int max_pages, int num_pages,
                                  uint8_t* k_pool, void* v_pool, int value_dtype, float* sz_pool,
                                  uint32_t* status, cudaStream_t stream) {
  if (batch <= 0 || max_rows_per_seq < 0 || num_heads <= 0 || head_dim <= 0) return cudaErrorInvalidValue;
  if (head_dim % 4 != 0 || page_tokens <= 0 || group_tokens <= 0) return cudaErrorInvalidValue;
  if (group_tokens % page_tokens != 0 || group_tokens > kRegGroupMax) return cudaErrorInvalidValue;
  if (value_dtype != INT4KV_VALUES_F32 && value_dtype != INT4KV_VALUES_F16 &&
      value_dtype != INT4KV_VALUES_BF16)
    return cudaErrorInvalidValue;
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
              num_heads, head_dim, k_pool, v_pool, value_dtype, sz_pool, status};
  grouped_quant_kernel<true><<<grid, kQuantThreads, 0, stream>>>(k, max_rows_per_seq, (int)C,
                                                                  group_tokens, OutContig{}, op);
  return cudaGetLastError();
}

cudaError_t int4kv_rope(const float* x, const int32_t* positions, int rows, int num_heads,
                        int head_dim, const float* rope_cos, const float* rope_sin,
                        int rope_positions, float* out, uint32_t* status, cudaStream_t stream) {
  if (rows < 0 || num_heads <= 0 || head_dim <= 0 || head_dim % 8 != 0 || rope_positions <= 0)
    return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  if (!x || !positions || !rope_cos || !rope_sin || !out) return cudaErrorInvalidValue;
  if (!aligned16(x) || !aligned16(out) || !aligned16(rope_cos) || !aligned16(rope_sin))
    return cudaErrorInvalidValue;
  {  // each output channel reads its partner channel of x: no overlap at all
    const char *xb = reinterpret_cast<const char*>(x), *ob = reinterpret_cast<const char*>(out);
    const size_t n = (size_t)rows * num_heads * head_dim * 4;
    if (xb < ob + n && ob < xb + n) return cudaErrorInvalidValue;
  }
  const long long total4 = (long long)rows * num_heads * head_dim / 4;
  const long long blocks = (total4 + 255) / 256;
  const unsigned grid = (unsigned)(blocks < 148 * 16 ? blocks : 148 * 16);
  rope_rows_kernel<<<grid, 256, 0, stream>>>(x, positions, rows, num_heads, head_dim, rope_cos,
                                             rope_sin, rope_positions, out, status);
  return cudaGetLastError();
}

cudaError_t int4kv_cache_append_rope(const float* k_new, const float* v_new,
                                     const int32_t* positions, const int32_t* stage_slots,
                                     float* k_stage, int num_slots, int batch, int num_heads,
                                     int head_dim, int group_tokens, int page_tokens,
                                     const int32_t* block_table, int max_pages, int num_pages,
                                     uint8_t* k_pool, void* v_pool, int value_dtype, float* sz_pool,
                                     const float* rope_cos, const float* rope_sin,
                                     int rope_positions, const float* q_in, float* q_out,
                                     int num_q_heads, uint32_t* status, cudaStream_t stream) {
  if (batch <= 0 || batch > 65535 || num_heads <= 0 || head_dim <= 0 || num_slots <= 0)
    return cudaErrorInvalidValue;
  if (head_dim % 4 != 0 || page_tokens <= 0 || group_tokens <= 0) return cudaErrorInvalidValue;
  if (group_tokens % page_tokens != 0 || group_tokens > kRegGroupMax) return cudaErrorInvalidValue;
  if (value_dtype != INT4KV_VALUES_F32 && value_dtype != INT4KV_VALUES_F16 &&
      value_dtype != INT4KV_VALUES_BF16)
    return cudaErrorInvalidValue;
  if (!k_new || !positions || !stage_slots || !k_stage || !block_table || !k_pool || !sz_pool)
    return cudaErrorInvalidValue;
  if (!aligned16(k_new) || !aligned16(k_stage)) return cudaErrorInvalidValue;
  if (v_new && (!v_pool || !aligned16(v_new) || !aligned16(v_pool))) return cudaErrorInvalidValue;
  if (max_pages <= 0 || num_pages <= 0) return cudaErrorInvalidValue;
  if ((rope_cos != nullptr) != (rope_sin != nullptr)) return cudaErrorInvalidValue;
  if (rope_cos && (head_dim % 8 != 0 || rope_positions <= 0 || !aligned16(rope_cos) ||
                   !aligned16(rope_sin)))
    return cudaErrorInvalidValue;
  if (q_in && (!q_out || num_q_heads <= 0 || !aligned16(q_in) || !aligned16(q_out)))
    return cudaErrorInvalidValue;
  const long long C = (long long)num_heads * head_dim;
  if (C > (1 << 30) || (q_in && (long long)num_q_heads * head_dim > (1 << 30))) return cudaErrorInvalidValue;
  dim3 grid((unsigned)((C + kSlab - 1) / kSlab), batch, 1);
  AppendArgs ap{k_new, v_new, positions, stage_slots, k_stage, num_slots,
                rope_cos, rope_sin, rope_positions, q_in, q_out, q_in ? num_q_heads : 0};
  OutPaged op{nullptr, nullptr, nullptr, block_table, max_pages, page_tokens, num_pages,
              num_heads, head_dim, k_pool, v_pool, value_dtype, sz_pool, status};
  append_quant_kernel<<<grid, kQuantThreads, 0, stream>>>(ap, (int)C, group_tokens, op);
  return cudaGetLastError();
}

cudaError_t int4kv_cache_append(const float* k_new, const float* v_new, const int32_t* positions,
                                const int32_t* stage_slots, float* k_stage, int num_slots,
                                int batch, int num_heads, int head_dim, int group_tokens,
                                int page_tokens, const int32_t* block_table, int max_pages,
                                int num_pages, uint8_t* k_pool, void* v_pool, int value_dtype,
                                float* sz_pool, uint32_t* status, cudaStream_t stream) {
  return int4kv_cache_append_rope(k_new, v_new, positions, stage_slots, k_stage, num_slots, batch,
                                  num_heads, head_dim, group_tokens, page_tokens, block_table,
                                  max_pages, num_pages, k_pool, v_pool, value_dtype, sz_pool,
                                  nullptr, nullptr, 0, nullptr, nullptr, 0, status, stream);
}

cudaError_t int4kv_cache_write(const float* k, const float* v, const int32_t* tok_offsets,
                               const int32_t* start_pos, int batch, int max_rows_per_seq,
                               int num_heads, int head_dim, int group_tokens, int page_tokens,
                               const int32_t* block_table, int max_pages, int num_pages,
                               uint8_t* k_pool, float* v_pool, float* sz_pool, uint32_t* status,
                               cudaStream_t stream) {
  return int4kv_cache_write_ex(k, v, tok_offsets, start_pos, batch, max_rows_per_seq, num_heads,
                               head_dim, group_tokens, page_tokens, block_table, max_pages,
                               num_pages, k_pool, v_pool, INT4KV_VALUES_F32, sz_pool, status,
                               stream);
}

}  // extern "C"
