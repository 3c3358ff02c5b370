// INT4 flash-decode over ONE shared page stream (the reference's
// cu_flash_decode_int4 contract, csrc/flash_decode_int4.cu:104-284): every
// query of [batch, heads] attends to the same list of pages, each page
// [block_size, head_dim] with one code per byte (or two, in the vLLM-style
// block cache), its own per-channel scale / zero-point and a valid-row count.
// Any head_dim in [1, 256], any page size. No softmax scale.
//
// With all queries on one stream the work is attention-shaped, not GEMV-shaped:
// every staged key / value byte serves a tile of queries. B200 mapping:
//
//   * Grid: query tiles x S stream ranges; the S CTAs of one query tile form a
//     thread-block cluster (S <= 16: the non-portable size where the GPU can
//     schedule it, else 8). Each CTA runs an online softmax over its
//     contiguous range of 16-row page tiles; the S partial (m, l, acc) states
//     are merged through distributed shared memory at the end -- split-KV with
//     no workspace and no second launch.
//   * Staging: 64-row chunks of keys and values, double-buffered in shared
//     memory with 16-byte asynchronous copies (cp.async) into padded rows.
//   * Logits on the tensor cores, exactly: q_d * s_d (exact in float64) is put
//     in fixed point against the query's largest magnitude 2^E and split into
//     eight base-128 digits; one mma.m16n8k32 (u8 codes x s8 digits, int32
//     sums) per digit and 32 channels gives a 16-token x 8-query tile of
//     code x digit sums, recombined in float64 with weights 2^(E-7-7j). The
//     key is thereby dequantized as c*s - zp*s without rounding; the bias
//     sum_d q_d zp_d s_d is a float64 sum.
//   * Softmax: float64 running max per query, float32 weights (ex2 of the
//     float64 difference), Kahan-compensated float32 sums.
//   * P.V in float32 FMAs: each thread owns 2 queries x 4 channels.
//   * QT x DP = 2048 (queries per CTA x padded head dim): 16 queries at d128;
//     eight warps, and under 114 KB of shared memory up to d128 so that two
//     CTAs share an SM.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"
#include "../../include/int4kv_b200.h"

namespace cg = cooperative_groups;
using namespace i4kv;

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kChunk = 64;     // staged rows per chunk: four 16-row MMA tiles
constexpr int kDig = 8;        // base-128 digits of the fixed-point q * s
constexpr int kMaxSplit = 16;  // cluster size: 16 where the GPU allows it (non-portable), else 8
constexpr int kMaxD = 256;
constexpr uint32_t kFull = 0xffffffffu;

struct DenseArgs {
  const float* q;      // [nq, D]
  const uint8_t* kq;   // [num_blocks, bs, RB]: RB = D (one code per byte) or ceil(D/2)
  const float* ks;     // [num_blocks, D]
  const float* kz;     // [num_blocks, D]
  const void* v;       // [num_blocks, bs, D] of the value type
  const int* lens;     // [num_blocks] valid rows per block (clamped to [0, bs])
  const int* ids;      // nullable: stream page pi is storage block ids[pi]
  int nq, D, np, bs, num_blocks;  // np: pages in the stream
  float* out;          // [nq, D]
};

template <int DP, bool PACKED, int VK>
struct DCfg {
  static constexpr int QT = 2048 / DP;                     // queries per CTA
  static constexpr int NOCT = QT / 8;                      // 8-query MMA column blocks
  static constexpr int KK = DP / 32;                       // 32-position k-steps of a digit row
  static constexpr int VB = VK == 0 ? 4 : 2;               // stored value bytes
  // Staged key rows and digit rows are padded by 16 bytes: a row stride of
  // 4 x (odd) words puts the eight rows an ldmatrix / B-operand load touches
  // on distinct banks.
  static constexpr int KROW = (PACKED ? DP / 2 : DP) + 16;
  static constexpr int DROW = DP + 16;
  static constexpr int QP = QT / 2;                        // P.V: query pairs
  static constexpr int DG = DP / 4;                        // P.V: channel groups of 4
  static_assert(QP * DG == kThreads, "P.V: one (2 queries x 4 channels) block per thread");
  static constexpr int PROW = kChunk + 1;                  // weights [QT][PROW]: conflict-free
  // shared-memory layout (bytes); the chunk's weights overwrite its logits
  static constexpr size_t OFF_DIG = 0;                                    // u8 [kDig][QT][DROW]
  static constexpr size_t OFF_K = OFF_DIG + (size_t)kDig * QT * DROW;     // u8 [2][kChunk][KROW]
  static constexpr size_t OFF_V = OFF_K + (size_t)2 * kChunk * KROW;      // [2][kChunk][DP] values
  static constexpr size_t OFF_LG = OFF_V + (size_t)2 * kChunk * DP * VB;  // double [QT][kChunk]
  static constexpr size_t OFF_P = OFF_LG;                                 // float [QT][PROW]
  static_assert((size_t)QT * PROW * 4 <= (size_t)QT * kChunk * 8, "weights fit over the logits");
  static constexpr size_t OFF_BIAS = OFF_LG + (size_t)QT * kChunk * 8;    // double [QT]
  static constexpr size_t OFF_M = OFF_BIAS + (size_t)QT * 8;              // double [QT]
  static constexpr size_t OFF_W = OFF_M + (size_t)QT * 8;                 // double [QT][kMaxSplit]
  static constexpr size_t OFF_L = OFF_W + (size_t)QT * kMaxSplit * 8;     // float [QT] (l), [QT] (c)
  static constexpr size_t OFF_E = OFF_L + (size_t)QT * 8;                 // int [QT]
  static constexpr size_t OFF_CORR = OFF_E + (size_t)QT * 4;              // float [QT]
  static constexpr size_t OFF_LL = OFF_CORR + (size_t)QT * 4;             // double [QT] (merged L)
  static constexpr size_t SMEM = OFF_LL + (size_t)QT * 8;
  // the merge reuses the value stages for acc [QT][DP] float
  static_assert((size_t)QT * DP * 4 <= (size_t)2 * kChunk * DP * VB, "acc fits the value stages");
  static_assert(OFF_DIG % 16 == 0 && OFF_K % 16 == 0 && OFF_V % 16 == 0 && OFF_LG % 16 == 0 &&
                    OFF_P % 16 == 0,
                "alignment");
};

template <int VK>
__device__ __forceinline__ float4 load_v4(const char* p) {
  if constexpr (VK == 0) {
    return *reinterpret_cast<const float4*>(p);
  } else {
    const uint2 w = *reinterpret_cast<const uint2*>(p);
    if constexpr (VK == 1) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
      return make_float4(a.x, a.y, b.x, b.y);
    } else {
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
      return make_float4(a.x, a.y, b.x, b.y);
    }
  }
}

// One chunk of the CTA's range: rows [row0, row0 + rows) of stream page pi
// (storage block pg), rows > 0.
struct Chunk {
  int pi, pg, row0, rows;
};

// The next non-empty chunk at or after tile `cur` (tiles of 16 rows, tpp per
// page) and before `end`; advances `cur` past it. Uniform across the CTA.
__device__ __forceinline__ bool next_chunk(const DenseArgs& a, int tpp, int& cur, int end,
                                           Chunk& c) {
  while (cur < end) {
    const int pi = cur / tpp;
    const int i = cur - pi * tpp;
    const int nt = min(min(4, tpp - i), end - cur);
    cur += nt;
    const int pg = a.ids ? __ldg(a.ids + pi) : pi;
    if (pg < 0 || pg >= a.num_blocks) continue;  // unknown block id: skipped, never read
    const int len = min(max(__ldg(a.lens + pg), 0), a.bs);
    const int row0 = 16 * i;
    const int rows = min(16 * nt, len - row0);
    if (rows <= 0) continue;
    c = Chunk{pi, pg, row0, rows};
    return true;
  }
  return false;
}

// Stage the codes and values of chunk c into buffer `buf` (asynchronous when
// every row starts on a 16-byte boundary, else plain loads).
template <int DP, bool PACKED, int VK>
__device__ __forceinline__ void load_chunk(const DenseArgs& a, const Chunk& c, char* smem, int buf,
                                           bool aligned) {
  using Cf = DCfg<DP, PACKED, VK>;
  const int RB = PACKED ? (a.D + 1) / 2 : a.D;
  uint8_t* sk = reinterpret_cast<uint8_t*>(smem + Cf::OFF_K) + (size_t)buf * kChunk * Cf::KROW;
  char* sv = smem + Cf::OFF_V + (size_t)buf * kChunk * DP * Cf::VB;
  const uint8_t* gk = a.kq + ((size_t)c.pg * a.bs + c.row0) * RB;
  const char* gv = static_cast<const char*>(a.v) + ((size_t)c.pg * a.bs + c.row0) * a.D * Cf::VB;
  const int vrow = a.D * Cf::VB;
  if (aligned && a.D == DP) {  // full rows: 16-byte pieces per row known at compile time
    constexpr int KP = (PACKED ? DP / 2 : DP) / 16, VP = DP * Cf::VB / 16;
    for (int i = threadIdx.x; i < c.rows * KP; i += kThreads) {
      const int r = i / KP, j = i - r * KP;
      cp_async16(sk + r * Cf::KROW + 16 * j, gk + (size_t)r * (KP * 16) + 16 * j);
    }
    for (int i = threadIdx.x; i < c.rows * VP; i += kThreads) {
      const int r = i / VP, j = i - r * VP;
      cp_async16(sv + (size_t)r * DP * Cf::VB + 16 * j, gv + (size_t)r * (VP * 16) + 16 * j);
    }
  } else if (aligned) {
    const int kp = RB / 16, vp = vrow / 16;
    for (int i = threadIdx.x; i < c.rows * kp; i += kThreads) {
      const int r = i / kp, j = i - r * kp;
      cp_async16(sk + r * Cf::KROW + 16 * j, gk + (size_t)r * RB + 16 * j);
    }
    for (int i = threadIdx.x; i < c.rows * vp; i += kThreads) {
      const int r = i / vp, j = i - r * vp;
      cp_async16(sv + (size_t)r * DP * Cf::VB + 16 * j, gv + (size_t)r * vrow + 16 * j);
    }
  } else {
    for (int i = threadIdx.x; i < c.rows * RB; i += kThreads) {
      const int r = i / RB, j = i - r * RB;
      sk[r * Cf::KROW + j] = __ldg(gk + (size_t)r * RB + j);
    }
    for (int i = threadIdx.x; i < c.rows * a.D; i += kThreads) {
      const int r = i / a.D, d = i - r * a.D;
      if constexpr (Cf::VB == 4) {
        reinterpret_cast<float*>(sv)[(size_t)r * DP + d] =
            __ldg(reinterpret_cast<const float*>(gv) + (size_t)r * a.D + d);
      } else {
        reinterpret_cast<uint16_t*>(sv)[(size_t)r * DP + d] =
            __ldg(reinterpret_cast<const unsigned short*>(gv) + (size_t)r * a.D + d);
      }
    }
  }
}

// Position of channel d in a digit row: d itself for one code per byte; for
// packed codes the even channels of each 64-channel block come first, then the
// odd ones (the low / high nibbles of the block's 32 key bytes).
template <bool PACKED>
__device__ __forceinline__ int dig_pos(int d) {
  if constexpr (PACKED) return (d & ~63) | ((d & 1) << 5) | ((d & 63) >> 1);
  else return d;
}

// Fixed-point digits and bias of the CTA's queries (q0 ..) against page pg's
// scales: each thread takes 8 channels of one query.
template <int DP, bool PACKED, int VK>
__device__ __forceinline__ void page_digits(const DenseArgs& a, int q0, int pg, char* smem) {
  using Cf = DCfg<DP, PACKED, VK>;
  constexpr int TPQ = kThreads / Cf::QT;  // threads per query (a power of two <= 32)
  static_assert(TPQ * 8 == DP, "8 channels per thread");
  uint8_t* sdig = reinterpret_cast<uint8_t*>(smem + Cf::OFF_DIG);
  const int q = threadIdx.x / TPQ;
  const int d0 = (threadIdx.x % TPQ) * 8;
  const bool qok = q0 + q < a.nq;
  const float* qrow = a.q + (size_t)(q0 + q) * a.D;
  double qs[8];
  double amax = 0.0, bsum = 0.0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int d = d0 + k;
    double x = 0.0;
    if (qok && d < a.D) {
      const double qd = (double)__ldg(qrow + d);
      const double sd = (double)__ldg(a.ks + (size_t)pg * a.D + d);
      x = qd * sd;  // exact: a product of two float32 values
      bsum = fma(qd, (double)__ldg(a.kz + (size_t)pg * a.D + d) * sd, bsum);
    }
    qs[k] = x;
    amax = fmax(amax, fabs(x));
  }
  int bexp = amax > 0.0 ? ((__double2hiint(amax) >> 20) & 0x7FF) : 0;
#pragma unroll
  for (int o = TPQ / 2; o > 0; o >>= 1) {
    bexp = max(bexp, __shfl_xor_sync(kFull, bexp, o));
    bsum += __shfl_xor_sync(kFull, bsum, o);
  }
  // |q*s| < 2^E; float32 products lie in [2^-298, 2^256], so every power of
  // two used here and in the recombination is a normal double
  const int E = bexp > 0 ? bexp - 1022 : 0;
  if (threadIdx.x % TPQ == 0) {
    reinterpret_cast<double*>(smem + Cf::OFF_BIAS)[q] = bsum;
    reinterpret_cast<int*>(smem + Cf::OFF_E)[q] = E;
  }
  const double scale = __hiloint2double((1023 + 56 - E) << 20, 0);
  long long X[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) X[k] = __double2ll_rn(qs[k] * scale);  // |X| < 2^56
#pragma unroll
  for (int j = 0; j < kDig; ++j) {  // digit j: bits [49 - 7j, 56 - 7j) of X, the top one signed
    const int sh = 49 - 7 * j;
    const long long m = j == 0 ? 0xFF : 0x7F;
    uint8_t* row = sdig + ((size_t)j * Cf::QT + q) * Cf::DROW;
    const uint32_t w0 = (uint32_t)(((X[0] >> sh) & m) | (((X[1] >> sh) & m) << 8) |
                                   (((X[2] >> sh) & m) << 16) | (((X[3] >> sh) & m) << 24));
    const uint32_t w1 = (uint32_t)(((X[4] >> sh) & m) | (((X[5] >> sh) & m) << 8) |
                                   (((X[6] >> sh) & m) << 16) | (((X[7] >> sh) & m) << 24));
    if constexpr (PACKED) {
      // even channels d0, d0+2, .., d0+6 and the odd ones: 4 bytes each
      *reinterpret_cast<uint32_t*>(row + dig_pos<true>(d0)) = __byte_perm(w0, w1, 0x6420);
      *reinterpret_cast<uint32_t*>(row + dig_pos<true>(d0 + 1)) = __byte_perm(w0, w1, 0x7531);
    } else {
      *reinterpret_cast<uint2*>(row + d0) = make_uint2(w0, w1);
    }
  }
}

template <int DP, bool PACKED, int VK>
__global__ void __launch_bounds__(kThreads)
shared_stream_decode_kernel(DenseArgs a) {
  using Cf = DCfg<DP, PACKED, VK>;
  constexpr int QT = Cf::QT;
  // launched with programmatic stream serialization: wait for the previous
  // kernel on the stream (its completion and memory) before anything else
  grid_dependency_wait();
  extern __shared__ __align__(128) char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const int q0 = (blockIdx.x / S) * QT;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;

  double* s_lg = reinterpret_cast<double*>(smem + Cf::OFF_LG);
  float* s_p = reinterpret_cast<float*>(smem + Cf::OFF_P);
  double* s_bias = reinterpret_cast<double*>(smem + Cf::OFF_BIAS);
  double* s_m = reinterpret_cast<double*>(smem + Cf::OFF_M);
  float* s_l = reinterpret_cast<float*>(smem + Cf::OFF_L);
  float* s_lc = s_l + QT;
  int* s_E = reinterpret_cast<int*>(smem + Cf::OFF_E);
  float* s_corr = reinterpret_cast<float*>(smem + Cf::OFF_CORR);
  const uint8_t* sdig = reinterpret_cast<const uint8_t*>(smem + Cf::OFF_DIG);

  for (int i = threadIdx.x; i < QT; i += kThreads) {
    s_m[i] = -INFINITY;
    s_l[i] = 0.f;
    s_lc[i] = 0.f;
  }

  // this CTA's contiguous range of 16-row tiles of the stream
  const int tpp = (a.bs + 15) / 16;
  const int total = a.np * tpp;  // < 2^31 (checked on the host)
  int cur = (int)((long long)total * rank / S);
  const int end = (int)((long long)total * (rank + 1) / S);
  const int RB = PACKED ? (a.D + 1) / 2 : a.D;
  const bool aligned = (RB % 16 == 0) && ((a.D * Cf::VB) % 16 == 0) &&
                       ((reinterpret_cast<uintptr_t>(a.kq) | reinterpret_cast<uintptr_t>(a.v)) & 15u) == 0;

  // P.V ownership: queries 2qp, 2qp+1 x channels 4dg .. 4dg+3
  const int qp = threadIdx.x % Cf::QP, dg = threadIdx.x / Cf::QP;
  float acc[2][4], acc_c[2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f, acc_c[i][j] = 0.f;

  Chunk c{}, nc{};
  bool have = next_chunk(a, tpp, cur, end, c);
  if (have) {
    load_chunk<DP, PACKED, VK>(a, c, smem, 0, aligned);
    cp_async_commit();
  }
  int dig_pg = -1;
  int buf = 0;
  __syncthreads();  // running state initialised
  while (have) {
    const bool more = next_chunk(a, tpp, cur, end, nc);
    if (more) load_chunk<DP, PACKED, VK>(a, nc, smem, buf ^ 1, aligned);
    cp_async_commit();
    if (c.pg != dig_pg) {  // new page: its scales into the query digits
      page_digits<DP, PACKED, VK>(a, q0, c.pg, smem);
      dig_pg = c.pg;
    }
    cp_async_wait<1>();  // this chunk's copies (the next chunk's may still fly)
    __syncthreads();

    // ---- logits: units (8-query block o, 16-row tile ti), one per warp at d128 ----
    const uint8_t* sk = reinterpret_cast<const uint8_t*>(smem + Cf::OFF_K) + (size_t)buf * kChunk * Cf::KROW;
    for (int u = warp; u < Cf::NOCT * 4; u += kWarps) {
      const int o = u >> 2, ti = u & 3;
      if (16 * ti >= c.rows) continue;  // warp-uniform
      uint32_t A[Cf::KK][4];
      const uint8_t* rowp = sk + (16 * ti + (lane & 7) + 8 * ((lane >> 3) & 1)) * Cf::KROW + 16 * (lane >> 4);
      if constexpr (PACKED) {
#pragma unroll
        for (int e = 0; e < Cf::KK / 2; ++e) {
          uint32_t r[4];
          ldmatrix_x4(r, rowp + 32 * e);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            A[2 * e][k] = r[k] & 0x0F0F0F0Fu;
            A[2 * e + 1][k] = (r[k] >> 4) & 0x0F0F0F0Fu;
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < Cf::KK; ++e) ldmatrix_x4(A[e], rowp + 32 * e);
      }
      // eight independent accumulator chains, one per digit
      int cs[kDig][4];
#pragma unroll
      for (int j = 0; j < kDig; ++j) cs[j][0] = cs[j][1] = cs[j][2] = cs[j][3] = 0;
      const uint8_t* dcol = sdig + (size_t)(8 * o + g) * Cf::DROW + 4 * t;
#pragma unroll
      for (int kk = 0; kk < Cf::KK; ++kk) {
#pragma unroll
        for (int j = 0; j < kDig; ++j) {
          const uint8_t* drow = dcol + (size_t)j * QT * Cf::DROW + 32 * kk;
          mma_u8s8_16832(cs[j], A[kk], *reinterpret_cast<const uint32_t*>(drow),
                         *reinterpret_cast<const uint32_t*>(drow + 16));
        }
      }
      const int qa = 8 * o + 2 * t, qb = qa + 1;
      double wa = __hiloint2double((1023 + s_E[qa] - 7) << 20, 0);
      double wb = __hiloint2double((1023 + s_E[qb] - 7) << 20, 0);
      double lg[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
      for (int j = 0; j < kDig; ++j) {
        lg[0] = fma((double)cs[j][0], wa, lg[0]);
        lg[1] = fma((double)cs[j][1], wb, lg[1]);
        lg[2] = fma((double)cs[j][2], wa, lg[2]);
        lg[3] = fma((double)cs[j][3], wb, lg[3]);
        wa *= 0.0078125;  // 2^-7: the next digit's weight (exact)
        wb *= 0.0078125;
      }
      const int r0 = 16 * ti + g, r1 = r0 + 8;
      s_lg[qa * kChunk + r0] = r0 < c.rows ? lg[0] - s_bias[qa] : -INFINITY;
      s_lg[qb * kChunk + r0] = r0 < c.rows ? lg[1] - s_bias[qb] : -INFINITY;
      s_lg[qa * kChunk + r1] = r1 < c.rows ? lg[2] - s_bias[qa] : -INFINITY;
      s_lg[qb * kChunk + r1] = r1 < c.rows ? lg[3] - s_bias[qb] : -INFINITY;
    }
    __syncthreads();

    // ---- online softmax over the chunk: lane covers rows lane, lane + 32 ----
    constexpr int QW = (QT + kWarps - 1) / kWarps;  // queries per warp
    double xs[QW][2];
#pragma unroll
    for (int k = 0; k < QW; ++k) {
      const int qi = warp + k * kWarps;
      xs[k][0] = (qi < QT && lane < c.rows) ? s_lg[qi * kChunk + lane] : -INFINITY;
      xs[k][1] = (qi < QT && lane + 32 < c.rows) ? s_lg[qi * kChunk + lane + 32] : -INFINITY;
    }
    __syncthreads();  // the weights overwrite the logits
#pragma unroll
    for (int k = 0; k < QW; ++k) {
      const int qi = warp + k * kWarps;
      if (qi >= QT) break;
      double mx = fmax(xs[k][0], xs[k][1]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmax(mx, __shfl_xor_sync(kFull, mx, off));
      const double m_old = s_m[qi];
      const double m_new = fmax(m_old, mx);
      float p0 = 0.f, p1 = 0.f, corr = 1.f;
      if (m_new != -INFINITY) {
        p0 = exp_neg(xs[k][0] - m_new);
        p1 = exp_neg(xs[k][1] - m_new);
        corr = exp_neg(m_old - m_new);  // 0 for the first live chunk (m_old = -inf)
      }
      s_p[qi * Cf::PROW + lane] = p0;
      s_p[qi * Cf::PROW + lane + 32] = p1;
      float ps = p0 + p1;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(kFull, ps, off);
      if (lane == 0) {
        float l = s_l[qi], lc = s_lc[qi];
        kahan_rescale_add(l, lc, corr, ps);
        s_l[qi] = l;
        s_lc[qi] = lc;
        s_m[qi] = m_new;
        s_corr[qi] = corr;
      }
    }
    __syncthreads();

    // ---- P.V: this thread's 2 queries x 4 channels ----
    {
      const char* vp = smem + Cf::OFF_V + (size_t)buf * kChunk * DP * Cf::VB + (size_t)(4 * dg) * Cf::VB;
      const float* pa = s_p + (2 * qp) * Cf::PROW;
      const float* pb = pa + Cf::PROW;
      float ch[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
      for (int r = 0; r < c.rows; ++r) {  // paired FMAs: bit-identical to fmaf per lane
        const float4 v4 = load_v4<VK>(vp + (size_t)r * DP * Cf::VB);
        const float x = pa[r], y = pb[r];
        fma2_rn(ch[0][0], ch[0][1], v4.x, v4.y, x);
        fma2_rn(ch[0][2], ch[0][3], v4.z, v4.w, x);
        fma2_rn(ch[1][0], ch[1][1], v4.x, v4.y, y);
        fma2_rn(ch[1][2], ch[1][3], v4.z, v4.w, y);
      }
      const float ca = s_corr[2 * qp], cb = s_corr[2 * qp + 1];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kahan_rescale_add(acc[0][j], acc_c[0][j], ca, ch[0][j]);
        kahan_rescale_add(acc[1][j], acc_c[1][j], cb, ch[1][j]);
      }
    }
    __syncthreads();  // the stage, digits and weights are free for the next chunk
    c = nc;
    have = more;
    buf ^= 1;
  }
  cp_async_wait<0>();

  allow_dependent_launch();  // a following launch may be dispatched during the merge
  // ---- merge the cluster's S partial states through distributed shared memory ----
  float* s_acc = reinterpret_cast<float*>(smem + Cf::OFF_V);  // [QT][DP], over the value stages
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 2; ++i)
    *reinterpret_cast<float4*>(s_acc + (2 * qp + i) * DP + 4 * dg) =
        make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  cluster.sync();  // every rank's (m, l, acc) is final and visible
  double* s_w = reinterpret_cast<double*>(smem + Cf::OFF_W);
  double* s_L = reinterpret_cast<double*>(smem + Cf::OFF_LL);
  for (int qi = threadIdx.x; qi < QT; qi += kThreads) {
    double M = -INFINITY;
    for (int r = 0; r < S; ++r) M = fmax(M, cluster.map_shared_rank(s_m, r)[qi]);
    double L = 0.0;
    for (int r = 0; r < S; ++r) {
      const double mr = cluster.map_shared_rank(s_m, r)[qi];
      const double w = mr == -INFINITY ? 0.0 : exp(mr - M);
      s_w[qi * kMaxSplit + r] = w;
      L = fma((double)cluster.map_shared_rank(s_l, r)[qi], w, L);
    }
    s_L[qi] = L;
  }
  __syncthreads();
  const int per = (QT * DP + S - 1) / S;  // (query, channel) outputs this rank finishes
  for (int i = threadIdx.x; i < per; i += kThreads) {
    const int idx = rank * per + i;
    if (idx >= QT * DP) break;
    const int qi = idx / DP, d = idx - qi * DP;
    if (q0 + qi >= a.nq || d >= a.D) continue;
    double o = 0.0;
    for (int r = 0; r < S; ++r)
      o = fma((double)cluster.map_shared_rank(s_acc, r)[qi * DP + d], s_w[qi * kMaxSplit + r], o);
    a.out[(size_t)(q0 + qi) * a.D + d] = (float)(o / fmax(s_L[qi], 1e-10));
  }
  cluster.sync();  // peers finished reading this CTA's shared memory
}

template <int DP, bool PACKED, int VK>
cudaError_t launch_shared(const DenseArgs& a, cudaStream_t stream) {
  using Cf = DCfg<DP, PACKED, VK>;
  static std::mutex mu;
  static int max_split[64] = {};  // per device: 16 when a 16-CTA cluster can be scheduled
  int dev = 0, sms = 148;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  auto kern = shared_stream_decode_kernel<DP, PACKED, VK>;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!max_split[dev]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cf::SMEM);
      if (e != cudaSuccess) return e;
      int ms = 8;
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
          cudaSuccess) {
        cudaLaunchConfig_t probe = {};
        probe.gridDim = dim3(16, 1, 1);
        probe.blockDim = dim3(kThreads, 1, 1);
        probe.dynamicSmemBytes = Cf::SMEM;
        cudaLaunchAttribute pa[1];
        pa[0].id = cudaLaunchAttributeClusterDimension;
        pa[0].val.clusterDim.x = 16;
        pa[0].val.clusterDim.y = 1;
        pa[0].val.clusterDim.z = 1;
        probe.attrs = pa;
        probe.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kern, &probe) == cudaSuccess && clusters >= 8)
          ms = 16;
      }
      (void)cudaGetLastError();  // a refused query leaves no error behind
      max_split[dev] = ms;
    }
  }
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int qtiles = (a.nq + Cf::QT - 1) / Cf::QT;
  const long long tiles = (long long)a.np * ((a.bs + 15) / 16);
  // enough stream ranges to give the GPU about two CTAs per SM, at most one
  // cluster per query tile and no more ranges than 16-row tiles. Clusters of
  // 16 only when each CTA still gets at least four 64-row chunks: measured at
  // 8 x 32 queries, 16 ranges took s8192 from 104 to 95 us and s32768 from 382
  // to 316 us, but s2048 from 35 to 41 us and s512 from 19 to 31 us.
  const int cap = tiles >= 16LL * 16 ? max_split[dev] : 8;
  int S = (2 * sms + qtiles - 1) / qtiles;
  S = (int)max(1LL, min((long long)min(S, cap), tiles));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(qtiles * S), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cf::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // programmatic dependent launch: dispatched while the previous kernel on
  // the stream finishes; the kernel's first instruction waits for it
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <bool PACKED, int VK>
cudaError_t dispatch_dp(const DenseArgs& a, cudaStream_t stream) {
  const int dp = PACKED ? ((a.D + 63) / 64) * 64 : ((a.D + 31) / 32) * 32;
  if constexpr (!PACKED) {
    if (dp <= 32) return launch_shared<32, PACKED, VK>(a, stream);
  }
  if (dp <= 64) return launch_shared<64, PACKED, VK>(a, stream);
  if (dp <= 128) return launch_shared<128, PACKED, VK>(a, stream);
  return launch_shared<256, PACKED, VK>(a, stream);
}

cudaError_t check(const float* query, const uint8_t* k_q, const float* k_scale, const float* k_zp,
                  const void* value, const int* block_lens, int batch_size, int num_heads,
                  int head_dim, int num_blocks, int block_size, const float* output) {
  if (head_dim <= 0 || head_dim > kMaxD) return cudaErrorInvalidValue;
  if (batch_size <= 0 || num_heads <= 0 || num_blocks < 0 || block_size < 0) return cudaErrorInvalidValue;
  if ((long long)batch_size * num_heads >= (1LL << 31) / kMaxD) return cudaErrorInvalidValue;
  if (!query || !output) return cudaErrorInvalidValue;
  if (num_blocks > 0 && (!k_q || !k_scale || !k_zp || !value || !block_lens)) return cudaErrorInvalidValue;
  return cudaSuccess;
}

cudaError_t run(const DenseArgs& a, bool packed, int value_dtype, cudaStream_t stream) {
  if ((long long)a.np * ((a.bs + 15) / 16) >= (1LL << 31)) return cudaErrorInvalidValue;
  if (a.np == 0 || a.bs == 0) {  // an empty stream: every output is 0 (reference: o / max(0, 1e-10))
    const cudaError_t e = cudaMemsetAsync(a.out, 0, (size_t)a.nq * a.D * sizeof(float), stream);
    return e != cudaSuccess ? e : cudaGetLastError();
  }
  if (!packed) return dispatch_dp<false, 0>(a, stream);
  switch (value_dtype) {
    case INT4KV_VALUES_F32: return dispatch_dp<true, 0>(a, stream);
    case INT4KV_VALUES_F16: return dispatch_dp<true, 1>(a, stream);
    default: return dispatch_dp<true, 2>(a, stream);
  }
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
  const DenseArgs a{query, k_q, k_scale, k_zp, value, block_lens, nullptr, batch_size * num_heads,
                    head_dim, num_blocks, block_size, num_blocks, output};
  return run(a, false, INT4KV_VALUES_F32, stream);
}

cudaError_t int4kv_dense_decode_workspace_size(int batch_size, int num_heads, int head_dim,
                                               int num_blocks, int block_size, size_t* bytes) {
  if (!bytes || head_dim <= 0 || head_dim > kMaxD || batch_size <= 0 || num_heads <= 0 ||
      num_blocks < 0 || block_size < 0)
    return cudaErrorInvalidValue;
  *bytes = 16;  // the split-KV merge runs in distributed shared memory: no workspace
  return cudaSuccess;
}

cudaError_t int4kv_dense_decode(const float* query, const uint8_t* k_q, const float* k_scale,
                                const float* k_zp, const float* value, const int* block_lens,
                                int batch_size, int num_heads, int head_dim, int num_blocks,
                                int block_size, float* output, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream) {
  (void)workspace;
  (void)workspace_bytes;
  return cu_flash_decode_int4(query, k_q, k_scale, k_zp, value, block_lens, batch_size, num_heads,
                              head_dim, num_blocks, block_size, output, stream);
}

cudaError_t int4kv_block_decode(const float* query, const uint8_t* k_packed, const float* k_scale,
                                const float* k_zp, const void* value, int value_dtype,
                                const int32_t* block_lens, const int32_t* block_ids,
                                int num_listed, int num_blocks, int batch_size, int num_heads,
                                int head_dim, int block_size, float* output, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream) {
  (void)workspace;
  (void)workspace_bytes;
  if ((!block_ids && num_listed > 0) || num_blocks < 0) return cudaErrorInvalidValue;
  cudaError_t e = check(query, k_packed, k_scale, k_zp, value, block_lens, batch_size, num_heads,
                        head_dim, num_listed, block_size, output);
  if (e != cudaSuccess) return e;
  if (value_dtype != INT4KV_VALUES_F32 && value_dtype != INT4KV_VALUES_F16 &&
      value_dtype != INT4KV_VALUES_BF16)
    return cudaErrorInvalidValue;
  const DenseArgs a{query, k_packed, k_scale, k_zp, value, block_lens, block_ids,
                    batch_size * num_heads, head_dim, num_listed, block_size, num_blocks, output};
  return run(a, true, value_dtype, stream);
}

const char* int4kv_build_info(void) {
  return "libint4kv_b200: sm_100a, IEEE float32 (no fast-math), built " __DATE__ " " __TIME__;
}

}  // extern "C"
