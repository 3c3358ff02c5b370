// Fused INT4 paged flash-decoding attention for sm_100a (CUDA cores; the op
// is HBM-bound GEMV work, so no tensor cores).
//
// Semantics: the reference's online softmax (src/flash_decode_ref.py:30-139),
// run once per (sequence b, kv head h) stream: raw logits q.k (no 1/sqrt(d)),
// keys dequantized as fl(fl(code*scale) - fl(zp*scale)) with the scale/zp of
// the key's 128-token group, output o / max(l, 1e-10).
//
// Work decomposition (stream-K over pages): the page-heads of all streams are
// laid end to end in (b, h, page) order -- T of them -- and the grid's NW warps
// each take one contiguous run of ~T/NW pages, so every warp moves the same
// number of bytes whatever the length distribution. A warp keeps its own
// online-softmax state and writes one (m, l, acc[D]) partial per stream
// segment it touched; a small combine kernel merges the partials of a stream.
//
// Data movement: each warp owns a ring of STAGES shared-memory slots and lane 0
// streams its pages into them with 1-D bulk async copies (cp.async.bulk, the
// TMA engine without a tensor map) completing on per-slot mbarriers: the 16
// valid-token rows of V (fp32) and of packed K, plus the group's scale/zp and
// the stream's query when they change. No multicast; the sources are this
// GPU's own pools.
//
// Numerics: keys are dequantized in float32 with exactly the oracle's
// roundings, then dotted with the query in float64, so logits are exact up to
// the reference's own key rounding; exponentials and the value accumulation
// are float32 with per-page rescaling. The result is at least as close to a
// float64 evaluation as the float32 reference is.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "../../include/int4kv_b200.h"

using namespace i4kv;

namespace {

constexpr int kPage = 16;
constexpr uint32_t kFull = 0xffffffffu;
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded mbarrier waits: 2 s of wall time

template <int D, int WARPS, int STAGES>
struct Cfg {
  static constexpr int LPT = D / 8;          // lanes per token in the logit phase (8 dims each)
  static constexpr int TPP = 32 / LPT;       // tokens per pass
  static constexpr int NJ = kPage / TPP;     // passes per page
  static constexpr int DPL = D / 32;         // value dims per lane in the P.V phase
  static constexpr int V_OFF = 0;
  static constexpr int K_OFF = kPage * D * 4;
  static constexpr int SZ_OFF = K_OFF + kPage * D / 2;
  static constexpr int Q_OFF = SZ_OFF + 2 * D * 4;
  static constexpr int STAGE_BYTES = Q_OFF + D * 4;
  static constexpr int WARP_BYTES = STAGES * STAGE_BYTES;
  static constexpr int REC_BYTES = 16 + 4 * D;
  static_assert(LPT * TPP == 32 && NJ * TPP == kPage, "lane mapping");
  static_assert(LPT == 2 * NJ, "reduce-scatter mapping needs LPT == 2*NJ");
  static_assert(STAGE_BYTES % 16 == 0, "stage alignment");
};

// Workspace layout shared by the decode and combine kernels.
//   [0, 16)              reserved
//   [16, 16 + pfx)       prefix[B+1]: exclusive prefix of pages-per-head over sequences
//   [rec_off, ...)       partial records, slot (warp + stream), REC_BYTES each
__host__ __device__ inline size_t pfx_bytes(int batch) { return ((size_t)(batch + 1) * 4 + 127) / 128 * 128; }
__host__ __device__ inline size_t rec_offset(int batch) { return 16 + pfx_bytes(batch) + 112; }

struct DecodeArgs {
  const float* q;
  const uint8_t* k_pool;
  const float* v_pool;
  const float* sz_pool;
  const int32_t* block_table;
  const int32_t* seq_lens;
  int batch, heads, max_pages, num_pages, group_pages;
  char* ws;
  uint32_t* status;
};

__device__ __forceinline__ void set_status(uint32_t* status, uint32_t bits) {
  if (status) atomicOr(status, bits);
}

// Exclusive prefix over sequences of pages-per-head, into s_pfx[0..B]; returns total.
__device__ int block_page_prefix(const DecodeArgs& a, int* s_pfx, int* s_tmp) {
  const int nthreads = blockDim.x;
  const int t = threadIdx.x;
  const int per = (a.batch + nthreads - 1) / nthreads;
  const int lo = min(a.batch, t * per), hi = min(a.batch, lo + per);
  const int cap = a.max_pages * kPage;
  int local = 0;
  for (int b = lo; b < hi; ++b) {
    int len = a.seq_lens[b];
    if (len < 0 || len > cap) {
      set_status(a.status, kStatusBadLength);
      len = len < 0 ? 0 : cap;
    }
    local += (len + kPage - 1) / kPage;
  }
  const int lane = t & 31, warp = t >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_tmp[warp] = incl;
  __syncthreads();
  int warp_base = 0;
  for (int w = 0; w < warp; ++w) warp_base += s_tmp[w];
  int run = warp_base + incl - local;
  for (int b = lo; b < hi; ++b) {
    s_pfx[b] = run;
    int len = a.seq_lens[b];
    len = len < 0 ? 0 : (len > cap ? cap : len);
    run += (len + kPage - 1) / kPage;
  }
  if (t == nthreads - 1) s_pfx[a.batch] = run;
  __syncthreads();
  return s_pfx[a.batch];
}

// Per-page descriptor, computed by one lane for one page of the warp's run.
struct Desc {
  int phys;   // physical page (valid when ntok > 0)
  int gphys;  // physical page holding the group's scale/zp (valid when has_sz)
  int meta;   // ntok | has_q << 8 | has_sz << 9
  int stream; // b * heads + h
};

__device__ __forceinline__ Desc make_desc(const DecodeArgs& a, const int* s_pfx, long long g,
                                          long long g0, long long g1) {
  Desc d{0, 0, 0, -1};
  if (g >= g1) return d;
  const long long gq = g / a.heads;
  int lo = 0, hi = a.batch - 1;  // last b with pfx[b] <= gq
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_pfx[mid] <= gq) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const int np = s_pfx[b + 1] - s_pfx[b];
  const long long rem = g - (long long)a.heads * s_pfx[b];
  const int h = (int)(rem / np);
  const int p = (int)(rem - (long long)h * np);
  int len = a.seq_lens[b];
  const int cap = a.max_pages * kPage;
  len = len < 0 ? 0 : (len > cap ? cap : len);
  const int ntok = min(kPage, len - p * kPage);
  const int32_t* row = a.block_table + (size_t)b * a.max_pages;
  const int phys = row[p];
  const int gphys = row[(p / a.group_pages) * a.group_pages];
  const bool first = (g == g0) || (p == 0);
  const bool grp = first || (p % a.group_pages) == 0;
  const bool gok = gphys >= 0 && gphys < a.num_pages;
  const bool pok = phys >= 0 && phys < a.num_pages;
  if (!gok || !pok) set_status(a.status, kStatusBadPage);
  d.phys = phys;
  d.gphys = gphys;
  d.meta = ((gok && pok) ? ntok : 0) | (first ? (1 << 8) : 0) | ((grp && gok) ? (1 << 9) : 0);
  d.stream = b * a.heads + h;
  return d;
}

__device__ __forceinline__ Desc shfl_desc(const Desc& d, int src) {
  Desc o;
  o.phys = __shfl_sync(kFull, d.phys, src);
  o.gphys = __shfl_sync(kFull, d.gphys, src);
  o.meta = __shfl_sync(kFull, d.meta, src);
  o.stream = __shfl_sync(kFull, d.stream, src);
  return o;
}

template <int D, int WARPS, int STAGES>
__device__ __forceinline__ void issue_page(const DecodeArgs& a, const Desc& d, char* slot,
                                           uint64_t* bar) {
  using C = Cfg<D, WARPS, STAGES>;
  const int ntok = d.meta & 0xff;
  const bool has_q = (d.meta >> 8) & 1, has_sz = (d.meta >> 9) & 1;
  const int h = d.stream % a.heads;
  uint32_t bytes = 0;
  if (ntok) bytes += (uint32_t)ntok * (D * 4 + D / 2);
  if (has_sz) bytes += 2 * D * 4;
  if (has_q) bytes += D * 4;
  fence_proxy_async_smem();
  mbar_arrive_expect_tx(bar, bytes);
  if (ntok) {
    const size_t ph = (size_t)d.phys * a.heads + h;
    bulk_g2s(slot + C::V_OFF, a.v_pool + ph * kPage * D, (uint32_t)ntok * D * 4, bar);
    bulk_g2s(slot + C::K_OFF, a.k_pool + ph * kPage * (D / 2), (uint32_t)ntok * (D / 2), bar);
  }
  if (has_sz) {
    bulk_g2s(slot + C::SZ_OFF, a.sz_pool + ((size_t)d.gphys * a.heads + h) * 2 * D, 2 * D * 4, bar);
  }
  if (has_q) bulk_g2s(slot + C::Q_OFF, a.q + (size_t)d.stream * D, D * 4, bar);
}

template <int D, int WARPS, int STAGES>
__global__ void __launch_bounds__(WARPS * 32)
paged_decode_kernel(DecodeArgs a) {
  using C = Cfg<D, WARPS, STAGES>;
  extern __shared__ __align__(128) char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);                 // WARPS*STAGES
  int* s_tmp = reinterpret_cast<int*>(smem + 8 * WARPS * STAGES);      // WARPS ints
  int* s_pfx = reinterpret_cast<int*>(smem + 256);                     // batch+1 ints
  char* stages = smem + 256 + pfx_bytes(a.batch);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = lane % C::LPT, tsub = lane / C::LPT;
  const int total_pages = block_page_prefix(a, s_pfx, s_tmp);
  if (blockIdx.x == 0) {
    int* g_pfx = reinterpret_cast<int*>(a.ws + 16);
    for (int i = threadIdx.x; i <= a.batch; i += blockDim.x) g_pfx[i] = s_pfx[i];
  }
  const long long T = (long long)a.heads * total_pages;
  const long long NW = (long long)gridDim.x * WARPS;
  const long long gw = (long long)blockIdx.x * WARPS + warp;
  const long long g0 = gw * T / NW, g1 = (gw + 1) * T / NW;
  const int n = (int)(g1 - g0);
  if (n <= 0) return;

  uint64_t* bar = bars + warp * STAGES;
  char* ring = stages + (size_t)warp * C::WARP_BYTES;
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) mbar_init(&bar[s], 1);
    fence_barrier_init();
  }
  __syncwarp();

  Desc cur = make_desc(a, s_pfx, g0 + lane, g0, g1);
  Desc nxt = make_desc(a, s_pfx, g0 + 32 + lane, g0, g1);
  // Prologue: the first STAGES pages (all inside chunk 0 since STAGES <= 32).
#pragma unroll
  for (int i = 0; i < STAGES; ++i) {
    const Desc d = shfl_desc(cur, i);
    if (lane == 0 && i < n) issue_page<D, WARPS, STAGES>(a, d, ring + i * C::STAGE_BYTES, &bar[i]);
  }

  double q64[8];
  float sc[8], ns[8], zs[8];
  float acc[C::DPL];
  double m_run = -INFINITY;
  float l_lane = 0.f;
  int seg_stream = -1;
  bool aborted = false;
  int abort_at = 0;
#pragma unroll
  for (int i = 0; i < C::DPL; ++i) acc[i] = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) { q64[i] = 0.0; sc[i] = 0.f; ns[i] = 0.f; zs[i] = 0.f; }

  char* recs = a.ws + rec_offset(a.batch);
  auto flush = [&](int stream) {
    float lsum = l_lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(kFull, lsum, o);
    char* rec = recs + (size_t)(gw + stream) * C::REC_BYTES;
    if (lane == 0) {
      *reinterpret_cast<double*>(rec) = m_run;
      *reinterpret_cast<float*>(rec + 8) = lsum;
    }
    float* racc = reinterpret_cast<float*>(rec + 16);
    if constexpr (C::DPL == 2) {
      *reinterpret_cast<float2*>(racc + 2 * lane) = make_float2(acc[0], acc[1]);
    } else {
#pragma unroll
      for (int v4 = 0; v4 < C::DPL / 4; ++v4)
        *reinterpret_cast<float4*>(racc + v4 * 128 + 4 * lane) =
            make_float4(acc[4 * v4], acc[4 * v4 + 1], acc[4 * v4 + 2], acc[4 * v4 + 3]);
    }
  };

  for (int i = 0; i < n; ++i) {
    if (i > 0 && (i & 31) == 0) {
      cur = nxt;
      nxt = make_desc(a, s_pfx, g0 + i + 32 + lane, g0, g1);
    }
    const int st = i % STAGES;
    char* slot = ring + st * C::STAGE_BYTES;
    const Desc d = shfl_desc(cur, i & 31);
    const int ntok = d.meta & 0xff;
    const bool has_q = (d.meta >> 8) & 1, has_sz = (d.meta >> 9) & 1;

    if (!mbar_wait_bounded(&bar[st], (uint32_t)((i / STAGES) & 1), kWaitNs)) {
      set_status(a.status, kStatusWaitTimeout);
      aborted = true;
      abort_at = i;
      break;
    }

    if (has_q) {
      if (seg_stream >= 0) flush(seg_stream);
      seg_stream = d.stream;
      m_run = -INFINITY;
      l_lane = 0.f;
#pragma unroll
      for (int k = 0; k < C::DPL; ++k) acc[k] = 0.f;
      const float4* qs = reinterpret_cast<const float4*>(slot + C::Q_OFF) + 2 * c;
      const float4 qa = qs[0], qb = qs[1];
      q64[0] = qa.x; q64[1] = qa.y; q64[2] = qa.z; q64[3] = qa.w;
      q64[4] = qb.x; q64[5] = qb.y; q64[6] = qb.z; q64[7] = qb.w;
    }
    if (has_sz) {
      const float4* ss = reinterpret_cast<const float4*>(slot + C::SZ_OFF) + 2 * c;
      const float4* zz = reinterpret_cast<const float4*>(slot + C::SZ_OFF + D * 4) + 2 * c;
      const float4 sa = ss[0], sb = ss[1], za = zz[0], zb = zz[1];
      const float s8[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
      const float z8[8] = {za.x, za.y, za.z, za.w, zb.x, zb.y, zb.z, zb.w};
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        sc[k] = s8[k];
        ns[k] = __fmul_rn(s8[k], -8388608.0f);  // exact: power-of-two scaling
        zs[k] = __fmul_rn(z8[k], s8[k]);        // the oracle's zp*scale
      }
    }

    if (ntok > 0) {
      // ---- logits: lane (c, tsub) dots dims [8c, 8c+8) of tokens j*TPP + tsub ----
      const uint32_t* kw = reinterpret_cast<const uint32_t*>(slot + C::K_OFF);
      double part[C::NJ];
#pragma unroll
      for (int j = 0; j < C::NJ; ++j) {
        const uint32_t w = kw[j * 32 + lane];
        const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
        double s = 0.0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const float k0 = __fsub_rn(__fmaf_rn(magic_from_byte(lo, b), sc[2 * b], ns[2 * b]), zs[2 * b]);
          const float k1 =
              __fsub_rn(__fmaf_rn(magic_from_byte(hi, b), sc[2 * b + 1], ns[2 * b + 1]), zs[2 * b + 1]);
          s = fma((double)k0, q64[2 * b], s);
          s = fma((double)k1, q64[2 * b + 1], s);
        }
        part[j] = s;
      }
      // reduce-scatter over the LPT lanes of a token group: lane c ends with token j = c >> 1
#pragma unroll
      for (int step = 0; (C::NJ >> step) > 1; ++step) {
        const int half = (C::NJ >> step) >> 1;
        const int mask = C::LPT >> (step + 1);
        const bool upper = (c & mask) != 0;
#pragma unroll
        for (int k = 0; k < half; ++k) {
          const double send = upper ? part[k] : part[k + half];
          const double keep = upper ? part[k + half] : part[k];
          part[k] = keep + __shfl_xor_sync(kFull, send, mask);
        }
      }
      double logit = part[0] + __shfl_xor_sync(kFull, part[0], 1);
      const int tok = (c >> 1) * C::TPP + tsub;
      if (tok >= ntok) logit = -INFINITY;

      // ---- online softmax update for the page ----
      double pmax = logit;
#pragma unroll
      for (int o = 16; o > 1; o >>= 1) pmax = fmax(pmax, __shfl_xor_sync(kFull, pmax, o));
      const double m_new = fmax(m_run, pmax);
      const float corr = expf((float)(m_run - m_new));
      const float p = expf((float)(logit - m_new));
      l_lane = l_lane * corr + (((c & 1) == 0) ? p : 0.f);
      m_run = m_new;
#pragma unroll
      for (int k = 0; k < C::DPL; ++k) acc[k] *= corr;

      // ---- P.V over the page's valid rows ----
      const float* vs = reinterpret_cast<const float*>(slot + C::V_OFF);
#pragma unroll
      for (int t = 0; t < kPage; ++t) {
        if (t < ntok) {
          const float pt = __shfl_sync(kFull, p, (t % C::TPP) * C::LPT + 2 * (t / C::TPP));
          if constexpr (C::DPL == 2) {
            const float2 v = *reinterpret_cast<const float2*>(vs + t * D + 2 * lane);
            acc[0] = fmaf(pt, v.x, acc[0]);
            acc[1] = fmaf(pt, v.y, acc[1]);
          } else {
#pragma unroll
            for (int v4 = 0; v4 < C::DPL / 4; ++v4) {
              const float4 v = *reinterpret_cast<const float4*>(vs + t * D + v4 * 128 + 4 * lane);
              acc[4 * v4 + 0] = fmaf(pt, v.x, acc[4 * v4 + 0]);
              acc[4 * v4 + 1] = fmaf(pt, v.y, acc[4 * v4 + 1]);
              acc[4 * v4 + 2] = fmaf(pt, v.z, acc[4 * v4 + 2]);
              acc[4 * v4 + 3] = fmaf(pt, v.w, acc[4 * v4 + 3]);
            }
          }
        }
      }
    }

    __syncwarp();
    const int nx = i + STAGES;
    if (nx < n) {
      const int src = nx & 31;
      const Desc dn = (nx >> 5) == (i >> 5) ? shfl_desc(cur, src) : shfl_desc(nxt, src);
      if (lane == 0) issue_page<D, WARPS, STAGES>(a, dn, slot, &bar[st]);
    }
  }

  if (aborted) {
    // Drain what this warp still has in flight (bounded) before leaving, so no
    // bulk copy lands in shared memory after the CTA has exited.
    for (int k = abort_at; k < n && k < abort_at + STAGES; ++k)
      (void)mbar_wait_bounded(&bar[k % STAGES], (uint32_t)((k / STAGES) & 1), kWaitNs);
    return;
  }
  if (seg_stream >= 0) flush(seg_stream);
}

// One warp per stream: merge the partial records written by the warps whose
// page runs overlap the stream; empty streams get exact zeros.
template <int D>
__global__ void __launch_bounds__(128)
combine_kernel(const char* __restrict__ ws, int batch, int heads, long long nw, float* __restrict__ out) {
  constexpr int REC = 16 + 4 * D;
  constexpr int DPL = D / 32;
  const int lane = threadIdx.x & 31;
  const long long s = (long long)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (s >= (long long)batch * heads) return;
  const int b = (int)(s / heads), h = (int)(s % heads);
  const int* pfx = reinterpret_cast<const int*>(ws + 16);
  const long long total = (long long)heads * pfx[batch];
  const int np = pfx[b + 1] - pfx[b];
  float o[DPL];
#pragma unroll
  for (int k = 0; k < DPL; ++k) o[k] = 0.f;
  float* dst = out + (size_t)s * D;
  if (np > 0 && total > 0) {
    const long long gs = (long long)heads * pfx[b] + (long long)h * np, ge = gs + np;
    const long long w_lo = ((gs + 1) * nw - 1) / total, w_hi = (ge * nw - 1) / total;
    const char* recs = ws + rec_offset(batch);
    double M = -INFINITY;
    for (long long w = w_lo + lane; w <= w_hi; w += 32)
      M = fmax(M, *reinterpret_cast<const double*>(recs + (size_t)(w + s) * REC));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmax(M, __shfl_xor_sync(kFull, M, off));
    float L = 0.f;
    if (M != -INFINITY) {
      for (long long w = w_lo; w <= w_hi; ++w) {
        const char* rec = recs + (size_t)(w + s) * REC;
        const double m = *reinterpret_cast<const double*>(rec);
        if (m == -INFINITY) continue;
        const float e = expf((float)(m - M));
        L = fmaf(*reinterpret_cast<const float*>(rec + 8), e, L);
        const float* ra = reinterpret_cast<const float*>(rec + 16);
        if constexpr (DPL == 2) {
          const float2 v = *reinterpret_cast<const float2*>(ra + 2 * lane);
          o[0] = fmaf(v.x, e, o[0]);
          o[1] = fmaf(v.y, e, o[1]);
        } else {
#pragma unroll
          for (int v4 = 0; v4 < DPL / 4; ++v4) {
            const float4 v = *reinterpret_cast<const float4*>(ra + v4 * 128 + 4 * lane);
            o[4 * v4 + 0] = fmaf(v.x, e, o[4 * v4 + 0]);
            o[4 * v4 + 1] = fmaf(v.y, e, o[4 * v4 + 1]);
            o[4 * v4 + 2] = fmaf(v.z, e, o[4 * v4 + 2]);
            o[4 * v4 + 3] = fmaf(v.w, e, o[4 * v4 + 3]);
          }
        }
      }
      const float den = fmaxf(L, 1e-10f);
#pragma unroll
      for (int k = 0; k < DPL; ++k) o[k] = __fdiv_rn(o[k], den);
    }
  }
  if constexpr (DPL == 2) {
    *reinterpret_cast<float2*>(dst + 2 * lane) = make_float2(o[0], o[1]);
  } else {
#pragma unroll
    for (int v4 = 0; v4 < DPL / 4; ++v4)
      *reinterpret_cast<float4*>(dst + v4 * 128 + 4 * lane) =
          make_float4(o[4 * v4], o[4 * v4 + 1], o[4 * v4 + 2], o[4 * v4 + 3]);
  }
}

// ---- host side ----
constexpr int kWarps = 4;
constexpr int kStages = 2;

template <int D>
size_t dyn_smem(int batch) {
  return 256 + pfx_bytes(batch) + (size_t)kWarps * Cfg<D, kWarps, kStages>::WARP_BYTES;
}

struct OccCache {
  std::mutex mu;
  int dev[16] = {};
  int d[16] = {};
  size_t smem[16] = {};
  int grid[16] = {};
  int n = 0;
};
OccCache g_occ;

template <int D>
cudaError_t decode_grid(int batch, int* grid_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const size_t smem = dyn_smem<D>(batch);
  {
    std::lock_guard<std::mutex> lk(g_occ.mu);
    for (int i = 0; i < g_occ.n; ++i)
      if (g_occ.dev[i] == dev && g_occ.d[i] == D && g_occ.smem[i] == smem) {
        *grid_out = g_occ.grid[i];
        return cudaSuccess;
      }
  }
  auto kern = paged_decode_kernel<D, kWarps, kStages>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0, sms = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kWarps * 32, smem);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  if (per_sm <= 0) return cudaErrorInvalidConfiguration;
  const int grid = per_sm * sms;
  {
    std::lock_guard<std::mutex> lk(g_occ.mu);
    if (g_occ.n < 16) {
      g_occ.dev[g_occ.n] = dev; g_occ.d[g_occ.n] = D; g_occ.smem[g_occ.n] = smem;
      g_occ.grid[g_occ.n] = grid; ++g_occ.n;
    }
  }
  *grid_out = grid;
  return cudaSuccess;
}

template <int D>
cudaError_t ws_size(int batch, int heads, size_t* out) {
  int grid = 0;
  cudaError_t e = decode_grid<D>(batch, &grid);
  if (e != cudaSuccess) return e;
  const size_t nrec = (size_t)grid * kWarps + (size_t)batch * heads;
  *out = rec_offset(batch) + nrec * Cfg<D, kWarps, kStages>::REC_BYTES;
  return cudaSuccess;
}

template <int D>
cudaError_t launch(const DecodeArgs& a, float* out, size_t ws_bytes, cudaStream_t stream,
                   cudaEvent_t ev_before, cudaEvent_t ev_after) {
  int grid = 0;
  cudaError_t e = decode_grid<D>(a.batch, &grid);
  if (e != cudaSuccess) return e;
  size_t need = 0;
  e = ws_size<D>(a.batch, a.heads, &need);
  if (e != cudaSuccess) return e;
  if (ws_bytes < need) return cudaErrorInvalidValue;
  if (ev_before && (e = cudaEventRecord(ev_before, stream)) != cudaSuccess) return e;
  paged_decode_kernel<D, kWarps, kStages><<<grid, kWarps * 32, dyn_smem<D>(a.batch), stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (ev_after && (e = cudaEventRecord(ev_after, stream)) != cudaSuccess) return e;
  const long long streams = (long long)a.batch * a.heads;
  combine_kernel<D><<<(unsigned)((streams + 3) / 4), 128, 0, stream>>>(a.ws, a.batch, a.heads,
                                                                      (long long)grid * kWarps, out);
  return cudaGetLastError();
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

cudaError_t int4kv_paged_decode_workspace_size(int batch, int num_q_heads, int num_kv_heads,
                                               int head_dim, size_t* bytes) {
  if (!bytes || batch <= 0 || num_kv_heads <= 0 || num_q_heads != num_kv_heads) return cudaErrorInvalidValue;
  if (batch > kMaxPagedBatch) return cudaErrorInvalidValue;
  switch (head_dim) {
    case 64: return ws_size<64>(batch, num_kv_heads, bytes);
    case 128: return ws_size<128>(batch, num_kv_heads, bytes);
    case 256: return ws_size<256>(batch, num_kv_heads, bytes);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t int4kv_paged_decode_profiled(const float* query, const uint8_t* k_pool,
                                         const float* v_pool, const float* sz_pool,
                                         const int32_t* block_table, const int32_t* seq_lens,
                                         int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                         int page_tokens, int group_tokens, int max_pages,
                                         int num_pages, float* out, void* workspace,
                                         size_t workspace_bytes, uint32_t* status,
                                         cudaStream_t stream, cudaEvent_t ev_before,
                                         cudaEvent_t ev_after) {
  if (batch <= 0 || batch > kMaxPagedBatch || num_kv_heads <= 0 || num_q_heads != num_kv_heads)
    return cudaErrorInvalidValue;
  if (page_tokens != kPage || group_tokens <= 0 || group_tokens % kPage != 0) return cudaErrorInvalidValue;
  if (max_pages <= 0 || num_pages <= 0) return cudaErrorInvalidValue;
  if ((long long)batch * num_kv_heads * max_pages >= (1LL << 31)) return cudaErrorInvalidValue;
  if (!query || !k_pool || !v_pool || !sz_pool || !block_table || !seq_lens || !out || !workspace)
    return cudaErrorInvalidValue;
  if (!al16(query) || !al16(k_pool) || !al16(v_pool) || !al16(sz_pool) || !al16(out) || !al16(workspace))
    return cudaErrorInvalidValue;
  DecodeArgs a{query, k_pool, v_pool, sz_pool, block_table, seq_lens, batch, num_kv_heads,
               max_pages, num_pages, group_tokens / kPage, static_cast<char*>(workspace), status};
  switch (head_dim) {
    case 64: return launch<64>(a, out, workspace_bytes, stream, ev_before, ev_after);
    case 128: return launch<128>(a, out, workspace_bytes, stream, ev_before, ev_after);
    case 256: return launch<256>(a, out, workspace_bytes, stream, ev_before, ev_after);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t int4kv_paged_decode(const float* query, const uint8_t* k_pool, const float* v_pool,
                                const float* sz_pool, const int32_t* block_table,
                                const int32_t* seq_lens, int batch, int num_q_heads,
                                int num_kv_heads, int head_dim, int page_tokens, int group_tokens,
                                int max_pages, int num_pages, float* out, void* workspace,
                                size_t workspace_bytes, uint32_t* status, cudaStream_t stream) {
  return int4kv_paged_decode_profiled(query, k_pool, v_pool, sz_pool, block_table, seq_lens, batch,
                                      num_q_heads, num_kv_heads, head_dim, page_tokens,
                                      group_tokens, max_pages, num_pages, out, workspace,
                                      workspace_bytes, status, stream, nullptr, nullptr);
}

}  // extern "C"
