// Fused INT4 paged flash-decoding attention for sm_100a. The op is HBM-bound
// GEMV work; the tensor cores serve only to cut instructions: each page's
// code x query sums are four int8 MMAs per warp (see Numerics).
//
// Semantics: the reference's online softmax (src/flash_decode_ref.py:30-139),
// run once per (sequence b, query head h) stream over the pages of kv head
// h / G, G = query heads / kv heads (G = 1 without GQA): raw logits q.k (no
// 1/sqrt(d)), keys dequantized as code*scale - zp*scale with the scale/zp of the key's
// 128-token group, output o / max(l, 1e-10); empty streams give exact zeros.
//
// Grouped queries (GQA): when 4 (or 2) divides G, each warp serves HW = 4 (2)
// query heads of one kv head: it stages, unpacks and reads each kv page once
// for them, the heads' logits coming from one set of code fragments. For odd
// G, ring groups: gs = gcd(G, WARPS) one-head warps share one ring of staged
// pages, so a kv page crosses HBM once for those gs queries, and each warp
// does its own query's logits, softmax and P.V on the page.
//
// Work decomposition (stream-K over pages): the page-heads of all page
// streams (b, kv-head group) are laid end to end -- T of them -- and the
// grid's NW ring groups each take one contiguous run of ~T/NW pages, so every
// group moves the same number of bytes whatever the length distribution. A
// warp keeps its own online-softmax state per stream segment. A stream covered
// by one run is finished by its warp; otherwise each contributing warp writes
// an (m, l, acc[D]) partial, bumps the stream's counter, and the warp that
// arrives last merges the partials and writes the output (counters reset to
// zero on the way out, so the workspace stays zero-filled between launches).
// A warp publishes its first segment's partial as soon as that segment ends
// (the other contributors reach that stream only at the ends of their runs)
// and its last segment's at the end of its run, so a warp has at most one
// merge to do when its run is over.
//
// Data movement: each ring group owns STAGES * gs shared-memory slots and one
// lane streams its pages into them with 1-D bulk async copies (cp.async.bulk,
// the TMA engine without a tensor map) completing on per-slot mbarriers: the
// valid rows of V and of packed K, plus the group's scale/zp and the gs
// queries when they change. Each copy has one destination CTA; the sources
// are this GPU's own pools.
//
// Numerics: with qs_d = q_d*s_d (exact in float64) and c_d the 4-bit code,
// the logit is sum_d qs_d*c_d - sum_d q_d*zp_d*s_d, i.e. the key dequantized
// exactly as c*s - zp*s. The first sum runs on the tensor cores in exact
// integer arithmetic: per (query, group) the qs_d are written in fixed point
// relative to their largest magnitude (56 bits, eight base-128 digits), one
// mma.m16n8k32 (u8 codes x s8 digits, int32 sums) per 32 bytes of packed key
// row and nibble half gives every token's code x digit sums, and float64
// weights recombine them. The truncation to 56 bits is finer than float64
// accumulation, so the logits are those of the reference's float64 arbiter
// to rounding; softmax weights are float32 exponentials, values are summed per
// page in float32 and across pages in float32 with Kahan compensation;
// partials are merged in float64.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "../../include/int4kv_b200.h"

using namespace i4kv;

namespace {

constexpr int kPage = 16;
constexpr int kXRanks = INT4KV_EXCHANGE_MAX_RANKS;
constexpr uint64_t kPeerWaitNs = 2000000000ull;  // bounded waits on other GPUs: 2 s

// Exchange buffer of the fused split decode, per rank, S query streams:
//   step u32 [S]                 steps this rank completed for each stream
//   flag u32 [2][kXRanks][S]     flag[parity][src][s] = step of rank src
//   recs     [2][kXRanks][S]     records pushed by rank src for that step
__host__ __device__ inline size_t x_align(size_t v) { return (v + 127) / 128 * 128; }
__host__ __device__ inline size_t x_off_flag(long long S) { return x_align((size_t)S * 4); }
__host__ __device__ inline size_t x_off_recs(long long S) {
  return x_off_flag(S) + x_align((size_t)2 * kXRanks * S * 4);
}
__host__ __device__ inline size_t x_bytes(long long S, int d) {
  return x_off_recs(S) + (size_t)2 * kXRanks * S * (16 + 4 * (size_t)d);
}
constexpr uint32_t kFull = 0xffffffffu;
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded mbarrier waits: 2 s of wall time

// P.V of a full page as two interleaved float32 sums (even / odd rows) in
// place of one.
#ifndef I4KV_PV_TWO_CHAINS
#define I4KV_PV_TWO_CHAINS 0
#endif

// Share of a warp pair's run each warp takes unasked, in eighths (the rest
// is claimed page by page), for float32 and for 16-bit value pools. Measured
// side by side on one B200 (float32): 3/8 against 2/8 and 0 (every page
// claimed) -- config 0 61.2 / 61.8 / 62.1 us, cfg2 L=512 29.1 / 29.2 / 30.0,
// cfg2 L=8192 193.6 / 194.1 / 194.5, cfg3 d64 757 / 767 / 804, cfg3 d128
// 1432 / 1429 / 1445; 16-bit values at config 0: 46.5 (3/8), 47.2 (2/8),
// 49.1 (0) -- a claim sits on the page's dependency chain.
#ifndef I4KV_PAIR_OWN_EIGHTHS_F32
#define I4KV_PAIR_OWN_EIGHTHS_F32 3
#endif
#ifndef I4KV_PAIR_OWN_EIGHTHS_16
#define I4KV_PAIR_OWN_EIGHTHS_16 3
#endif
// ... and for warps serving several query heads (either value kind).
// Measured side by side (GQA-4 at 32768 tokens, float32): 3/8 229.4 us,
// 2/8 233.5, 1/8 237.6; equal within noise at config 0's shape.
#ifndef I4KV_PAIR_OWN_EIGHTHS_MH
#define I4KV_PAIR_OWN_EIGHTHS_MH 3
#endif

// Programmatic dependent launch: the decode is launched with programmatic
// stream serialization, so its CTAs may become resident while the kernel
// before it on the stream is still running; every thread first waits for
// that kernel's completion and memory (griddepcontrol.wait, a no-op when the
// predecessor was not a kernel or the attribute is off), so nothing is read
// early. Each thread signals its own dependents after its page loop, so a
// following launch of this kernel can be dispatched while this one merges.
#ifndef I4KV_DECODE_PDL
#define I4KV_DECODE_PDL 1
#endif

// Minimum resident CTAs per SM the compiler plans registers for, for warps
// serving several query heads over 16-bit value pools.
#ifndef I4KV_MULTIHEAD16_MIN_CTAS
#define I4KV_MULTIHEAD16_MIN_CTAS 3
#endif

// Pages in flight per warp of a GQA ring group (the ring holds gs times this).
#ifndef I4KV_GQA_RING_PAGES_PER_WARP
#define I4KV_GQA_RING_PAGES_PER_WARP 1
#endif

// Value storage kinds (INT4KV_VALUES_*): 0 float32, 1 float16, 2 bfloat16.
template <int VK>
struct ValueKind {
  static constexpr int BYTES = VK == 0 ? 4 : 2;
};

template <int D, int WARPS, int STAGES, int VK = 0>
struct Cfg {
  static constexpr int VB = ValueKind<VK>::BYTES;  // bytes per stored value
  static constexpr int KT = D / 64;          // 32-byte k-tiles of a packed key row
  static constexpr int DPL = D / 32;         // value dims per lane in the P.V phase
  static constexpr int V_OFF = 0;
  static constexpr int K_OFF = kPage * D * VB;
  static constexpr int SZ_OFF = K_OFF + kPage * D / 2;
  static constexpr int Q_OFF = SZ_OFF + 2 * D * 4;
  static constexpr int STAGE_BYTES = Q_OFF + D * 4;  // one query (gs == 1)
  static constexpr int REC_BYTES = 16 + 4 * D;  // [m f64][l f64][acc D f32]
  static_assert(Q_OFF % 16 == 0 && STAGE_BYTES % 16 == 0, "stage alignment");
};

// Workspace layout (zero-filled before first use; every completed launch
// leaves the counters at zero again):
//   [0, cnt_bytes)            per-stream arrival counters, int32 [batch*heads]
//   [cnt_bytes, ...)          partial records, slot (warp + stream), REC_BYTES each
__host__ __device__ inline size_t cnt_bytes(long long streams) {
  return ((size_t)streams * 4 + 127) / 128 * 128;
}
__host__ __device__ inline size_t pfx_bytes(int batch) { return ((size_t)(batch + 1) * 4 + 127) / 128 * 128; }

struct DecodeArgs {
  const float* q;
  const uint8_t* k_pool;
  const void* v_pool;  // float32 / float16 / bfloat16 [pages, heads, 16, D]
  const float* sz_pool;
  const int32_t* block_table;
  const int32_t* seq_lens;
  float* out;
  int batch, heads, max_pages, num_pages, group_pages;
  char* ws;
  uint32_t* status;
  char* part_out;  // nullable: write per-stream partial records instead of outputs
  int kv_heads;    // heads of the pools; `heads` (query heads, one stream each) is a
  int group_q;     // multiple: query head h reads kv head h / group_q (GQA)
  int gs;          // warps sharing one ring
  int hw;          // query heads per warp (the kernel's HW); gs * hw heads share a staged page
  int vheads;      // heads / (gs * hw): the page streams of the work decomposition
  // Fused sequence-split exchange (xworld > 0): every stream's GPU-local
  // (m, l, acc) goes to every rank's exchange buffer, and the final output is
  // the merge of all ranks' records. xbuf[r] = rank r's buffer as mapped here.
  int xworld, xrank;
  char* xbuf[kXRanks];
};


__device__ __forceinline__ void set_status(uint32_t* status, uint32_t bits) {
  if (status) atomicOr(status, bits);
}

__device__ __forceinline__ int clamp_len(int len, int cap) { return len < 0 ? 0 : (len > cap ? cap : len); }

// Exclusive prefix over sequences of pages-per-head, into s_pfx[0..B]; returns total.
__device__ int block_page_prefix(const DecodeArgs& a, int* s_pfx, int* s_tmp) {
  const int nthreads = blockDim.x;
  const int t = threadIdx.x;
  const int per = (a.batch + nthreads - 1) / nthreads;
  const int lo = min(a.batch, t * per), hi = min(a.batch, lo + per);
  const int cap = a.max_pages * kPage;
  int local = 0;
  for (int b = lo; b < hi; ++b) {
    const int len = a.seq_lens[b];
    if ((len < 0 || len > cap) && blockIdx.x == 0) set_status(a.status, kStatusBadLength);
    local += (clamp_len(len, cap) + kPage - 1) / kPage;
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
    run += (clamp_len(a.seq_lens[b], cap) + kPage - 1) / kPage;
  }
  if (t == nthreads - 1) s_pfx[a.batch] = run;
  __syncthreads();
  return s_pfx[a.batch];
}

// Per-page descriptor, computed by one lane for one page of the warp's run.
struct Desc {
  int phys;   // physical page (valid when ntok > 0)
  int gphys;  // physical page holding the group's scale/zp (valid when has_sz)
  int meta;   // ntok | has_q << 8 | has_sz << 9 | kv head << 16
  int stream; // b * vheads + h (queries stream * gs + j, j < gs, read it)
};

// Sequence b, head h and page p of page-head g of the end-to-end order.
__device__ __forceinline__ void locate_page(const DecodeArgs& a, const int* s_pfx, int g, int& b, int& h,
                                            int& p, int& np) {
  const int gq = g / a.vheads;
  int lo = 0, hi = a.batch - 1;  // last b with pfx[b] <= gq
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_pfx[mid] <= gq) lo = mid; else hi = mid - 1;
  }
  b = lo;
  np = s_pfx[b + 1] - s_pfx[b];
  const int rem = g - a.vheads * s_pfx[b];
  h = rem / np;
  p = rem - h * np;
}

// Descriptor of page-head g for a warp whose pages lie in [glo, ghi) and whose
// first page is gfirst; `backward` warps take their pages in descending order,
// so their segments start at a stream's last page and their groups at a
// group's last page.
__device__ __forceinline__ Desc make_desc(const DecodeArgs& a, const int* s_pfx, int g, int gfirst,
                                          int glo, int ghi, bool backward) {
  Desc d{0, 0, 0, -1};
  if (g < glo || g >= ghi) return d;
  int b, h, p, np;
  locate_page(a, s_pfx, g, b, h, p, np);
  const int len = clamp_len(a.seq_lens[b], a.max_pages * kPage);
  const int ntok = min(kPage, len - p * kPage);
  const int32_t* row = a.block_table + (size_t)b * a.max_pages;
  const int phys = row[p];
  const int gphys = row[(p / a.group_pages) * a.group_pages];
  const bool first = (g == gfirst) || (backward ? p == np - 1 : p == 0);
  const bool grp = first || (p % a.group_pages) == (backward ? a.group_pages - 1 : 0);
  const bool gok = gphys >= 0 && gphys < a.num_pages;
  const bool pok = phys >= 0 && phys < a.num_pages;
  if (!gok || !pok) set_status(a.status, kStatusBadPage);
  d.phys = phys;
  d.gphys = gphys;
  d.meta = ((gok && pok) ? ntok : 0) | (first ? (1 << 8) : 0) | ((grp && gok) ? (1 << 9) : 0) |
           (((h * a.gs * a.hw) / a.group_q) << 16);
  d.stream = b * a.vheads + h;
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

template <int D, int WARPS, int STAGES, int VK>
__device__ __forceinline__ void issue_page(const DecodeArgs& a, const Desc& d, char* slot,
                                           uint64_t* bar) {
  using C = Cfg<D, WARPS, STAGES, VK>;
  const int ntok = d.meta & 0xff;
  const bool has_q = (d.meta >> 8) & 1, has_sz = (d.meta >> 9) & 1;
  const int kvh = d.meta >> 16;
  uint32_t bytes = 0;
  if (ntok) bytes += (uint32_t)ntok * (D * C::VB + D / 2);
  if (has_sz) bytes += 2 * D * 4;
  if (has_q) bytes += (uint32_t)a.gs * a.hw * D * 4;
  fence_proxy_async_smem();
  mbar_arrive_expect_tx(bar, bytes);
  if (ntok) {
    const size_t ph = (size_t)d.phys * a.kv_heads + kvh;
    bulk_g2s(slot + C::V_OFF, static_cast<const char*>(a.v_pool) + ph * kPage * D * C::VB,
             (uint32_t)ntok * D * C::VB, bar);
    bulk_g2s(slot + C::K_OFF, a.k_pool + ph * kPage * (D / 2), (uint32_t)ntok * (D / 2), bar);
  }
  if (has_sz) {
    bulk_g2s(slot + C::SZ_OFF,
             a.sz_pool + ((size_t)d.gphys * a.kv_heads + kvh) * 2 * D, 2 * D * 4, bar);
  }
  if (has_q)
    bulk_g2s(slot + C::Q_OFF, a.q + (size_t)d.stream * a.gs * a.hw * D,
             (uint32_t)a.gs * a.hw * D * 4, bar);
}


// Two 16-bit stored values (one 32-bit word, low half first) widened to
// float32 exactly.
template <int VK>
__device__ __forceinline__ float2 widen2(uint32_t w) {
  if constexpr (VK == 1) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  } else {  // bfloat16: the float32 with the same top 16 bits
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  }
}

// ps += p[t] * V[t, lane's dims] (lane layout of store_lane_vec); V rows are
// stored as float32 (VK 0) or as 16-bit floats widened on load (VK 1, 2).
template <int D, int VK>
__device__ __forceinline__ void pv_row(const char* vs, float pt, int t, int lane, float* ps) {
  constexpr int DPL = D / 32;
  if constexpr (VK == 0) {
    const float* row = reinterpret_cast<const float*>(vs) + t * D;
    if constexpr (DPL == 2) {
      const float2 v = *reinterpret_cast<const float2*>(row + 2 * lane);
      fma2_rn(ps[0], ps[1], v.x, v.y, pt);
    } else {
#pragma unroll
      for (int v4 = 0; v4 < DPL / 4; ++v4) {
        const float4 v = *reinterpret_cast<const float4*>(row + v4 * 128 + 4 * lane);
        fma2_rn(ps[4 * v4 + 0], ps[4 * v4 + 1], v.x, v.y, pt);
        fma2_rn(ps[4 * v4 + 2], ps[4 * v4 + 3], v.z, v.w, pt);
      }
    }
  } else {
    const uint16_t* row = reinterpret_cast<const uint16_t*>(vs) + t * D;
    if constexpr (DPL == 2) {
      const float2 v = widen2<VK>(*reinterpret_cast<const uint32_t*>(row + 2 * lane));
      fma2_rn(ps[0], ps[1], v.x, v.y, pt);
    } else {
#pragma unroll
      for (int v4 = 0; v4 < DPL / 4; ++v4) {
        const uint2 w = *reinterpret_cast<const uint2*>(row + v4 * 128 + 4 * lane);
        const float2 lo = widen2<VK>(w.x), hi = widen2<VK>(w.y);
        fma2_rn(ps[4 * v4 + 0], ps[4 * v4 + 1], lo.x, lo.y, pt);
        fma2_rn(ps[4 * v4 + 2], ps[4 * v4 + 3], hi.x, hi.y, pt);
      }
    }
  }
}


// ps[h] += pt[h] * V[t, lane's dims] for the HW heads of a warp: the value row
// is loaded (and 16-bit values widened) once for all heads.
template <int D, int VK, int HW>
__device__ __forceinline__ void pv_row_heads(const char* vs, const float* pt_row, int t, int lane,
                                             float (&ps)[HW][D / 32]) {
  constexpr int DPL = D / 32;
  float pt[HW];
  if constexpr (HW == 4) {
    const float4 x = *reinterpret_cast<const float4*>(pt_row);
    pt[0] = x.x; pt[1] = x.y; pt[2] = x.z; pt[3] = x.w;
  } else if constexpr (HW == 2) {
    const float2 x = *reinterpret_cast<const float2*>(pt_row);
    pt[0] = x.x; pt[1] = x.y;
  } else {
#pragma unroll
    for (int h = 0; h < HW; ++h) pt[h] = pt_row[h];
  }
  float v[DPL];
  if constexpr (VK == 0) {
    const float* row = reinterpret_cast<const float*>(vs) + t * D;
    if constexpr (DPL == 2) {
      const float2 x = *reinterpret_cast<const float2*>(row + 2 * lane);
      v[0] = x.x; v[1] = x.y;
    } else {
#pragma unroll
      for (int v4 = 0; v4 < DPL / 4; ++v4) {
        const float4 x = *reinterpret_cast<const float4*>(row + v4 * 128 + 4 * lane);
        v[4 * v4] = x.x; v[4 * v4 + 1] = x.y; v[4 * v4 + 2] = x.z; v[4 * v4 + 3] = x.w;
      }
    }
  } else {
    const uint16_t* row = reinterpret_cast<const uint16_t*>(vs) + t * D;
    if constexpr (DPL == 2) {
      const float2 x = widen2<VK>(*reinterpret_cast<const uint32_t*>(row + 2 * lane));
      v[0] = x.x; v[1] = x.y;
    } else {
#pragma unroll
      for (int v4 = 0; v4 < DPL / 4; ++v4) {
        const uint2 w = *reinterpret_cast<const uint2*>(row + v4 * 128 + 4 * lane);
        const float2 lo = widen2<VK>(w.x), hi = widen2<VK>(w.y);
        v[4 * v4] = lo.x; v[4 * v4 + 1] = lo.y; v[4 * v4 + 2] = hi.x; v[4 * v4 + 3] = hi.y;
      }
    }
  }
#pragma unroll
  for (int h = 0; h < HW; ++h)
#pragma unroll
    for (int k = 0; k < DPL; k += 2) fma2_rn(ps[h][k], ps[h][k + 1], v[k], v[k + 1], pt[h]);
}

// Fused split exchange, push side: store this GPU's (m, l, acc) of query
// stream qs into every rank's buffer (plain 16-byte stores through the peer
// mappings), then raise this rank's flag for qs there (release, system scope).
// No waiting: a warp pushes everything it owns before it waits on anything.
template <int D>
__device__ __forceinline__ void x_push(const DecodeArgs& a, long long S, long long qs, double m,
                                       double l, const float* o, int lane) {
  constexpr int REC = 16 + 4 * D;
  const uint32_t E = reinterpret_cast<const uint32_t*>(a.xbuf[a.xrank])[qs] + 1u;
  const int par = (int)(E & 1u);
  for (int r = 0; r < a.xworld; ++r) {
    char* rec = a.xbuf[r] + x_off_recs(S) + (((size_t)par * kXRanks + a.xrank) * S + qs) * REC;
    if (lane == 0) {
      *reinterpret_cast<double*>(rec) = m;
      *reinterpret_cast<double*>(rec + 8) = l;
    }
    store_lane_vec<D>(reinterpret_cast<float*>(rec + 16), o, lane);
  }
  fence_acq_rel_sys();
  __syncwarp();
  if (lane < a.xworld) {
    uint32_t* f = reinterpret_cast<uint32_t*>(a.xbuf[lane] + x_off_flag(S)) +
                  ((size_t)par * kXRanks + a.xrank) * S + qs;
    st_release_sys(f, E);
  }
}

// Fused split exchange, merge side: wait (bounded) for every rank's flag of
// qs in this rank's buffer, then merge the ranks' records -- the reference's
// LSE merge (csrc/flash_decode_int4.cu:199-220) across GPUs, in float64 --
// into the output. A rank that does not arrive within 2 s gives NaN and
// INT4KV_STATUS_PEER_TIMEOUT instead of a hang. `dead` is the warp's record of
// an earlier timeout: its later streams give up without waiting again, so a
// lost peer costs a warp one wait, not one per stream.
template <int D>
__device__ __forceinline__ void x_finish(const DecodeArgs& a, long long S, long long qs, int lane,
                                         bool& dead) {
  constexpr int REC = 16 + 4 * D;
  constexpr int DPL = D / 32;
  char* own = a.xbuf[a.xrank];
  uint32_t* step = reinterpret_cast<uint32_t*>(own);
  const uint32_t E = step[qs] + 1u;
  const int par = (int)(E & 1u);
  bool ok = true;
  if (lane < a.xworld) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(own + x_off_flag(S)) +
                        ((size_t)par * kXRanks + lane) * S + qs;
    ok = ld_acquire_sys(f) == E;
    if (!ok && !dead) {
      const uint64_t t0 = global_ns();
      while (!(ok = ld_acquire_sys(f) == E)) {
        if (global_ns() - t0 > kPeerWaitNs) break;
        __nanosleep(256);
      }
    }
  }
  ok = __all_sync(0xffffffffu, ok);
  // lane r acquired rank r's flag; the warp barrier orders those acquires
  // before every lane's reads of every rank's record
  __syncwarp();
  dead = dead || !ok;
  if (lane == 0) step[qs] = E;
  float o[DPL];
  if (!ok) {
    if (lane == 0) set_status(a.status, kStatusPeerTimeout);
#pragma unroll
    for (int k = 0; k < DPL; ++k) o[k] = __int_as_float(0x7fc00000);
  } else {
    const char* base = own + x_off_recs(S) + ((size_t)par * kXRanks * S + qs) * REC;
    const size_t stride = (size_t)S * REC;
    double M = -INFINITY;
    for (int r = 0; r < a.xworld; ++r)
      M = fmax(M, __ldcg(reinterpret_cast<const double*>(base + r * stride)));
    double L = 0.0, O[DPL];
#pragma unroll
    for (int k = 0; k < DPL; ++k) O[k] = 0.0;
    if (M != -INFINITY) {
      for (int r = 0; r < a.xworld; ++r) {
        const char* rec = base + r * stride;
        const double m = __ldcg(reinterpret_cast<const double*>(rec));
        if (m == -INFINITY) continue;
        const double e = exp(m - M);
        L = fma(__ldcg(reinterpret_cast<const double*>(rec + 8)), e, L);
        float v[DPL];
        load_lane_vec_cg<D>(reinterpret_cast<const float*>(rec + 16), v, lane);
#pragma unroll
        for (int k = 0; k < DPL; ++k) O[k] = fma((double)v[k], e, O[k]);
      }
    }
    const double den = fmax(L, 1e-10);
#pragma unroll
    for (int k = 0; k < DPL; ++k) o[k] = (float)(O[k] / den);
  }
  store_lane_vec<D>(a.out + (size_t)qs * D, o, lane);
}

// Streams without a page on this GPU (its token range of them is empty) still
// take part in the exchange: group gw pushes, then finishes, the empty
// records of streams gw, gw + NW, ...
template <int D>
__device__ __forceinline__ void x_empty_streams(const DecodeArgs& a, const int* s_pfx, long long S,
                                                long long gw, long long NW, int gs, int gj, int lane,
                                                bool finish, bool& dead) {
  constexpr int DPL = D / 32;
  float z[DPL];
#pragma unroll
  for (int k = 0; k < DPL; ++k) z[k] = 0.f;
  const long long SV = (long long)a.batch * a.vheads;
  for (long long vs = gw; vs < SV; vs += NW) {
    const int b = (int)(vs / a.vheads);
    if (s_pfx[b + 1] != s_pfx[b]) continue;
    const long long qs = vs * gs + gj;
    if (finish) x_finish<D>(a, S, qs, lane, dead);
    else x_push<D>(a, S, qs, -INFINITY, 0.0, z, lane);
  }
}

// 16-bit value pools halve the stage size, so up to four CTAs fit an SM's
// shared memory; registers are capped at 128 so that four could be resident,
// but the grid launches three per SM (I4KV_DECODE_MAX_CTAS_16: measured 45.5
// us at config 0 against 46.5 with four and 53.5 with two). Float32 pools with
// D <= 128 are held to 168 registers, the budget of three 128-thread CTAs per
// SM that a grouped-query ring group runs at (D = 256 keeps its full budget).
//
// HW = query heads per warp (grouped-query attention, HW in {1, 2, 4}): one
// warp serves HW consecutive query heads of every kv page it takes. With
// HW > 1 the heads sit in the MMA's columns: pass p's eight B columns are
// (head, digit) pairs -- for HW = 4, columns 2t and 2t + 1 are digits 2p and
// 2p + 1 of head t -- so after HW passes lane (g, t) holds head t's logits of
// tokens g and g + 8 without any cross-lane sum, and the softmax of the HW
// heads runs side by side across the lanes (lane t owns head t * HW / 4). The
// page's codes are loaded into A fragments once and each value row once for all
// heads. HW = 1 is plain one-head-per-warp decoding.
template <int D, int WARPS, int STAGES, int VK, int HW>
__global__ void __launch_bounds__(WARPS * 32, VK == 0 ? (D <= 128 ? (HW >= 4 ? 2 : 3) : 1)
                                                       : (HW > 1 ? I4KV_MULTIHEAD16_MIN_CTAS : 4))
paged_decode_kernel(DecodeArgs a) {
  using C = Cfg<D, WARPS, STAGES, VK>;
  constexpr int DPL = C::DPL;
  if constexpr (I4KV_DECODE_PDL) grid_dependency_wait();  // the predecessor's writes are visible
  extern __shared__ __align__(128) char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);                 // WARPS*STAGES
  int* s_tmp = reinterpret_cast<int*>(smem + 8 * WARPS * STAGES);      // WARPS ints
  // warp pairs: claim word (forward count | backward count << 32) and the
  // end-of-run handoff counter of each pair
  unsigned long long* s_claim = reinterpret_cast<unsigned long long*>(smem + 128);  // WARPS / 2
  int* s_pair_done = reinterpret_cast<int*>(smem + 128 + 8 * (WARPS / 2));         // WARPS / 2
  static_assert(8 * WARPS * STAGES + 4 * WARPS <= 128 && 128 + 12 * (WARPS / 2) <= 256, "header layout");
  int* s_pfx = reinterpret_cast<int*>(smem + 256);                     // batch+1 ints
  char* stages = smem + 256 + pfx_bytes(a.batch);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int fg = lane >> 2, ft = lane & 3;  // mma fragment row group / thread in group
  const int hl = (ft * HW) / 4;              // HW > 1: the head whose softmax this lane runs
  // Ring groups: gs warps share one ring of STAGES * gs slots; warp gj of the
  // group serves query heads (vh * gs + gj) * HW + k, k < HW, of every page the
  // group stages (gs = 1, HW = 1 without GQA: one warp, one ring, one query).
  const int gs = a.gs, gpc = WARPS / gs;
  const int gi = warp / gs, gj = warp - gi * gs;
  // slots per ring: STAGES pages per warp alone; a ring group keeps gs pages
  // in flight (its queries share each page, so it needs fewer bytes in flight
  // and fits more CTAs per SM)
  const int depth = gs == 1 ? STAGES : gs * I4KV_GQA_RING_PAGES_PER_WARP;
  const int sb = C::Q_OFF + gs * HW * D * 4;  // stage bytes with gs * HW queries
  const bool leader = gj == 0;
  {  // the block table into L2 while the lengths load (first descriptors hit L2)
    const size_t bt_bytes = (size_t)a.batch * a.max_pages * 4;
    const size_t off = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 128;
    if (off < bt_bytes)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(a.block_table) + off));
  }
  const bool xmode = HW == 1 && a.xworld > 0;  // the fused split runs one head per warp
  // Warp pairs: with one warp per ring (no grouped-query sharing) in a plain
  // decode, warps 2k and 2k + 1 share one run; the first takes its pages
  // forward from the run's start, the second backward from its end, each
  // claiming its next page from the pair's shared claim word, so the pair
  // finishes together however its two warps' page rates differ.
  const bool paired = (WARPS % 2 == 0) && STAGES >= 2 && gs == 1 && !xmode && a.part_out == nullptr;
  const bool bwd = paired && (warp & 1);
  uint64_t* bar = bars + gi * depth;
  if (leader && lane == 0) {  // ordered before every wait by the barriers of the length prefix
    for (int s = 0; s < depth; ++s) mbar_init(&bar[s], 1);
    fence_barrier_init();
  }
  if (paired && !bwd && lane == 0) {
    s_claim[warp / 2] = 0ull;
    s_pair_done[warp / 2] = 0;
  }
  const int total_pages = block_page_prefix(a, s_pfx, s_tmp);
  const long long streams = (long long)a.batch * a.heads;

  // Empty streams get exact zeros (the reference returns 0 / max(0, 1e-10)),
  // or, in partial mode, the empty record (m = -inf, l = 0, acc = 0); run
  // after this warp's first copies are out.
  auto zero_empty_streams = [&]() {
    for (long long s = (long long)blockIdx.x * blockDim.x + threadIdx.x; s < streams;
         s += (long long)gridDim.x * blockDim.x) {
      const int b = (int)(s / a.heads);
      if (s_pfx[b + 1] == s_pfx[b] && a.xworld == 0) {
        float* dst = a.out + (size_t)s * D;
        if (a.part_out) {
          char* rec = a.part_out + (size_t)s * C::REC_BYTES;
          *reinterpret_cast<double*>(rec) = -INFINITY;
          *reinterpret_cast<double*>(rec + 8) = 0.0;
          dst = reinterpret_cast<float*>(rec + 16);
        }
        for (int k = 0; k < D; k += 4) *reinterpret_cast<float4*>(dst + k) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  };

  const long long T = (long long)a.vheads * total_pages;  // < 2^31 (checked on the host)
  const long long NW = (long long)gridDim.x * gpc;         // ring groups in the grid
  const long long gw = (long long)blockIdx.x * gpc + gi;
  // contribution units of the stream-K order: warp pairs, or ring groups
  const long long NU = paired ? (long long)gridDim.x * (WARPS / 2) : NW;
  const long long gu = paired ? (long long)blockIdx.x * (WARPS / 2) + warp / 2 : gw;
  const int g0 = (int)floor_div_s52(gu * T, NU), g1 = (int)floor_div_s52((gu + 1) * T, NU);
  // page-head of the warp's i-th page, and its page count (in a pair, the
  // pair's length until a claim fails)
  auto page_at = [&](int i) -> int { return bwd ? g1 - 1 - i : g0 + i; };
  const int gfirst = bwd ? g1 - 1 : g0;
  int n = g1 - g0;
  // Each warp of a pair takes a share of the run from its end without asking
  // (3/8 each, leaving a middle quarter -- enough to absorb page rates 25 %
  // apart -- so most pages cost no claim); the rest is claimed page by page.
  constexpr int kOwnEighths = HW > 1 ? I4KV_PAIR_OWN_EIGHTHS_MH
                              : (VK == 0 ? I4KV_PAIR_OWN_EIGHTHS_F32 : I4KV_PAIR_OWN_EIGHTHS_16);
  const int n_own = paired ? (int)(((long long)n * kOwnEighths) / 8) : n;
  // Claims are pipelined: after a claim succeeds, lane 0 sends the next one at
  // once and its answer is read when that page is due, so the shared-memory
  // atomic's round trip overlaps a page of work. Claims go in page order, so
  // every claim that succeeds is consumed.
  unsigned long long claim_word = 0ull;  // lane 0: the outstanding claim's answer
  bool claim_out = false;                // a claim is outstanding (warp-uniform)
  auto claim_send = [&]() {
    if (lane == 0) claim_word = atomicAdd(&s_claim[warp / 2], bwd ? (1ull << 32) : 1ull);
    claim_out = true;
  };
  auto claim = [&](int i) -> bool {  // the warp's i-th page, unless the partner has taken it
    if (i < n_own) return true;
    if (!claim_out) claim_send();
    const unsigned long long old = __shfl_sync(kFull, claim_word, 0);
    claim_out = false;
    const bool ok = (long long)(uint32_t)old + (long long)(old >> 32) < (long long)(g1 - g0 - 2 * n_own);
    if (ok) claim_send();
    return ok;
  };
  if (n <= 0) {
    zero_empty_streams();
    if (xmode) {  // no pages here, but maybe empty streams to exchange
      bool dead = false;
      x_empty_streams<D>(a, s_pfx, streams, gw, NW, gs, gj, lane, false, dead);
      x_empty_streams<D>(a, s_pfx, streams, gw, NW, gs, gj, lane, true, dead);
    }
    return;
  }

  char* ring = stages + (size_t)gi * depth * sb;
  // this warp's digit staging bytes (4 rows of D + 32: the padding puts the
  // four rows a round reads in different banks), dig[g * (D + 32) + c]
  // = digit g (mod 4) of channel c; the page's softmax weights reuse its
  // first 64 * HW bytes between group changes
  constexpr int kDigRow = D + 32;
  uint8_t* dig = reinterpret_cast<uint8_t*>(stages + (size_t)gpc * depth * sb +
                                            (size_t)warp * 4 * kDigRow);
  float* p_tab = reinterpret_cast<float*>(dig);  // [16 tokens][HW heads]

  Desc cur = make_desc(a, s_pfx, page_at(lane), gfirst, g0, g1, bwd);
  for (int i = 0; i < depth && i < n; ++i) {  // prologue: the first `depth` pages (all in chunk 0)
    if (paired && !claim(i)) {
      n = i;
      break;
    }
    const Desc d = shfl_desc(cur, i);
    if (leader && lane == 0) issue_page<D, WARPS, STAGES, VK>(a, d, ring + i * sb, &bar[i]);
  }
  Desc nxt = make_desc(a, s_pfx, page_at(32 + lane), gfirst, g0, g1, bwd);
  zero_empty_streams();

  // Logits of the current group: q.k = sum_c qs_c code_c - bias with
  // qs_c = q_c s_c (exact in float64) and bias = sum_c q_c zp_c s_c. The code
  // sum runs on the tensor cores in exact integer arithmetic: qs_c in fixed
  // point, X_c = round(qs_c 2^(56-E)) with |qs_c| < 2^E, written as eight
  // base-128 digits (the top one signed); mma.m16n8k32 (u8 codes x s8 digits,
  // int32 sums, at most 128 * 15 * 128 in magnitude) gives per token the sum
  // of code x digit p for the two digits p = 2t, 2t+1 of this lane, and
  // float64 weights 2^(E - 7 - 7p) recombine them. Truncation is below
  // 2^(E-56) per channel, as fine as float64 accumulation.
  uint32_t bfrag[HW][2 * C::KT][2];  // mma B operands: [head][2e + parity][half] of k-tile e
  float qv[HW][DPL];                 // the warp's queries at channels lane * DPL + j
  double w0[HW], w1[HW];             // weights of digits 2ft and 2ft + 1
  double bias[HW];
  // Value and denominator sums: float32 with a Kahan compensation term, so
  // long page runs accumulate without float64 conversions on the hot path.
  float acc[HW][DPL], acc_c[HW][DPL];
  float l_lane[HW], l_c[HW];
  double m_run[HW];
  int seg_stream = -1;
  bool aborted = false;
  int abort_at = 0;
#pragma unroll
  for (int h = 0; h < HW; ++h) {
    w0[h] = w1[h] = bias[h] = 0.0;
    l_lane[h] = l_c[h] = 0.f;
    m_run[h] = -INFINITY;
#pragma unroll
    for (int k = 0; k < DPL; ++k) { acc[h][k] = 0.f; acc_c[h][k] = 0.f; qv[h][k] = 0.f; }
#pragma unroll
    for (int k = 0; k < 2 * C::KT; ++k) { bfrag[h][k][0] = 0u; bfrag[h][k][1] = 0u; }
  }

  int xm0 = -1, xm1 = -1;  // exchange mode: streams this warp merged locally (at most 2)
  int* counters = reinterpret_cast<int*>(a.ws);
  char* recs = a.ws + cnt_bytes(streams);

  // Warps [w_lo, w_hi] whose runs touch `stream`; returns how many of them
  // hold a non-empty run (those are the stream's contributors).
  // ... and the stream's pages [g_lo, g_hi) of the end-to-end order.
  auto stream_span = [&](int stream, long long& w_lo, long long& w_hi, int& g_lo, int& g_hi) -> int {
    const int b = stream / a.vheads, h = stream - b * a.vheads;
    const int np = s_pfx[b + 1] - s_pfx[b];
    const long long gs0 = (long long)a.vheads * s_pfx[b] + (long long)h * np, ge = gs0 + np;
    g_lo = (int)gs0;
    g_hi = (int)ge;
    w_lo = floor_div_s52((gs0 + 1) * NU - 1, T);
    w_hi = floor_div_s52(ge * NU - 1, T);
    return (T >= NU) ? (int)(w_hi - w_lo + 1) : np;
  };
  auto contributors_of = [&](int stream, long long& w_lo, long long& w_hi) -> int {
    int g_lo, g_hi;
    return stream_span(stream, w_lo, w_hi, g_lo, g_hi);
  };
  // Multi-head warps: the current segment's contributors and pages, worked out
  // when the segment starts, so the end of the run (on the launch's critical
  // path) does no index arithmetic. Measured side by side on one B200 (means
  // of 22 launches): GQA-4 at config 0 39.0 -> 37.8 us; one-head warps keep
  // the end-of-run arithmetic (their registers are tighter: config 0 61.1 vs
  // 62.2 us with it).
  int seg_nc = 0, seg_g0 = 0, seg_g1 = 0, seg_wlo = 0, seg_whi = -1;  // unit indices < 2^31

  // Warp-wide sum of head h's lane denominators (float32 sum minus compensation).
  auto lane_sum = [&](int h) -> double {
    double lsum = (double)l_lane[h] - (double)l_c[h];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(kFull, lsum, o);
    return lsum;
  };

  auto put_record = [&](char* rec, double m, double l, const float* o) {
    if (lane == 0) {
      *reinterpret_cast<double*>(rec) = m;
      *reinterpret_cast<double*>(rec + 8) = l;
    }
    store_lane_vec<D>(reinterpret_cast<float*>(rec + 16), o, lane);
  };

  // Per-head running max and denominator. HW = 1: the warp's own state. HW > 1:
  // lane (g, t) keeps the state of head t * HW / 4 in m_run[0] / l_lane[0]
  // (for HW = 2 the odd lanes t duplicate the even ones and add nothing).
  auto head_src = [&](int h) -> int { return (h * 4) / HW; };  // lane (0, t) of head h
  auto head_m = [&](int h) -> double {
    if constexpr (HW == 1) return m_run[h];
    else return __shfl_sync(kFull, m_run[0], head_src(h));
  };
  auto head_l = [&](int h) -> double {
    if constexpr (HW == 1) {
      return lane_sum(h);
    } else {
      double x = (HW == 2 && (ft & 1)) ? 0.0 : (double)l_lane[0] - (double)l_c[0];
      x += __shfl_xor_sync(kFull, x, 4);
      x += __shfl_xor_sync(kFull, x, 8);
      x += __shfl_xor_sync(kFull, x, 16);
      return __shfl_sync(kFull, x, head_src(h));
    }
  };

  // A stream this warp covered alone: write its outputs (or, in partial mode,
  // its records) straight from the running state, head by head.
  auto finish_alone = [&](int stream) {
#pragma unroll
    for (int h = 0; h < HW; ++h) {
      const size_t qstream = ((size_t)stream * gs + gj) * HW + h;
      const double lsum = head_l(h);
      const double mh = head_m(h);
      float o[DPL];
      if (a.part_out || xmode) {
#pragma unroll
        for (int k = 0; k < DPL; ++k) o[k] = (float)((double)acc[h][k] - (double)acc_c[h][k]);
        if (xmode) x_push<D>(a, streams, (long long)qstream, mh, lsum, o, lane);
        else put_record(a.part_out + qstream * C::REC_BYTES, mh, lsum, o);
        continue;
      }
      const double rden = rcp_f64(fmax(lsum, 1e-10));
#pragma unroll
      for (int k = 0; k < DPL; ++k) o[k] = (float)(((double)acc[h][k] - (double)acc_c[h][k]) * rden);
      store_lane_vec<D>(a.out + qstream * D, o, lane);
    }
  };

  // Merge every contributor's record of `stream` (this warp arrived last) and
  // write the output, or in partial mode the merged record. Contributors are
  // taken eight at a time: lane j loads the (m, l) of the round's j-th record
  // while 16-byte asynchronous copies bring the round's value sums into the
  // warp's ring slot, so a round costs one round trip to L2 (the records were
  // written by other SMs, often on the other die); rounds combine online in
  // float64. The loops stay rolled: this code runs once per warp, at the end
  // of the launch, where every branch target and constant is fetched cold.
  bool keep_last_slot = false;  // a pair partner still reads this warp's last ring slot
  auto merge_stream = [&](int stream, long long w_lo, long long w_hi) {
    constexpr int MC = 8;  // records per round: (m, l) in lanes 0..7, values staged in shared memory
    // the warp's staging area: a ring slot, free once the group's run is over
    // (slot gj of a group ring is at least MC * D floats for every instantiation)
    char* stage = ring + (size_t)(gj % depth) * sb;
    const bool all_run = T >= NU;
#pragma unroll 1
    for (int h = 0; h < HW; ++h) {
      double M = -INFINITY, L = 0.0, O[DPL];
#pragma unroll
      for (int k = 0; k < DPL; ++k) O[k] = 0.0;
#pragma unroll 1
      for (long long base = w_lo; base <= w_hi; base += MC) {
        const int cnt = (int)min((long long)MC, w_hi - base + 1);
#pragma unroll 1
        for (int j = 0; j < cnt; ++j) {
          const char* src = recs + (((size_t)(base + j + stream) * gs + gj) * HW + h) * C::REC_BYTES + 16;
          for (int u = 16 * lane; u < 4 * D; u += 512) cp_async16(stage + j * 4 * D + u, src + u);
        }
        cp_async_commit();
        const long long wj = base + lane;
        const bool okj = lane < cnt && (all_run || floor_div_s52(wj * T, NU) != floor_div_s52((wj + 1) * T, NU));
        double mj = -INFINITY, lj = 0.0;
        if (okj) {
          const char* r = recs + (((size_t)(wj + stream) * gs + gj) * HW + h) * C::REC_BYTES;
          mj = __ldcg(reinterpret_cast<const double*>(r));
          lj = __ldcg(reinterpret_cast<const double*>(r + 8));
        }
        double cm = mj;
#pragma unroll
        for (int o = MC / 2; o > 0; o >>= 1) cm = fmax(cm, __shfl_xor_sync(kFull, cm, o));
        const double m_new = fmax(M, __shfl_sync(kFull, cm, 0));
        cp_async_wait<0>();
        __syncwarp();
        if (m_new == -INFINITY) continue;  // nothing live yet
        double c = 0.0;  // rescale of the earlier rounds (streams with more than MC records)
        if (M != -INFINITY) c = exp_nonpos(M - m_new);
        const double ej = (okj && mj != -INFINITY) ? exp_nonpos(mj - m_new) : 0.0;
        double lc = lj * ej;
#pragma unroll
        for (int o = MC / 2; o > 0; o >>= 1) lc += __shfl_xor_sync(kFull, lc, o);
        L = fma(L, c, __shfl_sync(kFull, lc, 0));
#pragma unroll
        for (int k = 0; k < DPL; ++k) O[k] *= c;
#pragma unroll 1
        for (int j = 0; j < cnt; ++j) {
          const double e = __shfl_sync(kFull, ej, j);
          if (e != 0.0) {  // records of empty runs are never read into the sum
            float v[DPL];
            load_lane_vec_smem<D>(reinterpret_cast<const float*>(stage + j * 4 * D), v, lane);
#pragma unroll
            for (int k = 0; k < DPL; ++k) O[k] = fma((double)v[k], e, O[k]);
          }
        }
        __syncwarp();  // the stage is read before the next round's copies
        M = m_new;
      }
      const size_t qstream = ((size_t)stream * gs + gj) * HW + h;
      float o[DPL];
      if (a.part_out || xmode) {  // the merged (M, L, O) of this GPU's share of the stream
#pragma unroll
        for (int k = 0; k < DPL; ++k) o[k] = (float)O[k];
        if (xmode) {
          x_push<D>(a, streams, (long long)qstream, M, L, o, lane);
          (xm0 < 0 ? xm0 : xm1) = stream;  // finished after the warp's last push
        } else {
          put_record(a.part_out + qstream * C::REC_BYTES, M, L, o);
        }
        continue;
      }
      const double rden = rcp_f64(fmax(L, 1e-10));
#pragma unroll
      for (int k = 0; k < DPL; ++k) o[k] = (float)(O[k] * rden);
      store_lane_vec<D>(a.out + qstream * D, o, lane);
    }
  };

  // The same merge for a warp serving HW > 1 heads: a contributor's HW records
  // are adjacent, so each round stages whole contributors (every head's record,
  // headers included) with one set of 16-byte asynchronous copies, and lane
  // j * HW + h takes the (m, l) of contributor j's head h from the staged
  // copy. A round thus costs one round trip to L2 for all heads, where a round
  // per head would cost HW. Contributors per round: as many as the warp's free
  // ring bytes hold, at most 32 / HW.
  auto merge_stream_heads = [&](int stream, long long w_lo, long long w_hi) {
    constexpr int REC = C::REC_BYTES;
    char* stage = ring + (size_t)(gj % depth) * sb;
    // bytes of the ring this warp owns, less a last slot its pair partner may still read
    const int cap = gs == 1 ? (keep_last_slot ? depth - 1 : depth) * sb : sb;
    const int per = min(32 / HW, cap / (HW * REC));
    const bool all_run = T >= NU;
    double M = -INFINITY, L = 0.0;  // running (m, l) of head lane % HW
    double O[HW][DPL];
#pragma unroll
    for (int h = 0; h < HW; ++h)
#pragma unroll
      for (int k = 0; k < DPL; ++k) O[h][k] = 0.0;
#pragma unroll 1
    for (long long base = w_lo; base <= w_hi; base += per) {
      const int cnt = (int)min((long long)per, w_hi - base + 1);
#pragma unroll 1
      for (int j = 0; j < cnt; ++j) {
        const char* src = recs + (((size_t)(base + j + stream) * gs + gj) * HW) * REC;
        for (int u = 16 * lane; u < HW * REC; u += 512) cp_async16(stage + j * HW * REC + u, src + u);
      }
      cp_async_commit();
      cp_async_wait<0>();
      __syncwarp();
      const int jl = lane / HW;
      const long long wj = base + jl;
      const bool okj = jl < cnt && (all_run || floor_div_s52(wj * T, NU) != floor_div_s52((wj + 1) * T, NU));
      double mj = -INFINITY, lj = 0.0;
      if (okj) {
        const char* r = stage + (size_t)lane * REC;  // contributor jl, head lane % HW
        mj = *reinterpret_cast<const double*>(r);
        lj = *reinterpret_cast<const double*>(r + 8);
      }
      double cm = mj;
#pragma unroll
      for (int o = HW; o < 32; o <<= 1) cm = fmax(cm, __shfl_xor_sync(kFull, cm, o));
      const double m_new = fmax(M, cm);
      double c = 1.0, ej = 0.0;
      if (m_new != -INFINITY) {
        c = M != -INFINITY ? exp_nonpos(M - m_new) : 0.0;
        ej = (okj && mj != -INFINITY) ? exp_nonpos(mj - m_new) : 0.0;
      }
      double lc = lj * ej;
#pragma unroll
      for (int o = HW; o < 32; o <<= 1) lc += __shfl_xor_sync(kFull, lc, o);
      L = m_new != -INFINITY ? fma(L, c, lc) : L;
#pragma unroll
      for (int h = 0; h < HW; ++h) {
        const double ch = __shfl_sync(kFull, c, h);
#pragma unroll
        for (int k = 0; k < DPL; ++k) O[h][k] *= ch;
      }
      // branch-free, so the loads and shuffles of a contributor's heads issue
      // together; a record with weight 0 (an empty run's, never written) is
      // replaced by zeros before it can reach the sum
#pragma unroll 1
      for (int j = 0; j < cnt; ++j) {
        double e[HW];
        float v[HW][DPL];
#pragma unroll
        for (int h = 0; h < HW; ++h) {
          e[h] = __shfl_sync(kFull, ej, j * HW + h);
          load_lane_vec_smem<D>(reinterpret_cast<const float*>(stage + (size_t)(j * HW + h) * REC + 16), v[h], lane);
        }
#pragma unroll
        for (int h = 0; h < HW; ++h)
#pragma unroll
          for (int k = 0; k < DPL; ++k) O[h][k] = fma(e[h] != 0.0 ? (double)v[h][k] : 0.0, e[h], O[h][k]);
      }
      __syncwarp();  // the stage is read before the next round's copies
      M = m_new;
    }
#pragma unroll
    for (int h = 0; h < HW; ++h) {
      const double Mh = __shfl_sync(kFull, M, h), Lh = __shfl_sync(kFull, L, h);
      const size_t qstream = ((size_t)stream * gs + gj) * HW + h;
      float o[DPL];
      if (a.part_out) {  // the merged (M, L, O) of this launch's share of the stream
#pragma unroll
        for (int k = 0; k < DPL; ++k) o[k] = (float)O[h][k];
        put_record(a.part_out + qstream * C::REC_BYTES, Mh, Lh, o);
        continue;
      }
      const double rden = rcp_f64(fmax(Lh, 1e-10));
#pragma unroll
      for (int k = 0; k < DPL; ++k) o[k] = (float)(O[h][k] * rden);
      store_lane_vec<D>(a.out + qstream * D, o, lane);
    }
  };

  // The warp's first segment, when its stream is shared with earlier warps and
  // ends inside this run: its record is stored and its arrival counted as soon
  // as the segment ends; the arrival's ticket (the counter's old value) is
  // read only at the end of the run.
  int held_stream = -1, held_n = 0, held_ticket = 0;

  auto end_segment = [&](int stream) {
    long long w_lo, w_hi;
    const int nc = contributors_of(stream, w_lo, w_hi);
    if (nc == 1) {
      finish_alone(stream);
      return;
    }
    // Only the run's first segment can get here mid-run. Its record is
    // published now and its arrival counted at once; the ticket is read only
    // at the end of the run, so the atomic's round trip overlaps the pages
    // that follow (the other contributors reach this stream at the ends of
    // their runs, so this warp is almost never the last arrival).
    held_stream = stream;
    held_n = nc;
#pragma unroll
    for (int h = 0; h < HW; ++h) {
      float o[DPL];
#pragma unroll
      for (int k = 0; k < DPL; ++k) o[k] = (float)((double)acc[h][k] - (double)acc_c[h][k]);
      const double lh = head_l(h), mh = head_m(h);
      put_record(recs + (((size_t)(gu + stream) * gs + gj) * HW + h) * C::REC_BYTES, mh, lh, o);
    }
    __syncwarp();
    if (lane == 0) held_ticket = atom_add_acq_rel_gpu(&counters[(size_t)stream * gs + gj], 1);
  };

  // End of the run: publish the last segment's record (if shared) with one
  // release + acquire arrival, then merge every stream this warp arrived last
  // at (the first segment's only when its ticket says so, which is rare).
  auto end_run = [&]() {
    long long lo_c = 0, hi_c = -1;
    int n_cur = 0;
    if (seg_stream >= 0) {
      if constexpr (HW > 1) {
        n_cur = seg_nc;
        lo_c = seg_wlo;
        hi_c = seg_whi;
      } else {
        n_cur = contributors_of(seg_stream, lo_c, hi_c);
      }
    }
    // A pair's meeting point m splits its run: the forward warp took [g0, m),
    // the backward one [m, g1). When both warps' last segments lie in the same
    // stream, each leaves its partial(s) in its ring's last slot (free now;
    // the merges below stage in the slots before it while the partner may
    // still read it) and the second to arrive merges the two;
    // that stream then counts as one contributor of the pair, like every other
    // stream of the run.
    bool have_cur = seg_stream >= 0;  // this warp holds the last segment's state
    bool pair_merged = false;         // ... merged with the partner's (in pm, pl, po)
    double pm[HW], pl[HW], po[HW][DPL];
    if (paired && have_cur) {
      const int m = bwd ? g1 - n : g0 + n;
      bool split = false;
      if constexpr (HW > 1) {
        // the partner's page next to the meeting point (m for the forward
        // warp, m - 1 for the backward one) lies in this warp's last stream
        split = bwd ? (m > g0 && m - 1 >= seg_g0) : (m < g1 && m < seg_g1);
      } else if (bwd ? m > g0 : m < g1) {
        int b, h, p, np;
        locate_page(a, s_pfx, bwd ? m - 1 : m, b, h, p, np);
        split = b * a.vheads + h == seg_stream;
      }
      if (split) {
        float o[HW][DPL];
        double lsum[HW], mh[HW];
#pragma unroll
        for (int h = 0; h < HW; ++h) {
#pragma unroll
          for (int k = 0; k < DPL; ++k) o[h][k] = __fsub_rn(acc[h][k], acc_c[h][k]);
          lsum[h] = head_l(h);
          mh[h] = head_m(h);
          put_record(ring + (size_t)(depth - 1) * sb + (size_t)h * C::REC_BYTES, mh[h], lsum[h], o[h]);
        }
        __threadfence_block();
        __syncwarp();
        int arrived = 0;
        if (lane == 0) arrived = atomicAdd(&s_pair_done[warp / 2], 1);
        arrived = __shfl_sync(kFull, arrived, 0);
        if (arrived == 0) {
          have_cur = false;  // the partner finishes the stream
          keep_last_slot = true;  // ... reading this warp's record from its last ring slot
        } else {
          __threadfence_block();
          __syncwarp();
          const char* other = stages + ((size_t)(warp ^ 1) * depth + depth - 1) * sb;
#pragma unroll
          for (int h = 0; h < HW; ++h) {
            const char* oh = other + (size_t)h * C::REC_BYTES;
            const double m2 = *reinterpret_cast<const double*>(oh);
            const double l2 = *reinterpret_cast<const double*>(oh + 8);
            float o2[DPL];
            load_lane_vec_smem<D>(reinterpret_cast<const float*>(oh + 16), o2, lane);
            pm[h] = fmax(mh[h], m2);
            const double e1 = exp_nonpos(mh[h] - pm[h]), e2 = exp_nonpos(m2 - pm[h]);
            pl[h] = fma(lsum[h], e1, l2 * e2);
#pragma unroll
            for (int k = 0; k < DPL; ++k) po[h][k] = fma((double)o[h][k], e1, (double)o2[k] * e2);
          }
          pair_merged = true;
        }
      }
    }
    if (have_cur && n_cur == 1) {  // the stream lies inside this run (or pair): finish it here
      if (pair_merged) {
#pragma unroll
        for (int h = 0; h < HW; ++h) {
          const double rden = rcp_f64(fmax(pl[h], 1e-10));
          float o[DPL];
#pragma unroll
          for (int k = 0; k < DPL; ++k) o[k] = (float)(po[h][k] * rden);
          store_lane_vec<D>(a.out + ((size_t)seg_stream * HW + h) * D, o, lane);
        }
      } else {
        finish_alone(seg_stream);
      }
      have_cur = false;
    }
    const bool pub_cur = have_cur;
    bool last_held = false;
    if (held_stream >= 0) {
      const int t = __shfl_sync(kFull, held_ticket, 0);
      last_held = t == held_n - 1;
      if (last_held && lane == 0) counters[(size_t)held_stream * gs + gj] = 0;  // zero-filled again
    }
    if (!pub_cur && !last_held) return;
    bool last_cur = false;
    if (pub_cur) {
      if (pair_merged) {
#pragma unroll
        for (int h = 0; h < HW; ++h) {
          float o[DPL];
#pragma unroll
          for (int k = 0; k < DPL; ++k) o[k] = (float)po[h][k];
          put_record(recs + ((size_t)(gu + seg_stream) * HW + h) * C::REC_BYTES, pm[h], pl[h], o);
        }
      } else {
#pragma unroll
        for (int h = 0; h < HW; ++h) {
          float o[DPL];
#pragma unroll
          for (int k = 0; k < DPL; ++k) o[k] = (float)((double)acc[h][k] - (double)acc_c[h][k]);
          const double lsum = head_l(h), mh = head_m(h);
          put_record(recs + (((size_t)(gu + seg_stream) * gs + gj) * HW + h) * C::REC_BYTES,
                     mh, lsum, o);
        }
      }
      // the warp's record stores, then one release + acquire arrival (the warp
      // barrier orders every lane's stores before the release)
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        int* ctr = &counters[(size_t)seg_stream * gs + gj];
        last = atom_add_acq_rel_gpu(ctr, 1) == n_cur - 1;
        if (last) *ctr = 0;  // leave the workspace zero-filled
      }
      last_cur = __shfl_sync(kFull, last, 0) != 0;
    }
    if (!last_held && !last_cur) return;
    __syncwarp();  // the acquiring lane's view before every lane's record loads
    // one merge site for both streams, so a second merge runs cached code
#pragma unroll 1
    for (int t = 0; t < 2; ++t) {
      if (!(t == 0 ? last_held : last_cur)) continue;
      long long lo = lo_c, hi = hi_c;
      if (t == 0) contributors_of(held_stream, lo, hi);
      if constexpr (HW > 1) merge_stream_heads(t == 0 ? held_stream : seg_stream, lo, hi);
      else merge_stream(t == 0 ? held_stream : seg_stream, lo, hi);
    }
  };

  int st = 0;          // ring slot of page i
  uint32_t phase = 0;  // parity of that slot's mbarrier phase for page i
  for (int i = 0; i < n; ++i) {
    if (i > 0 && (i & 31) == 0) {
      cur = nxt;
      nxt = make_desc(a, s_pfx, page_at(i + 32 + lane), gfirst, g0, g1, bwd);
    }
    char* slot = ring + st * sb;
    const Desc d = shfl_desc(cur, i & 31);
    const int ntok = d.meta & 0xff;
    const bool has_q = (d.meta >> 8) & 1, has_sz = (d.meta >> 9) & 1;

    // every lane waits (each needs the copy's completion); the verdict is made
    // warp-uniform, and group-uniform below, so a timeout never splits a warp
    // or a ring group
    const bool ok = __all_sync(kFull, mbar_wait_bounded(&bar[st], phase, kWaitNs));
    if (!ok && gs == 1) {
      set_status(a.status, kStatusWaitTimeout);
      aborted = true;
      abort_at = i;
      break;
    }

    if (ok) {
      if (has_q) {
        if (seg_stream >= 0) end_segment(seg_stream);
        seg_stream = d.stream;
        if constexpr (HW > 1) {
          long long wl, wh;
          seg_nc = stream_span(seg_stream, wl, wh, seg_g0, seg_g1);
          seg_wlo = (int)wl;
          seg_whi = (int)wh;
        }
#pragma unroll
        for (int h = 0; h < HW; ++h) {
          m_run[h] = -INFINITY;
          l_lane[h] = 0.f;
          l_c[h] = 0.f;
#pragma unroll
          for (int k = 0; k < DPL; ++k) { acc[h][k] = 0.f; acc_c[h][k] = 0.f; }
          // this lane's query channels lane * DPL + j, kept for the segment's groups
          const float* qsrc =
              reinterpret_cast<const float*>(slot + C::Q_OFF + (gj * HW + h) * D * 4) + lane * DPL;
#pragma unroll
          for (int j = 0; j < DPL; j += 2) {
            const float2 x = *reinterpret_cast<const float2*>(qsrc + j);
            qv[h][j] = x.x;
            qv[h][j + 1] = x.y;
          }
        }
      }
      if (has_sz) {
#pragma unroll
        for (int hh = 0; hh < HW; ++hh) {
        // Each lane takes its DPL channels c = lane * DPL + j: q*s, the bias
        // terms and the fixed-point digits; the digits go through the warp's
        // staging bytes to the lanes whose mma B operands hold them (lane
        // (fg, ft): digit fg of channels 64e + 32h + 8ft + [0, 8)).
        const float* sv = reinterpret_cast<const float*>(slot + C::SZ_OFF) + lane * DPL;
        const float* zv = sv + D;
        double qsj[DPL];
        double amax = 0.0, bsum = 0.0;
#pragma unroll
        for (int j = 0; j < DPL; j += 2) {
          const float2 s2 = *reinterpret_cast<const float2*>(sv + j);
          const float2 z2 = *reinterpret_cast<const float2*>(zv + j);
          const float sa[2] = {s2.x, s2.y}, za[2] = {z2.x, z2.y};
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const double qd = (double)qv[hh][j + k], sd = (double)sa[k];
            qsj[j + k] = qd * sd;  // exact product
            amax = fmax(amax, fabs(qsj[j + k]));
            bsum = fma(qd, (double)za[k] * sd, bsum);
          }
        }
        // butterfly sums: every lane ends with the same value
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) bsum += __shfl_xor_sync(kFull, bsum, o);
        if constexpr (HW == 1) bias[hh] = bsum;
        else if (hl == hh) bias[0] = bsum;  // the head whose softmax this lane runs
        // |qs| < 2^E; q and s are float32, so a nonzero product lies in
        // [2^-298, 2^256] and every power of two used below is a normal double
        int bexp = amax > 0.0 ? ((__double2hiint(amax) >> 20) & 0x7FF) : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) bexp = max(bexp, __shfl_xor_sync(kFull, bexp, o));
        const int E = bexp > 0 ? bexp - 1022 : 0;
        const double scale = __hiloint2double((1023 + 56 - E) << 20, 0);
        if constexpr (HW == 1) {
          w0[hh] = __hiloint2double((1023 + E - 7 - 14 * ft) << 20, 0);
          w1[hh] = __hiloint2double((1023 + E - 14 - 14 * ft) << 20, 0);
        } else if (hl == hh) {
          // weight of this lane's first C column in pass 0: digit (2 ft) mod (8 / HW)
          w0[0] = __hiloint2double((1023 + E - 7 - 7 * ((2 * ft) % (8 / HW))) << 20, 0);
        }
        long long X[DPL];
#pragma unroll
        for (int j = 0; j < DPL; ++j) X[j] = __double2ll_rn(qsj[j] * scale);  // |X| < 2^56
        // Two rounds of four digits through the warp's 4*D staging bytes
        // (rows g & 3); the lanes whose digit is in the round load their B operands.
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          __syncwarp();  // the staging bytes (and the page weights aliased on them) are free
#pragma unroll
          for (int g4 = 0; g4 < 4; ++g4) {  // digit g: bits [49 - 7g, 56 - 7g) of X, the top one signed
            const int g = 4 * half + g4;
            const int sh = 49 - 7 * g;
            const long long m = g == 0 ? 0xFF : 0x7F;
            uint8_t* row = dig + g4 * kDigRow + lane * DPL;
            if constexpr (DPL == 2) {
              *reinterpret_cast<uint16_t*>(row) = (uint16_t)(((X[0] >> sh) & m) | (((X[1] >> sh) & m) << 8));
            } else {
#pragma unroll
              for (int j4 = 0; j4 < DPL; j4 += 4) {
                *reinterpret_cast<uint32_t*>(row + j4) =
                    (uint32_t)(((X[j4] >> sh) & m) | (((X[j4 + 1] >> sh) & m) << 8) |
                               (((X[j4 + 2] >> sh) & m) << 16) | (((X[j4 + 3] >> sh) & m) << 24));
              }
            }
          }
          __syncwarp();
          if constexpr (HW == 1) {
            if ((fg >> 2) == half) {
#pragma unroll
              for (int e = 0; e < C::KT; ++e) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                  const uint2 v =
                      *reinterpret_cast<const uint2*>(dig + (fg & 3) * kDigRow + 64 * e + 32 * hf + 8 * ft);
                  bfrag[hh][2 * e][hf] = __byte_perm(v.x, v.y, 0x6420);      // even channels
                  bfrag[hh][2 * e + 1][hf] = __byte_perm(v.x, v.y, 0x7531);  // odd channels
                }
              }
            }
          } else if ((fg * HW) / 8 == hh) {
            // B role: this lane holds column fg = (head fg * HW / 8, digit
            // p * (8 / HW) + fg % (8 / HW)) of every pass p
#pragma unroll
            for (int pp = 0; pp < HW; ++pp) {
              const int dg = pp * (8 / HW) + fg % (8 / HW);
              if ((dg >> 2) == half) {
#pragma unroll
                for (int e = 0; e < C::KT; ++e) {
#pragma unroll
                  for (int hf = 0; hf < 2; ++hf) {
                    const uint2 v = *reinterpret_cast<const uint2*>(dig + (dg & 3) * kDigRow + 64 * e +
                                                                   32 * hf + 8 * ft);
                    bfrag[pp][2 * e][hf] = __byte_perm(v.x, v.y, 0x6420);      // even channels
                    bfrag[pp][2 * e + 1][hf] = __byte_perm(v.x, v.y, 0x7531);  // odd channels
                  }
                }
              }
            }
          }
        }
        __syncwarp();  // staging read before the page weights overwrite it
        }
      }

      if (ntok > 0) {
        // ---- logits of tokens fg and fg + 8 (every lane of the row group) ----
        const char* krow = slot + C::K_OFF + ((lane & 7) + 8 * ((lane >> 3) & 1)) * (D / 2) +
                           16 * (lane >> 4);
        // float32 pools with one head per warp: four independent MMA chains
        // (even / odd channels x even / odd 32-byte chunk) instead of one chain
        // of 2 KT -- integer sums, so the split changes no bit of the result;
        // measured 63.2 -> 62.2 us at config 0. The 16-bit pools keep one chain
        // (their GQA step measured 0.8 us slower with four), and so do warps
        // serving several heads, whose heads are independent chains already.
        constexpr bool kSplit = VK == 0 && HW == 1;
        constexpr int NCH = kSplit ? 4 : 1;
        int cs[HW][NCH][4];
#pragma unroll
        for (int h = 0; h < HW; ++h)
#pragma unroll
          for (int c4 = 0; c4 < NCH; ++c4) cs[h][c4][0] = cs[h][c4][1] = cs[h][c4][2] = cs[h][c4][3] = 0;
#pragma unroll
        for (int e = 0; e < C::KT; ++e) {
          uint32_t r[4];
          ldmatrix_x4(r, krow + 32 * e);
          const uint32_t lo[4] = {r[0] & 0x0F0F0F0Fu, r[1] & 0x0F0F0F0Fu, r[2] & 0x0F0F0F0Fu,
                                  r[3] & 0x0F0F0F0Fu};
          const uint32_t hi[4] = {(r[0] >> 4) & 0x0F0F0F0Fu, (r[1] >> 4) & 0x0F0F0F0Fu,
                                  (r[2] >> 4) & 0x0F0F0F0Fu, (r[3] >> 4) & 0x0F0F0F0Fu};
#pragma unroll
          for (int h = 0; h < HW; ++h) {
            mma_u8s8_16832(cs[h][kSplit ? 2 * (e & 1) : 0], lo, bfrag[h][2 * e][0], bfrag[h][2 * e][1]);
            mma_u8s8_16832(cs[h][kSplit ? 2 * (e & 1) + 1 : 0], hi, bfrag[h][2 * e + 1][0],
                           bfrag[h][2 * e + 1][1]);
          }
        }
        if constexpr (HW == 1) {
          if constexpr (kSplit) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
              cs[0][0][k] = (cs[0][0][k] + cs[0][1 % NCH][k]) + (cs[0][2 % NCH][k] + cs[0][3 % NCH][k]);
          }
          // digits 2ft, 2ft + 1 weigh 128 w1 and w1: their int32 combination is
          // exact (|sum| < 2^25), so this is the float64 value of both terms
          double x0 = (double)(cs[0][0][0] * 128 + cs[0][0][1]) * w1[0];
          double x1 = (double)(cs[0][0][2] * 128 + cs[0][0][3]) * w1[0];
          x0 += __shfl_xor_sync(kFull, x0, 1);
          x1 += __shfl_xor_sync(kFull, x1, 1);
          x0 += __shfl_xor_sync(kFull, x0, 2);
          x1 += __shfl_xor_sync(kFull, x1, 2);
          const double lg0 = fg < ntok ? x0 - bias[0] : -INFINITY;
          const double lg1 = fg + 8 < ntok ? x1 - bias[0] : -INFINITY;

          // ---- online softmax: rescale only when the running max moves ----
          if (__any_sync(kFull, lg0 > m_run[0] || lg1 > m_run[0])) {
            double pmax = fmax(lg0, lg1);
#pragma unroll
            for (int o = 16; o > 2; o >>= 1) pmax = fmax(pmax, __shfl_xor_sync(kFull, pmax, o));
            const double m_new = fmax(m_run[0], pmax);
            const float corr = exp_neg(m_run[0] - m_new);
            l_lane[0] *= corr;
            l_c[0] *= corr;
#pragma unroll
            for (int k = 0; k < DPL; ++k) { acc[0][k] *= corr; acc_c[0][k] *= corr; }
            m_run[0] = m_new;
          }
          const float p0 = exp_neg(lg0 - m_run[0]), p1 = exp_neg(lg1 - m_run[0]);
          if (ft == 0) {  // one lane per row group owns tokens fg and fg + 8
            kahan_rescale_add(l_lane[0], l_c[0], 1.f, p0);
            kahan_rescale_add(l_lane[0], l_c[0], 1.f, p1);
            p_tab[fg] = p0;
            p_tab[fg + 8] = p1;
          }
        } else {
          // Column heads: pass p's C columns 2ft, 2ft + 1 are two digits of head
          // hl, weighted 2^(E - 7 - 7 dg); the passes advance dg by 8 / HW.
          double x0 = 0.0, x1 = 0.0, wa = w0[0];
          constexpr double kStep = HW == 4 ? 0x1p-14 : 0x1p-28;  // 2^(-7 * 8 / HW)
#pragma unroll
          for (int pp = 0; pp < HW; ++pp) {
            // the column's two digits (the second 2^-7 lower), combined exactly
            // in int32 (|sum| < 2^25) and weighed once
            const double wb = wa * 0.0078125;
            x0 = fma((double)(cs[pp][0][0] * 128 + cs[pp][0][1]), wb, x0);
            x1 = fma((double)(cs[pp][0][2] * 128 + cs[pp][0][3]), wb, x1);
            wa *= kStep;
          }
          if constexpr (HW == 2) {  // lanes ft and ft ^ 1 hold complementary digits of a head
            x0 += __shfl_xor_sync(kFull, x0, 1);
            x1 += __shfl_xor_sync(kFull, x1, 1);
          }
          const double lg0 = fg < ntok ? x0 - bias[0] : -INFINITY;
          const double lg1 = fg + 8 < ntok ? x1 - bias[0] : -INFINITY;

          // ---- online softmax of head hl across its lanes (g = 0..7) ----
          double pmax = fmax(lg0, lg1);
          pmax = fmax(pmax, __shfl_xor_sync(kFull, pmax, 4));
          pmax = fmax(pmax, __shfl_xor_sync(kFull, pmax, 8));
          pmax = fmax(pmax, __shfl_xor_sync(kFull, pmax, 16));
          if (__any_sync(kFull, pmax > m_run[0])) {
            const double m_new = fmax(m_run[0], pmax);
            const float corr = exp_neg(m_run[0] - m_new);  // exactly 1 when unmoved
            l_lane[0] *= corr;
            l_c[0] *= corr;
            m_run[0] = m_new;
#pragma unroll
            for (int h = 0; h < HW; ++h) {  // every lane holds channels of every head
              const float ch = __shfl_sync(kFull, corr, head_src(h));
              if (ch != 1.f) {
#pragma unroll
                for (int k = 0; k < DPL; ++k) { acc[h][k] *= ch; acc_c[h][k] *= ch; }
              }
            }
          }
          const float p0 = exp_neg(lg0 - m_run[0]), p1 = exp_neg(lg1 - m_run[0]);
          if (HW == 4 || (ft & 1) == 0) {  // one lane per (row group, head)
            kahan_rescale_add(l_lane[0], l_c[0], 1.f, p0);
            kahan_rescale_add(l_lane[0], l_c[0], 1.f, p1);
            p_tab[fg * HW + hl] = p0;
            p_tab[(fg + 8) * HW + hl] = p1;
          }
        }
        __syncwarp();

        // ---- P.V over the page's valid rows (float32 page sums, Kahan into the run);
        // each value row is loaded once for all HW heads ----
        const char* vs = slot + C::V_OFF;
        float ps[HW][DPL];
#pragma unroll
        for (int h = 0; h < HW; ++h)
#pragma unroll
          for (int k = 0; k < DPL; ++k) ps[h][k] = 0.f;
        if constexpr (HW == 1) {
          if (ntok == kPage) {
#if I4KV_PV_TWO_CHAINS
            // even and odd rows into separate sums: half the FMA chain depth
            float pq[DPL];
#pragma unroll
            for (int k = 0; k < DPL; ++k) pq[k] = 0.f;
#pragma unroll
            for (int t4 = 0; t4 < kPage / 4; ++t4) {
              const float4 pt = reinterpret_cast<const float4*>(p_tab)[t4];
              pv_row<D, VK>(vs, pt.x, 4 * t4 + 0, lane, ps[0]);
              pv_row<D, VK>(vs, pt.y, 4 * t4 + 1, lane, pq);
              pv_row<D, VK>(vs, pt.z, 4 * t4 + 2, lane, ps[0]);
              pv_row<D, VK>(vs, pt.w, 4 * t4 + 3, lane, pq);
            }
#pragma unroll
            for (int k = 0; k < DPL; ++k) ps[0][k] += pq[k];
#else
#pragma unroll
            for (int t4 = 0; t4 < kPage / 4; ++t4) {
              const float4 pt = reinterpret_cast<const float4*>(p_tab)[t4];
              pv_row<D, VK>(vs, pt.x, 4 * t4 + 0, lane, ps[0]);
              pv_row<D, VK>(vs, pt.y, 4 * t4 + 1, lane, ps[0]);
              pv_row<D, VK>(vs, pt.z, 4 * t4 + 2, lane, ps[0]);
              pv_row<D, VK>(vs, pt.w, 4 * t4 + 3, lane, ps[0]);
            }
#endif
          } else {
#pragma unroll
            for (int t = 0; t < kPage; ++t)
              if (t < ntok) pv_row<D, VK>(vs, p_tab[t], t, lane, ps[0]);
          }
        } else {
#pragma unroll 4
          for (int t = 0; t < ntok; ++t) pv_row_heads<D, VK, HW>(vs, p_tab + t * HW, t, lane, ps);
        }
#pragma unroll
        for (int h = 0; h < HW; ++h)
#pragma unroll
          for (int k = 0; k < DPL; k += 2)
            kahan_add2(acc[h][k], acc[h][k + 1], acc_c[h][k], acc_c[h][k + 1], ps[h][k], ps[h][k + 1]);
      }

    }
    // the slot is free once every warp of the group is done with it
    if (gs == 1) {
      __syncwarp();
    } else if (named_bar_or(1 + gi, gs * 32, !ok)) {
      if (!ok) set_status(a.status, kStatusWaitTimeout);
      aborted = true;
      abort_at = i;
      break;
    }
    const int nx = i + depth;
    if (nx < n && paired && !claim(nx)) n = nx;  // the partner took it: this warp's pages end at nx
    if (nx < n) {
      const int src = nx & 31;
      const Desc dn = (nx >> 5) == (i >> 5) ? shfl_desc(cur, src) : shfl_desc(nxt, src);
      if (leader && lane == 0) issue_page<D, WARPS, STAGES, VK>(a, dn, slot, &bar[st]);
    }
    if (++st == depth) {
      st = 0;
      phase ^= 1u;
    }
  }

  if constexpr (I4KV_DECODE_PDL) allow_dependent_launch();
  if (aborted) {
    // The group's leader drains what the ring still has in flight (bounded)
    // before leaving, so no bulk copy lands in shared memory after the CTA
    // has exited.
    if (leader)
      for (int k = abort_at; k < n && k < abort_at + depth; ++k)
        (void)mbar_wait_bounded(&bar[k % depth], (uint32_t)((k / depth) & 1), kWaitNs);
    return;
  }
  end_run();
  if (xmode) {
    // every push of this warp is out; now wait for the other ranks and merge:
    // the streams it finished alone (the interior of its run), the ones it
    // merged as the last local arrival, and its share of the empty streams
    bool dead = false;
    x_empty_streams<D>(a, s_pfx, streams, gw, NW, gs, gj, lane, false, dead);
    const int v_first = make_desc(a, s_pfx, g0, g0, g0, g1, false).stream;
    const int v_last = make_desc(a, s_pfx, g1 - 1, g0, g0, g1, false).stream;
    for (int vs = v_first; vs <= v_last; ++vs) {
      const int b = vs / a.vheads;
      if (s_pfx[b + 1] == s_pfx[b]) continue;  // no pages here: an empty stream's duty
      long long lo, hi;
      if (contributors_of(vs, lo, hi) == 1) x_finish<D>(a, streams, (long long)vs * gs + gj, lane, dead);
    }
    if (xm0 >= 0) x_finish<D>(a, streams, (long long)xm0 * gs + gj, lane, dead);
    if (xm1 >= 0) x_finish<D>(a, streams, (long long)xm1 * gs + gj, lane, dead);
    x_empty_streams<D>(a, s_pfx, streams, gw, NW, gs, gj, lane, true, dead);
  }
}

// Merge per-GPU partial records [parts][streams] of one decode step into
// outputs: the log-sum-exp combine of the reference's warp merge
// (csrc/flash_decode_int4.cu:199-220: M = max m, L = sum l*e^(m-M),
// out = sum acc*e^(m-M) / max(L, 1e-10), parts with m = -inf skipped), in
// float64. One warp per stream.
template <int D>
__global__ void __launch_bounds__(256) merge_partials_kernel(const char* parts, int num_parts,
                                                              int streams, float* out) {
  constexpr int DPL = D / 32;
  constexpr int REC_BYTES = 16 + 4 * D;  // [m f64][l f64][acc D f32]
  const int lane = threadIdx.x & 31;
  const long long s = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (s >= streams) return;
  const size_t stride = (size_t)streams * REC_BYTES;
  const char* base = parts + (size_t)s * REC_BYTES;
  double M = -INFINITY;
  for (int p = 0; p < num_parts; ++p) M = fmax(M, *reinterpret_cast<const double*>(base + p * stride));
  double L = 0.0, O[DPL];
#pragma unroll
  for (int k = 0; k < DPL; ++k) O[k] = 0.0;
  if (M != -INFINITY) {
    for (int p = 0; p < num_parts; ++p) {
      const char* r = base + p * stride;
      const double m = *reinterpret_cast<const double*>(r);
      if (m == -INFINITY) continue;
      const double e = exp(m - M);
      L = fma(*reinterpret_cast<const double*>(r + 8), e, L);
      float v[DPL];
      load_lane_vec_cg<D>(reinterpret_cast<const float*>(r + 16), v, lane);
#pragma unroll
      for (int k = 0; k < DPL; ++k) O[k] = fma((double)v[k], e, O[k]);
    }
  }
  const double den = fmax(L, 1e-10);
  float o[DPL];
#pragma unroll
  for (int k = 0; k < DPL; ++k) o[k] = (float)(O[k] / den);
  store_lane_vec<D>(out + (size_t)s * D, o, lane);
}

// ---- host side ----
#ifndef I4KV_DECODE_WARPS
#define I4KV_DECODE_WARPS 4
#endif
#ifndef I4KV_DECODE_STAGES
#define I4KV_DECODE_STAGES 2
#endif
#ifndef I4KV_DECODE_MAX_CTAS_F32
#define I4KV_DECODE_MAX_CTAS_F32 0
#endif
#ifndef I4KV_DECODE_MAX_CTAS_16
#define I4KV_DECODE_MAX_CTAS_16 3  // measured: 45.5 us at config 0 vs 46.5 (4) and 53.5 (2)
#endif
constexpr int kWarps = I4KV_DECODE_WARPS;    // warps per CTA
constexpr int kStages = I4KV_DECODE_STAGES;  // ring slots per warp
// CTAs per SM for the grid (0: as many as fit), float32 and 16-bit value pools
constexpr int kMaxCtasF32 = I4KV_DECODE_MAX_CTAS_F32;
constexpr int kMaxCtas16 = I4KV_DECODE_MAX_CTAS_16;

// Query heads per warp for GQA ratio g at head dim d: four when 4 divides g
// (at d <= 128: the per-head registers of d256 do not fit four), else two
// when 2 does, so a warp stages, unpacks and reads each kv page once for
// those heads, and warps pair up on one run as in plain decode; otherwise one
// head per warp, the warps of a ring group sharing each staged page. The
// fused split exchange runs one head per warp.
// Measured at config 0's shape with 32 query heads, L2 flushed (one B200):
// G = 4: 39.9 us (float32 values) with four heads per warp against 45.1 us
// with one; G = 2: 41.0 us with two against 45. Groups of four-head warps
// sharing a page (G = 8 as two-warp groups) measured 45-56 us: no warp pairs
// in a ring group, and each stream's many records are merged by one warp at
// the end; so multi-head warps run alone, one run of pages per pair.
#ifndef I4KV_MAX_HEADS_PER_WARP
#define I4KV_MAX_HEADS_PER_WARP 4
#endif
int heads_per_warp(int g, int d, bool xmode) {
  constexpr int kMaxHw = I4KV_MAX_HEADS_PER_WARP;
  if (xmode) return 1;
  if (kMaxHw >= 4 && g % 4 == 0 && d <= 128) return 4;
  if (kMaxHw >= 2 && g % 2 == 0) return 2;
  return 1;
}

// Warps sharing one ring: one for multi-head warps; else the largest divisor
// of kWarps (a power of two) that divides g, so a CTA holds whole groups of
// query heads.
int ring_group(int num_q_heads, int num_kv_heads, int hw) {
  if (hw > 1) return 1;
  const int g = num_q_heads / num_kv_heads;
  int x = kWarps;
  while (g % x) x >>= 1;
  return x;
}

template <int D, int VK>
size_t dyn_smem(int batch, int gs, int hw) {
  using C = Cfg<D, kWarps, kStages, VK>;
  const size_t ring_slots = gs == 1 ? (size_t)kWarps * kStages
                                     : (size_t)kWarps * I4KV_GQA_RING_PAGES_PER_WARP;  // groups x depth
  return 256 + pfx_bytes(batch) + ring_slots * (C::Q_OFF + (size_t)gs * hw * D * 4) +
         (size_t)kWarps * 4 * (D + 32);  // rings, then per-warp digit staging / page weights
}

struct OccCache {
  std::mutex mu;
  int dev[128] = {};
  int key[128] = {};  // ((D * 4 + value kind) * 8 + ring group) * 8 + heads per warp
  size_t smem[128] = {};
  int grid[128] = {};
  int n = 0;
  // Dynamic shared-memory opt-in per (device, kernel): only ever raised, so a
  // launch whose grid came from the cache never exceeds the kernel's limit.
  int attr_dev[128] = {};
  int attr_key[128] = {};  // (D * 4 + value kind) * 8 + heads per warp
  size_t attr_max[128] = {};
  int n_attr = 0;
};
OccCache g_occ;

// Raise the kernel's dynamic shared-memory limit on `dev` to at least `smem`.
template <typename K>
cudaError_t ensure_smem_attr(K kern, int dev, int kkey, size_t smem) {
  std::lock_guard<std::mutex> lk(g_occ.mu);
  int i = 0;
  while (i < g_occ.n_attr && !(g_occ.attr_dev[i] == dev && g_occ.attr_key[i] == kkey)) ++i;
  if (i < g_occ.n_attr && g_occ.attr_max[i] >= smem) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if (i == g_occ.n_attr) {
    if (g_occ.n_attr == 128) return cudaSuccess;  // 24 kernels x 5 devices fit; never reached
    g_occ.attr_dev[i] = dev;
    g_occ.attr_key[i] = kkey;
    ++g_occ.n_attr;
  }
  g_occ.attr_max[i] = smem;
  return cudaSuccess;
}

template <int D, int VK, int HW>
cudaError_t decode_grid(int batch, int gs, int* grid_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const size_t smem = dyn_smem<D, VK>(batch, gs, HW);
  const int key = ((D * 4 + VK) * 8 + gs) * 8 + HW;
  {
    std::lock_guard<std::mutex> lk(g_occ.mu);
    for (int i = 0; i < g_occ.n; ++i)
      if (g_occ.dev[i] == dev && g_occ.key[i] == key && g_occ.smem[i] == smem) {
        *grid_out = g_occ.grid[i];
        return cudaSuccess;
      }
  }
  auto kern = paged_decode_kernel<D, kWarps, kStages, VK, HW>;
  e = ensure_smem_attr(kern, dev, (D * 4 + VK) * 8 + HW, smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0, sms = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kWarps * 32, smem);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  if (per_sm <= 0) return cudaErrorInvalidConfiguration;
  const int cap = VK == 0 ? kMaxCtasF32 : kMaxCtas16;
  if (cap > 0 && per_sm > cap) per_sm = cap;
  const int grid = per_sm * sms;
  {
    std::lock_guard<std::mutex> lk(g_occ.mu);
    if (g_occ.n < 128) {
      g_occ.dev[g_occ.n] = dev; g_occ.key[g_occ.n] = key; g_occ.smem[g_occ.n] = smem;
      g_occ.grid[g_occ.n] = grid; ++g_occ.n;
    }
  }
  *grid_out = grid;
  return cudaSuccess;
}

// Records: one per (warp, head) slot of the grid plus one per query stream.
template <int D, int VK, int HW>
cudaError_t ws_size_hw(int batch, int heads, int gs, size_t* out) {
  int grid = 0;
  cudaError_t e = decode_grid<D, VK, HW>(batch, gs, &grid);
  if (e != cudaSuccess) return e;
  const long long streams = (long long)batch * heads;
  const size_t nrec = (size_t)grid * kWarps * HW + (size_t)streams;
  *out = cnt_bytes(streams) + nrec * Cfg<D, kWarps, kStages, VK>::REC_BYTES;
  return cudaSuccess;
}

template <int D, int VK>
cudaError_t ws_size_one(int batch, int heads, int kv_heads, int hw, size_t* out) {
  const int gs = ring_group(heads, kv_heads, hw);
  switch (hw) {
    case 4:
      if constexpr (D <= 128 && I4KV_MAX_HEADS_PER_WARP >= 4)
        return ws_size_hw<D, VK, 4>(batch, heads, gs, out);
      return cudaErrorInvalidValue;
    case 2:
      if constexpr (I4KV_MAX_HEADS_PER_WARP >= 2) return ws_size_hw<D, VK, 2>(batch, heads, gs, out);
      return cudaErrorInvalidValue;
    default: return ws_size_hw<D, VK, 1>(batch, heads, gs, out);
  }
}

// The workspace of a (batch, heads) shape: enough for the heads-per-warp the
// plain decode uses and for the one head per warp of the fused split.
template <int D, int VK>
cudaError_t ws_size(int batch, int heads, int kv_heads, size_t* out) {
  const int g = heads / kv_heads;
  size_t a = 0, b = 0;
  cudaError_t e = ws_size_one<D, VK>(batch, heads, kv_heads, heads_per_warp(g, D, false), &a);
  if (e != cudaSuccess) return e;
  e = ws_size_one<D, VK>(batch, heads, kv_heads, 1, &b);
  if (e != cudaSuccess) return e;
  *out = a > b ? a : b;
  return cudaSuccess;
}

template <int D, int VK, int HW>
cudaError_t launch_hw(const DecodeArgs& a, size_t ws_bytes, cudaStream_t stream,
                      cudaEvent_t ev_before, cudaEvent_t ev_after) {
  int grid = 0;
  cudaError_t e = decode_grid<D, VK, HW>(a.batch, a.gs, &grid);
  if (e != cudaSuccess) return e;
  size_t need = 0;
  e = ws_size_hw<D, VK, HW>(a.batch, a.heads, a.gs, &need);
  if (e != cudaSuccess) return e;
  if (ws_bytes < need) return cudaErrorInvalidValue;
  if (ev_before && (e = cudaEventRecord(ev_before, stream)) != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = dyn_smem<D, VK>(a.batch, a.gs, HW);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = I4KV_DECODE_PDL ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, paged_decode_kernel<D, kWarps, kStages, VK, HW>, a);
  if (e != cudaSuccess) return e;
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (ev_after && (e = cudaEventRecord(ev_after, stream)) != cudaSuccess) return e;
  return cudaSuccess;
}

template <int D, int VK>
cudaError_t launch(const DecodeArgs& a, size_t ws_bytes, cudaStream_t stream,
                   cudaEvent_t ev_before, cudaEvent_t ev_after) {
  switch (a.hw) {
    case 4:
      if constexpr (D <= 128 && I4KV_MAX_HEADS_PER_WARP >= 4)
        return launch_hw<D, VK, 4>(a, ws_bytes, stream, ev_before, ev_after);
      return cudaErrorInvalidValue;
    case 2:
      if constexpr (I4KV_MAX_HEADS_PER_WARP >= 2)
        return launch_hw<D, VK, 2>(a, ws_bytes, stream, ev_before, ev_after);
      return cudaErrorInvalidValue;
    default: return launch_hw<D, VK, 1>(a, ws_bytes, stream, ev_before, ev_after);
  }
}

template <int D>
cudaError_t launch_kind(int vk, const DecodeArgs& a, size_t ws_bytes, cudaStream_t stream,
                        cudaEvent_t ev_before, cudaEvent_t ev_after) {
  switch (vk) {
    case INT4KV_VALUES_F32: return launch<D, 0>(a, ws_bytes, stream, ev_before, ev_after);
    case INT4KV_VALUES_F16: return launch<D, 1>(a, ws_bytes, stream, ev_before, ev_after);
    case INT4KV_VALUES_BF16: return launch<D, 2>(a, ws_bytes, stream, ev_before, ev_after);
    default: return cudaErrorInvalidValue;
  }
}

template <int D>
cudaError_t ws_size_kind(int vk, int batch, int heads, int kv_heads, size_t* out) {
  switch (vk) {
    case INT4KV_VALUES_F32: return ws_size<D, 0>(batch, heads, kv_heads, out);
    case INT4KV_VALUES_F16: return ws_size<D, 1>(batch, heads, kv_heads, out);
    case INT4KV_VALUES_BF16: return ws_size<D, 2>(batch, heads, kv_heads, out);
    default: return cudaErrorInvalidValue;
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Argument checks shared by the decode entry points, then the launch. Exactly
// one of `out` (normalized outputs) and `part_out` (partial records) is used.
cudaError_t paged_entry(const float* query, const uint8_t* k_pool, const void* v_pool, int vk,
                        const float* sz_pool, const int32_t* block_table, const int32_t* seq_lens,
                        int batch, int num_q_heads, int num_kv_heads, int head_dim,
                        int page_tokens, int group_tokens, int max_pages, int num_pages,
                        float* out, char* part_out, void* workspace, size_t workspace_bytes,
                        uint32_t* status, cudaStream_t stream, cudaEvent_t ev_before,
                        cudaEvent_t ev_after, int xworld = 0, int xrank = 0,
                        void* const* xbufs = nullptr) {
  if (batch <= 0 || batch > kMaxPagedBatch || num_kv_heads <= 0 || num_q_heads < num_kv_heads ||
      num_q_heads % num_kv_heads != 0)
    return cudaErrorInvalidValue;
  if (page_tokens != kPage || group_tokens <= 0 || group_tokens % kPage != 0) return cudaErrorInvalidValue;
  if (max_pages <= 0 || num_pages <= 0) return cudaErrorInvalidValue;
  if ((long long)batch * num_q_heads * max_pages >= (1LL << 31) - 1024) return cudaErrorInvalidValue;
  if (!query || !k_pool || !v_pool || !sz_pool || !block_table || !seq_lens || !workspace)
    return cudaErrorInvalidValue;
  if (!out && !part_out) return cudaErrorInvalidValue;
  if (!al16(query) || !al16(k_pool) || !al16(v_pool) || !al16(sz_pool) || !al16(workspace))
    return cudaErrorInvalidValue;
  if ((out && !al16(out)) || (part_out && !al16(part_out))) return cudaErrorInvalidValue;
  DecodeArgs a{query, k_pool, v_pool, sz_pool, block_table, seq_lens, out, batch, num_q_heads,
               max_pages, num_pages, group_tokens / kPage, static_cast<char*>(workspace), status,
               part_out, num_kv_heads, num_q_heads / num_kv_heads, 1, 1, 0};
  a.hw = heads_per_warp(num_q_heads / num_kv_heads, head_dim, xworld > 0);
  a.gs = ring_group(num_q_heads, num_kv_heads, a.hw);
  a.vheads = num_q_heads / (a.gs * a.hw);
  if (xworld > 0) {  // fused split exchange: outputs merged over the ranks' records
    if (xworld > kXRanks || xrank < 0 || xrank >= xworld || !xbufs || part_out || !out)
      return cudaErrorInvalidValue;
    for (int r = 0; r < xworld; ++r) {
      if (!xbufs[r] || (reinterpret_cast<uintptr_t>(xbufs[r]) & 127u)) return cudaErrorInvalidValue;
      a.xbuf[r] = static_cast<char*>(xbufs[r]);
    }
    a.xworld = xworld;
    a.xrank = xrank;
  }
  switch (head_dim) {
    case 64: return launch_kind<64>(vk, a, workspace_bytes, stream, ev_before, ev_after);
    case 128: return launch_kind<128>(vk, a, workspace_bytes, stream, ev_before, ev_after);
    case 256: return launch_kind<256>(vk, a, workspace_bytes, stream, ev_before, ev_after);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

extern "C" {

cudaError_t int4kv_paged_decode_workspace_size(int batch, int num_q_heads, int num_kv_heads,
                                               int head_dim, size_t* bytes) {
  if (!bytes || batch <= 0 || num_kv_heads <= 0 || num_q_heads < num_kv_heads ||
      num_q_heads % num_kv_heads != 0)
    return cudaErrorInvalidValue;
  if (batch > kMaxPagedBatch) return cudaErrorInvalidValue;
  switch (head_dim) {
    case 64: return ws_size<64, 0>(batch, num_q_heads, num_kv_heads, bytes);
    case 128: return ws_size<128, 0>(batch, num_q_heads, num_kv_heads, bytes);
    case 256: return ws_size<256, 0>(batch, num_q_heads, num_kv_heads, bytes);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t int4kv_paged_decode_workspace_size_ex(int batch, int num_q_heads, int num_kv_heads,
                                                  int head_dim, int value_dtype, size_t* bytes) {
  if (!bytes || batch <= 0 || num_kv_heads <= 0 || num_q_heads < num_kv_heads ||
      num_q_heads % num_kv_heads != 0)
    return cudaErrorInvalidValue;
  if (batch > kMaxPagedBatch) return cudaErrorInvalidValue;
  switch (head_dim) {
    case 64: return ws_size_kind<64>(value_dtype, batch, num_q_heads, num_kv_heads, bytes);
    case 128: return ws_size_kind<128>(value_dtype, batch, num_q_heads, num_kv_heads, bytes);
    case 256: return ws_size_kind<256>(value_dtype, batch, num_q_heads, num_kv_heads, bytes);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t int4kv_paged_decode_ex(const float* query, const uint8_t* k_pool, const void* v_pool,
                                   int value_dtype, const float* sz_pool,
                                   const int32_t* block_table, const int32_t* seq_lens, int batch,
                                   int num_q_heads, int num_kv_heads, int head_dim,
                                   int page_tokens, int group_tokens, int max_pages, int num_pages,
                                   float* out, void* workspace, size_t workspace_bytes,
                                   uint32_t* status, cudaStream_t stream, cudaEvent_t ev_before,
                                   cudaEvent_t ev_after) {
  return paged_entry(query, k_pool, v_pool, value_dtype, sz_pool, block_table, seq_lens, batch,
                     num_q_heads, num_kv_heads, head_dim, page_tokens, group_tokens, max_pages,
                     num_pages, out, nullptr, workspace, workspace_bytes, status, stream,
                     ev_before, ev_after);
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
  return paged_entry(query, k_pool, v_pool, INT4KV_VALUES_F32, sz_pool, block_table, seq_lens,
                     batch, num_q_heads,
                     num_kv_heads, head_dim, page_tokens, group_tokens, max_pages, num_pages, out,
                     nullptr, workspace, workspace_bytes, status, stream, ev_before, ev_after);
}

cudaError_t int4kv_paged_decode_partials(const float* query, const uint8_t* k_pool,
                                         const float* v_pool, const float* sz_pool,
                                         const int32_t* block_table, const int32_t* seq_lens,
                                         int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                         int page_tokens, int group_tokens, int max_pages,
                                         int num_pages, void* partials, void* workspace,
                                         size_t workspace_bytes, uint32_t* status,
                                         cudaStream_t stream) {
  return int4kv_paged_decode_partials_ex(query, k_pool, v_pool, INT4KV_VALUES_F32, sz_pool,
                                         block_table, seq_lens, batch, num_q_heads, num_kv_heads,
                                         head_dim, page_tokens, group_tokens, max_pages, num_pages,
                                         partials, workspace, workspace_bytes, status, stream);
}

cudaError_t int4kv_paged_decode_partials_ex(const float* query, const uint8_t* k_pool,
                                            const void* v_pool, int value_dtype,
                                            const float* sz_pool, const int32_t* block_table,
                                            const int32_t* seq_lens, int batch, int num_q_heads,
                                            int num_kv_heads, int head_dim, int page_tokens,
                                            int group_tokens, int max_pages, int num_pages,
                                            void* partials, void* workspace,
                                            size_t workspace_bytes, uint32_t* status,
                                            cudaStream_t stream) {
  if (!partials) return cudaErrorInvalidValue;
  return paged_entry(query, k_pool, v_pool, value_dtype, sz_pool, block_table, seq_lens, batch,
                     num_q_heads, num_kv_heads, head_dim, page_tokens, group_tokens, max_pages,
                     num_pages, nullptr, static_cast<char*>(partials), workspace, workspace_bytes,
                     status, stream, nullptr, nullptr);
}

cudaError_t int4kv_merge_partials(const void* partials, int num_parts, int streams, int head_dim,
                                  float* out, cudaStream_t stream) {
  if (!partials || !out || num_parts <= 0 || streams <= 0) return cudaErrorInvalidValue;
  if (!al16(partials) || !al16(out)) return cudaErrorInvalidValue;
  const int warps = 8;
  const unsigned grid = (unsigned)((streams + warps - 1) / warps);
  const char* p = static_cast<const char*>(partials);
  switch (head_dim) {
    case 64: merge_partials_kernel<64><<<grid, warps * 32, 0, stream>>>(p, num_parts, streams, out); break;
    case 128: merge_partials_kernel<128><<<grid, warps * 32, 0, stream>>>(p, num_parts, streams, out); break;
    case 256: merge_partials_kernel<256><<<grid, warps * 32, 0, stream>>>(p, num_parts, streams, out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t int4kv_paged_decode_split_bytes(int batch, int num_q_heads, int head_dim,
                                            size_t* bytes) {
  if (!bytes || batch <= 0 || num_q_heads <= 0) return cudaErrorInvalidValue;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return cudaErrorInvalidValue;
  *bytes = x_bytes((long long)batch * num_q_heads, head_dim);
  return cudaSuccess;
}

cudaError_t int4kv_paged_decode_split(const float* query, const uint8_t* k_pool,
                                      const void* v_pool, int value_dtype, const float* sz_pool,
                                      const int32_t* block_table, const int32_t* seq_lens,
                                      int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                      int page_tokens, int group_tokens, int max_pages,
                                      int num_pages, void* const* peer_bufs, int world, int rank,
                                      float* out, void* workspace, size_t workspace_bytes,
                                      uint32_t* status, cudaStream_t stream) {
  if (world <= 0 || !peer_bufs) return cudaErrorInvalidValue;
  return paged_entry(query, k_pool, v_pool, value_dtype, sz_pool, block_table, seq_lens, batch,
                     num_q_heads, num_kv_heads, head_dim, page_tokens, group_tokens, max_pages,
                     num_pages, out, nullptr, workspace, workspace_bytes, status, stream, nullptr,
                     nullptr, world, rank, peer_bufs);
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

// ---------------------------------------------------------------------------
// Allocation-free variant: the same decode kernel, with its scratch (per-stream
// arrival counters + partial records) taken from a fixed device array instead
// of a caller-provided workspace. It serves callers that cannot allocate
// device memory on the decode path: a host runtime bound through the C ABI
// (a cgo / JNI / ctypes stub) that has no device allocator of its own, and a
// serving step whose device memory is fully reserved up front, where a
// cudaMalloc would fail or implicitly synchronize the device and stall the
// other streams.
//
// Contract:
//   * scratch is the file-scope array below, INT4KV_STATIC_SCRATCH_BYTES per
//     device; a call whose launch would need more is rejected with
//     cudaErrorInvalidValue and the bytes it would need in *scratch_needed;
//   * what must start at zero: the counter region [0, cnt_bytes(streams)) --
//     every call zeroes it on `stream` (cudaMemsetAsync, no allocation) before
//     the kernel; the partial records need no initial value;
//   * one scratch per device: calls that overlap in time on the same device
//     (concurrent streams, host threads) race on it -- serialize them;
//   * set-up: the first call on a device resolves the array's device address
//     (cudaGetSymbolAddress, with that device current) and the first call per
//     (head_dim, batch size class) sets the kernel's shared-memory attribute;
//     make those first calls before any stream capture begins. The address is
//     kept for the life of the process, so cudaDeviceReset (or destroying the
//     device's primary context) after the first call is not supported;
//   * float32 value pools only.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_static_scratch[INT4KV_STATIC_SCRATCH_BYTES];

namespace {

constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxScratchDevices] = {};

// Device address of g_static_scratch on the current device (set up once per device).
cudaError_t static_scratch_ptr(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxScratchDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return e;
    if (!p || (reinterpret_cast<uintptr_t>(p) & 255u)) return cudaErrorInvalidDevicePointer;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" cudaError_t int4kv_paged_decode_static_scratch(
    const float* query, const uint8_t* k_pool, const float* v_pool, const float* sz_pool,
    const int32_t* block_table, const int32_t* seq_lens, int batch, int num_q_heads,
    int num_kv_heads, int head_dim, int page_tokens, int group_tokens, int max_pages,
    int num_pages, float* out, uint32_t* status, size_t* scratch_needed, cudaStream_t stream) {
  size_t need = 0;
  cudaError_t e = int4kv_paged_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim,
                                                     &need);
  if (e != cudaSuccess) return e;
  if (scratch_needed) *scratch_needed = need;
  if (need > (size_t)INT4KV_STATIC_SCRATCH_BYTES) return cudaErrorInvalidValue;
  void* scratch = nullptr;
  e = static_scratch_ptr(&scratch);
  if (e != cudaSuccess) return e;
  const size_t zero_bytes = cnt_bytes((long long)batch * num_q_heads);
  e = cudaMemsetAsync(scratch, 0, zero_bytes, stream);
  if (e != cudaSuccess) return e;
  return int4kv_paged_decode(query, k_pool, v_pool, sz_pool, block_table, seq_lens, batch,
                             num_q_heads, num_kv_heads, head_dim, page_tokens, group_tokens,
                             max_pages, num_pages, out, scratch, INT4KV_STATIC_SCRATCH_BYTES,
                             status, stream);
}
