// Shared device helpers for the sm_100a INT4 KV kernels.
//
// Everything here is hand-written inline PTX for the Blackwell async-copy path
// (mbarrier + cp.async.bulk, i.e. the bulk/TMA engine without a tensor map)
// plus the exact-rounding float helpers the quantizer's bit-exact contract
// needs. The library is built WITHOUT --use_fast_math: every division below
// is IEEE round-to-nearest, as the reference's NumPy oracle computes it.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define I4KV_DEVINL __device__ __forceinline__

namespace i4kv {

// Status bits written into a caller-visible status word when a kernel had to
// defend itself against malformed device-resident metadata.
enum StatusBits : uint32_t {
  kStatusBadPage = 1u << 0,     // block-table entry outside [0, num_pages)
  kStatusBadLength = 1u << 1,   // sequence length < 0 or beyond its block-table row
  kStatusWaitTimeout = 1u << 2, // an mbarrier wait hit its iteration limit
  kStatusPeerTimeout = 1u << 3, // a peer GPU's exchange flag did not arrive in time
};

I4KV_DEVINL uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

I4KV_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

I4KV_DEVINL void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Release/acquire fence at GPU scope (lighter than the sequentially
// consistent __threadfence): with relaxed atomics on either side it orders
// the record stores before the arrival count and the merger's record loads
// after it.
I4KV_DEVINL void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// System-scope ordering for stores into another GPU's memory (peer mappings
// over NVLink): release the stores before a flag, acquire after reading one.
I4KV_DEVINL void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
I4KV_DEVINL void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
I4KV_DEVINL uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

I4KV_DEVINL void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

I4KV_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

I4KV_DEVINL bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// 16-byte asynchronous global -> shared copy (L2 only), its commit group and
// the wait for all but the newest N groups.
I4KV_DEVINL void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
I4KV_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
I4KV_DEVINL void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Atomic add with release and acquire semantics at GPU scope; returns the
// old value.
I4KV_DEVINL int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Store o[DPL] (this lane's dims of a D-vector) at dst with the P.V lane layout.
template <int D>
I4KV_DEVINL void store_lane_vec(float* dst, const float* o, int lane) {
  constexpr int DPL = D / 32;
  if constexpr (DPL == 2) {
    *reinterpret_cast<float2*>(dst + 2 * lane) = make_float2(o[0], o[1]);
  } else {
#pragma unroll
    for (int v4 = 0; v4 < DPL / 4; ++v4)
      *reinterpret_cast<float4*>(dst + v4 * 128 + 4 * lane) =
          make_float4(o[4 * v4], o[4 * v4 + 1], o[4 * v4 + 2], o[4 * v4 + 3]);
  }
}

template <int D>
I4KV_DEVINL void load_lane_vec_cg(const float* src, float* o, int lane) {
  constexpr int DPL = D / 32;
  if constexpr (DPL == 2) {
    const float2 v = __ldcg(reinterpret_cast<const float2*>(src + 2 * lane));
    o[0] = v.x; o[1] = v.y;
  } else {
#pragma unroll
    for (int v4 = 0; v4 < DPL / 4; ++v4) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(src + v4 * 128 + 4 * lane));
      o[4 * v4] = v.x; o[4 * v4 + 1] = v.y; o[4 * v4 + 2] = v.z; o[4 * v4 + 3] = v.w;
    }
  }
}

// The same lane layout read from shared memory.
template <int D>
I4KV_DEVINL void load_lane_vec_smem(const float* src, float* o, int lane) {
  constexpr int DPL = D / 32;
  if constexpr (DPL == 2) {
    const float2 v = *reinterpret_cast<const float2*>(src + 2 * lane);
    o[0] = v.x; o[1] = v.y;
  } else {
#pragma unroll
    for (int v4 = 0; v4 < DPL / 4; ++v4) {
      const float4 v = *reinterpret_cast<const float4*>(src + v4 * 128 + 4 * lane);
      o[4 * v4] = v.x; o[4 * v4 + 1] = v.y; o[4 * v4 + 2] = v.z; o[4 * v4 + 3] = v.w;
    }
  }
}

// Named barrier `id` (1..15) over `nthreads` threads (a multiple of 32; every
// lane of each participating warp executes it): bar.sync, and the form that
// also ORs a predicate across the participants.
I4KV_DEVINL void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
I4KV_DEVINL bool named_bar_or(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// ldmatrix.x4: lanes 8i..8i+7 give the row addresses (16-byte aligned, 16
// bytes each) of 8x8 b16 matrix i; lane L receives 32-bit word (L & 3) of row
// (L >> 2) of matrix i in r[i] -- the register layout of mma.sync operands.
I4KV_DEVINL void ldmatrix_x4(uint32_t (&r)[4], const void* row_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(row_addr))
               : "memory");
}

// d += A * B on the tensor cores, exact int32 arithmetic: A 16x32 u8 (row
// major: a[0] row g cols 4t..4t+3, a[1] row g+8, a[2] row g cols 16+4t..,
// a[3] row g+8 cols 16+4t..), B 32x8 s8 (column major: b0 rows 4t..4t+3 of
// column g, b1 rows 16+4t..), d 16x8 (d[0..1] row g cols 2t, 2t+1; d[2..3]
// row g+8), g = lane >> 2, t = lane & 3.
I4KV_DEVINL void mma_u8s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

I4KV_DEVINL uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes (woken promptly) or `hint_ns` elapses, instead of spinning.
I4KV_DEVINL bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// Bounded wait: sleeps on the barrier until the phase completes or `limit_ns`
// of wall time has passed, and then reports false. Callers record
// kStatusWaitTimeout and stop issuing work instead of waiting forever.
I4KV_DEVINL bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 100000u)) return true;
    if (global_ns() - t0 > limit_ns) return false;
  }
}

// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// Requirements (checked by callers): both addresses 16-byte aligned, size a
// multiple of 16. One destination CTA; the source is always this GPU's own memory.
I4KV_DEVINL void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// 2-D tiled TMA load of the box at element coordinates (x = inner, y = outer)
// through a tensor map held in kernel-parameter space; completion counted on
// `bar`. x * element size must be a multiple of 16 bytes (callers pass
// multiples of the box width). One destination CTA.
I4KV_DEVINL void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// Float32 value of a 4-bit code held in byte `sel` (0..3) of `w`, built without
// an integer->float conversion: the byte is placed in the low mantissa bits of
// 2^23, so the returned float is exactly 2^23 + code.
I4KV_DEVINL float magic_from_byte(uint32_t w, uint32_t sel) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | sel));
}

I4KV_DEVINL uint32_t ordered_key(float f) {  // monotone float -> uint32 map
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
I4KV_DEVINL float from_ordered_key(uint32_t k) {  // inverse of ordered_key
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Programmatic dependent launch (sm_90+): a kernel launched with the
// programmatic-serialization attribute may start while its predecessor on the
// stream is still running; grid_dependency_wait() blocks the calling thread
// until the predecessor grid has completed and its memory is visible (a no-op
// without the attribute), and allow_dependent_launch() lets the next kernel be
// scheduled once every CTA of this grid has called it or exited.
I4KV_DEVINL void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
I4KV_DEVINL void allow_dependent_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// The reference's per-channel parameters (src/quantize_int4_ref.py:65-70):
// range = max(max - min, 1e-8); scale = range / 15; zp = -min / scale.
I4KV_DEVINL void channel_params(float mn, float mx, float* scale, float* zp) {
  const float range = fmaxf(__fsub_rn(mx, mn), 1e-8f);
  const float s = __fdiv_rn(range, 15.0f);
  *scale = s;
  *zp = __fdiv_rn(-mn, s);
}

// The same code without a division per element, bit-identical: y = (x - mn)
// * RN(1/scale) is within 3 ulp of the IEEE quotient fl((x - mn) / scale); the
// two round to the same integer unless y lies within 2^-17 (> 3 ulp for
// y < 16) of a half-integer, and only there the IEEE quotient is computed.
// Round-half-even to an integer is one add of 1.5 * 2^23 (exact for
// |y| < 2^22; here 0 <= y <= 15 * (1 + 2^-22)), read back from the bits.
I4KV_DEVINL uint32_t quant_code_rcp(float x, float mn, float scale, float rcp) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23, bit pattern 0x4B400000
  const float a = __fsub_rn(x, mn);
  float y = __fmul_rn(a, rcp);
  float t = __fadd_rn(y, kMagic);  // 1.5 * 2^23 + rint(y), ties to even
  // y - rint(y) is exact (Sterbenz); |.| >= 0.5 - 2^-17 means "near a half"
  if (fabsf(__fsub_rn(y, __fsub_rn(t, kMagic))) >= 0.49999237060546875f) {
    y = __fdiv_rn(a, scale);
    t = __fadd_rn(y, kMagic);
  }
  // 0 <= y <= 15 * (1 + 3 * 2^-24) for x in [mn, max], so rint(y) is already
  // in [0, 15]: the mask only keeps the nibble (and maps a NaN input to 0).
  return static_cast<uint32_t>(__float_as_int(t) - 0x4B400000) & 15u;
}

// e^x for x <= 0 given in float64: 2^(x*log2(e)) with the hardware base-2
// exponential (relative error ~2^-22, far inside the decode's 1e-6 tolerance);
// x = -inf gives exactly 0.
I4KV_DEVINL float exp_neg(double x) {
  const float y = (float)(x * 1.4426950408889634);
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(y));
  return r;
}

// 1/d in float64 for normal 0 < d < 2^100: a float32 reciprocal estimate and
// two Newton-Raphson steps y += y(1 - dy), each squaring the relative error
// (2^-23 -> 2^-46 -> below the float64 rounding).
I4KV_DEVINL double rcp_f64(double d) {
  float yf;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(yf) : "f"((float)d));
  double y = (double)yf;
  double e = fma(-d, y, 1.0);
  y = fma(y, e, y);
  e = fma(-d, y, 1.0);
  return fma(y, e, y);
}

// floor(x / t) for 0 <= x < 2^52 and 0 < t < 2^31: a float64 quotient estimate
// (off by at most 2) corrected in exact integer arithmetic, in place of the
// 64-bit integer division routine.
I4KV_DEVINL long long floor_div_s52(long long x, long long t) {
  long long q = (long long)((double)x * rcp_f64((double)t));
  long long r = x - q * t;
  while (r < 0) { --q; r += t; }
  while (r >= t) { ++q; r -= t; }
  return q;
}

// e^x for x <= 0 in float64: Cody-Waite reduction x = n ln2 + r, |r| <= ln2/2,
// with ln2 split into a head of 21 significant bits (n * head is exact) and a
// tail, then the degree-11 Taylor polynomial of e^r (relative truncation error
// below 1e-14 on that range) and the exact scaling by 2^n. Arguments below
// -708 (and -inf) give 0.
I4KV_DEVINL double exp_nonpos(double x) {
  if (!(x >= -708.0)) return 0.0;
  const double n = rint(x * 1.4426950408889634);
  double r = fma(n, -0x1.62e42p-1, x);
  r = fma(n, -0x1.fdf473de6af28p-22, r);
  double p = 2.505210838544172e-08;  // 1/11!
  p = fma(p, r, 2.755731922398589e-07);
  p = fma(p, r, 2.755731922398589e-06);
  p = fma(p, r, 2.48015873015873e-05);
  p = fma(p, r, 0.0001984126984126984);
  p = fma(p, r, 0.001388888888888889);
  p = fma(p, r, 0.008333333333333333);
  p = fma(p, r, 0.041666666666666664);
  p = fma(p, r, 0.16666666666666666);
  p = fma(p, r, 0.5);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  return p * __hiloint2double(((int)n + 1023) << 20, 0);
}

// sum = sum*r + x with a running compensation term c (Kahan): the rescale
// applies to both, the addition captures its own rounding error in c.
I4KV_DEVINL void kahan_rescale_add(float& sum, float& c, float r, float x) {
  sum *= r;
  c *= r;
  const float y = __fsub_rn(x, c);
  const float t = __fadd_rn(sum, y);
  c = __fsub_rn(__fsub_rn(t, sum), y);
  sum = t;
}

// Two Kahan additions side by side in paired float32 arithmetic
// (sub/add.rn.f32x2): (s0, c0) += x0 and (s1, c1) += x1 exactly as two
// kahan_rescale_add(s, c, 1.f, x) calls would do them, in half the
// instructions.
I4KV_DEVINL void kahan_add2(float& s0, float& s1, float& c0, float& c1, float x0, float x1) {
  asm("{\n\t.reg .b64 s, c, x, y, t, u;\n\t"
      "mov.b64 s, {%0, %1};\n\tmov.b64 c, {%2, %3};\n\tmov.b64 x, {%4, %5};\n\t"
      "sub.rn.f32x2 y, x, c;\n\tadd.rn.f32x2 t, s, y;\n\tsub.rn.f32x2 u, t, s;\n\t"
      "sub.rn.f32x2 c, u, y;\n\tmov.b64 {%0, %1}, t;\n\tmov.b64 {%2, %3}, c;\n\t}"
      : "+f"(s0), "+f"(s1), "+f"(c0), "+f"(c1)
      : "f"(x0), "f"(x1));
}

// Three-input float32 min / max (sm_100), with fminf / fmaxf semantics.
I4KV_DEVINL float fmin3f(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
I4KV_DEVINL float fmax3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Paired IEEE float32 arithmetic (sm_100 f32x2 instructions, round to
// nearest even, subnormals kept): two lanes of work per instruction.
#define I4KV_F32X2_OP(name, op)                                                               \
  I4KV_DEVINL void name(float& d0, float& d1, float a0, float a1, float b0, float b1) {       \
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t" op \
        " rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"                                      \
        : "=f"(d0), "=f"(d1)                                                                \
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));                                              \
  }
I4KV_F32X2_OP(add2_rn, "add.rn.f32x2")
I4KV_F32X2_OP(sub2_rn, "sub.rn.f32x2")
I4KV_F32X2_OP(mul2_rn, "mul.rn.f32x2")
#undef I4KV_F32X2_OP

// Paired fused multiply-add, each lane rounded once: (c0, c1) += (a0 b, a1 b)
// for one scalar b -- exactly fmaf(a0, b, c0), fmaf(a1, b, c1).
I4KV_DEVINL void fma2_rn(float& c0, float& c1, float a0, float a1, float b) {
  asm("{\n\t.reg .b64 ra, rb, rc;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %4};\n\t"
      "mov.b64 rc, {%0, %1};\n\tfma.rn.f32x2 rc, ra, rb, rc;\n\tmov.b64 {%0, %1}, rc;\n\t}"
      : "+f"(c0), "+f"(c1)
      : "f"(a0), "f"(a1), "f"(b));
}

// Four codes of one row's channel quad (quant_code_rcp for each, in paired
// arithmetic), one per byte: c0 | c1 << 8 | c2 << 16 | c3 << 24. The low byte
// of the bits of 1.5 * 2^23 + rint(y) is rint(y) itself, so the codes are
// gathered with byte permutes.
I4KV_DEVINL uint32_t codes4_rcp(float4 v, float4 mn, float4 sc, float4 rc) {
  constexpr float kMagic = 12582912.0f;
  constexpr float kNearHalf = 0.49999237060546875f;  // 0.5 - 2^-17
  float a0, a1, a2, a3, y0, y1, y2, y3, t0, t1, t2, t3, r0, r1, r2, r3, d0, d1, d2, d3;
  sub2_rn(a0, a1, v.x, v.y, mn.x, mn.y);
  sub2_rn(a2, a3, v.z, v.w, mn.z, mn.w);
  mul2_rn(y0, y1, a0, a1, rc.x, rc.y);
  mul2_rn(y2, y3, a2, a3, rc.z, rc.w);
  add2_rn(t0, t1, y0, y1, kMagic, kMagic);
  add2_rn(t2, t3, y2, y3, kMagic, kMagic);
  sub2_rn(r0, r1, t0, t1, kMagic, kMagic);
  sub2_rn(r2, r3, t2, t3, kMagic, kMagic);
  sub2_rn(d0, d1, y0, y1, r0, r1);
  sub2_rn(d2, d3, y2, y3, r2, r3);
  if (fmaxf(fmaxf(fabsf(d0), fabsf(d1)), fmaxf(fabsf(d2), fabsf(d3))) >= kNearHalf) {
    if (fabsf(d0) >= kNearHalf) t0 = __fadd_rn(__fdiv_rn(a0, sc.x), kMagic);
    if (fabsf(d1) >= kNearHalf) t1 = __fadd_rn(__fdiv_rn(a1, sc.y), kMagic);
    if (fabsf(d2) >= kNearHalf) t2 = __fadd_rn(__fdiv_rn(a2, sc.z), kMagic);
    if (fabsf(d3) >= kNearHalf) t3 = __fadd_rn(__fdiv_rn(a3, sc.w), kMagic);
  }
  return __byte_perm(__byte_perm(__float_as_uint(t0), __float_as_uint(t1), 0x0040),
                     __byte_perm(__float_as_uint(t2), __float_as_uint(t3), 0x0040),
                     0x5410);  // bytes c0, c1, c2, c3 (each already in [0, 15])
}

// The same four codes nibble-packed: c0 | c1 << 4 | c2 << 8 | c3 << 12.
I4KV_DEVINL uint32_t pack4_rcp(float4 v, float4 mn, float4 sc, float4 rc) {
  const uint32_t x = codes4_rcp(v, mn, sc, rc);  // bytes c0, c1, c2, c3
  const uint32_t y = x | (x >> 4);                // c0|c1<<4, ., c2|c3<<4, .
  return __byte_perm(y, 0u, 0x4420);              // [c0|c1<<4][c2|c3<<4]
}

// q = clip(round_half_even((x - min) / scale), 0, 15)  (src/quantize_int4_ref.py:74-75)
I4KV_DEVINL uint32_t quant_code(float x, float mn, float scale) {
  const float t = __fdiv_rn(__fsub_rn(x, mn), scale);
  int q = __float2int_rn(t);
  q = q < 0 ? 0 : (q > 15 ? 15 : q);
  return static_cast<uint32_t>(q);
}

}  // namespace i4kv
