// Shared device helpers: element formats, bit tricks, bounded waits.
//
// All float-format conversions are written here from the format definitions
// (IEEE-754 binary32, bfloat16, OCP FP8 e4m3fn / e5m2) with integer
// arithmetic, so the rounding of every cast is explicit and matches the
// reference's PyTorch / Triton casts bit for bit:
//   * fp32 -> bf16: round to nearest even;
//   * fp32 -> e4m3fn: round to nearest even, |x| > 464 -> NaN (0x7F), which
//     is what torch's float8_e4m3fn cast does (c10 semantics);
//   * fp8 / bf16 -> fp32: exact.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/bitsparse.h"

namespace bs {

constexpr int kTileM = 64;
constexpr int kTileN = 64;
constexpr int kTileNumel = 4096;
constexpr int kTileBytes = 512;
constexpr int kThreads = 256;

// Upper bound on polls of another CTA's scan flag before giving up.  A poll
// is a few hundred ns, so this is far above any legitimate wait (the CTAs
// polled are already running) and well under a second.
constexpr uint32_t kMaxPolls = 1u << 21;

// ---------------------------------------------------------------------------
// Shared-memory barriers and 1-D bulk copies (TMA engine)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Generic-proxy accesses of shared memory before this fence are ordered
// before later async-proxy (TMA / bulk copy) accesses of it.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 1-D bulk copy global -> shared (no multicast): both addresses 16-byte
// aligned, bytes a multiple of 16; completes `bytes` on the mbarrier.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// Format helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) {
  return __uint_as_float(b << 16);
}

__device__ __forceinline__ uint32_t f32_to_bf16_bits(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return ((u >> 16) & 0x8000u) | 0x7FC0u;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return u >> 16;
}

// e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa; 0x7F/0xFF are NaN, no inf.
__device__ __forceinline__ float e4m3_bits_to_f32(uint32_t b) {
  uint32_t s = (b & 0x80u) << 24;
  uint32_t e = (b >> 3) & 0xFu, m = b & 7u;
  if ((b & 0x7Fu) == 0x7Fu) return __uint_as_float(0x7FC00000u | s);
  if (e == 0) {  // subnormal: m * 2^-9
    return __uint_as_float(s) + (s ? -1.f : 1.f) * (float)m * 0.001953125f;
  }
  return __uint_as_float(s | ((e + 120u) << 23) | (m << 20));
}

// e5m2: 1 sign, 5 exponent (bias 15), 2 mantissa; IEEE-style inf / NaN.
__device__ __forceinline__ float e5m2_bits_to_f32(uint32_t b) {
  uint32_t s = (b & 0x80u) << 24;
  uint32_t e = (b >> 2) & 0x1Fu, m = b & 3u;
  if (e == 0x1F) return __uint_as_float(s | 0x7F800000u | (m ? 0x400000u : 0u));
  if (e == 0) {  // subnormal: m * 2^-16
    return __uint_as_float(s) + (s ? -1.f : 1.f) * (float)m * 1.52587890625e-05f;
  }
  return __uint_as_float(s | ((e + 112u) << 23) | (m << 21));
}

template <int DT>
__device__ __forceinline__ float store_bits_to_f32(uint32_t b) {
  if constexpr (DT == BS_BF16) return bf16_bits_to_f32(b);
  else if constexpr (DT == BS_E4M3) return e4m3_bits_to_f32(b);
  else return e5m2_bits_to_f32(b);
}

// fp32 -> e4m3fn bits, round to nearest even (torch float8_e4m3fn cast).
__device__ __forceinline__ uint32_t f32_to_e4m3_bits(float f) {
  uint32_t u = __float_as_uint(f);
  uint32_t s = (u >> 24) & 0x80u;
  uint32_t a = u & 0x7FFFFFFFu;
  if (a > 0x43E80000u) return s | 0x7Fu;  // > 464 (or NaN): NaN
  if (a < 0x3C800000u) {                  // < 2^-6: subnormal range
    // value = a_f; quantum 2^-9.  Round a_f / 2^-9 to nearest even integer.
    float af = __uint_as_float(a) * 512.0f;  // exact (power of two scale)
    // af < 8; split into integer and fraction exactly.
    uint32_t i = (uint32_t)af;               // truncation
    float frac = af - (float)i;              // exact
    if (frac > 0.5f || (frac == 0.5f && (i & 1u))) ++i;
    return s | i;  // i == 8 gives 0x08 = smallest normal, correct
  }
  // normal: keep 3 mantissa bits, RNE on the 20 dropped bits
  uint32_t exp = (a >> 23) - 120u;  // biased e4m3 exponent, >= 1
  uint32_t mant = a & 0x7FFFFFu;
  uint32_t q = (exp << 3) | (mant >> 20);
  uint32_t rem = mant & 0xFFFFFu;
  if (rem > 0x80000u || (rem == 0x80000u && (q & 1u))) ++q;
  // q can reach 0x7F only for values in (448, 464]: 464 ties to even (0x7E)
  // is handled by RNE above; anything that rounds to 0x7F is > 464 and was
  // already caught by the NaN test.
  return s | q;
}

// Two fp32 -> bf16 conversions, round to nearest even (the hardware
// conversion, which torch's bf16 conversion on CUDA also uses).
__device__ __forceinline__ uint32_t bf16x2_from_f32(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Two fp32 values that are already representable-range e4m3 inputs (|v| <=
// 464, not NaN) -> two e4m3fn codes, round to nearest even, low byte = a.
// In that range the hardware conversion matches the torch cast exactly.
__device__ __forceinline__ uint32_t e4m3x2_bits(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return r;
}

// 1/s rounded to fp32, the quantisers' reciprocal, or 0 where it would not
// be an accurate normal number (s zero, subnormal, at or above 2^126, inf or
// NaN): every quantiser then takes its division for all values.
__device__ __forceinline__ float quant_rcp(float s) {
  const uint32_t e = (__float_as_uint(s) >> 23) & 0xFFu;
  return (e >= 1u && e <= 252u) ? __frcp_rn(s) : 0.f;
}

// x / s in fp32, close enough that rounding it to bf16 gives bf16(x / s) of
// the exact IEEE quotient: y1 = x*r corrected by one FMA residual step is
// within 1 fp32 ulp of the true quotient, so its bf16 rounding can only
// differ from the exact one when it lies within an ulp or two of a bf16
// rounding midpoint (low 16 bits near 0x8000); those rare quotients are
// recomputed with the exact division.  r = 1/s rounded, s > 0.
__device__ __forceinline__ float quotient_fp32(float x, float s, float r) {
  const float y0 = x * r;
  const float e = fmaf(-y0, s, x);  // exact residual
  const float y1 = fmaf(e, r, y0);
  const uint32_t lo = __float_as_uint(y1) & 0xFFFFu;
  // the quotient has x's sign (keeps -0, which the residual loses)
  return (r == 0.f || lo - 0x7FFCu <= 8u) ? __fdiv_rn(x, s) : copysignf(y1, x);
}

// to_fp8's quantiser on two bf16 values (as fp32): e4m3(bf16(x / s)).
__device__ __forceinline__ uint32_t div_e4m3x2(float x0, float x1, float s, float r) {
  const uint32_t b = bf16x2_from_f32(quotient_fp32(x0, s, r), quotient_fp32(x1, s, r));
  return e4m3x2_bits(bf16_bits_to_f32(b & 0xFFFFu), bf16_bits_to_f32(b >> 16));
}

// div_e4m3x2 on eight bf16 values (four words, low half first) -> two words
// of codes.  The corrected estimates of quotient_fp32 are taken branch-free;
// only if one of them lies near a bf16 rounding midpoint is the group redone
// with quotient_fp32's exact fallback -- one branch per eight values instead
// of one per value, and the same codes as div_e4m3x2.
// The rare exact case of div_e4m3x8, out of line so that the unrolled
// callers stay small (their instruction footprint matters more than a call).
static __device__ __noinline__ uint2 div_e4m3x8_exact(uint32_t w0, uint32_t w1, uint32_t w2,
                                               uint32_t w3, float s, float r) {
  const uint32_t w[4] = {w0, w1, w2, w3};
  uint32_t b[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    b[i] = bf16x2_from_f32(__fdiv_rn(__uint_as_float(w[i] << 16), s),
                           __fdiv_rn(__uint_as_float(w[i] & 0xFFFF0000u), s));
  uint32_t o[2];
#pragma unroll
  for (int i = 0; i < 2; ++i)
    o[i] = e4m3x2_bits(__uint_as_float(b[2 * i] << 16), __uint_as_float(b[2 * i] & 0xFFFF0000u)) |
           e4m3x2_bits(__uint_as_float(b[2 * i + 1] << 16),
                       __uint_as_float(b[2 * i + 1] & 0xFFFF0000u)) << 16;
  return make_uint2(o[0], o[1]);
}

__device__ __forceinline__ void div_e4m3x8(const uint32_t (&w)[4], float s, float r,
                                           uint32_t (&o)[2]) {
  uint32_t near = r == 0.f;  // no usable reciprocal: divide all
  float y[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float x = bf16_bits_to_f32(e & 1 ? w[e >> 1] >> 16 : w[e >> 1] & 0xFFFFu);
    const float y0 = x * r;
    const float y1 = fmaf(fmaf(-y0, s, x), r, y0);
    near |= (__float_as_uint(y1) & 0xFFFFu) - 0x7FFCu <= 8u;
    y[e] = copysignf(y1, x);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t b0 = bf16x2_from_f32(y[4 * i], y[4 * i + 1]);
    const uint32_t b1 = bf16x2_from_f32(y[4 * i + 2], y[4 * i + 3]);
    o[i] = e4m3x2_bits(bf16_bits_to_f32(b0 & 0xFFFFu), bf16_bits_to_f32(b0 >> 16)) |
           e4m3x2_bits(bf16_bits_to_f32(b1 & 0xFFFFu), bf16_bits_to_f32(b1 >> 16)) << 16;
  }
  if (near) {
    const uint2 e = div_e4m3x8_exact(w[0], w[1], w[2], w[3], s, r);
    o[0] = e.x;
    o[1] = e.y;
  }
}

// 1/448 rounded to fp32: the compiled to_fp8 computes amax / 448 as
// amax * (1/448), the reciprocal of the constant taken once.
constexpr float kRcp448 = 1.0f / 448.0f;

// The fp32 division of Triton's `/` operator (PTX div.full.f32, an
// approximate full-range division): the quotient the reference's compiled
// to_fp8 computes.
__device__ __forceinline__ float div_full(float x, float s) {
  float q;
  asm("div.full.f32 %0, %1, %2;" : "=f"(q) : "f"(x), "f"(s));
  return q;
}

// to_fp8's quantiser as the reference runs it on a GPU: its to_fp8 is
// @torch.compile'd (lib_sparse/fp8.py:123-129), and the generated Triton
// code divides the fp32 value by the scale with Triton's division and casts
// the quotient to e4m3 -- no rounding of the quotient to bf16 as eager
// PyTorch does.  The e4m3 code only depends on which side of the e4m3
// rounding midpoints the quotient lies: the estimate x * r (r = 1/s rounded
// to fp32) is within a few fp32 ulps of the division's result, so when it
// lies in the normal e4m3 range (>= 2^-6) and more than 64 ulps from a
// midpoint (fp32 mantissa bits 19..0 = 0x80000) both give the same code;
// only the others take the division itself.
__device__ __forceinline__ bool e4m3_code_settled(float q0) {
  const uint32_t b = __float_as_uint(q0);
  const uint32_t low = b & 0xFFFFFu, d = low > 0x80000u ? low - 0x80000u : 0x80000u - low;
  // a zero estimate is final too: 0*r and 0/s are the same signed zero (and
  // the same NaN when s is 0 or NaN), and an estimate that underflowed to 0
  // is below e4m3's smallest subnormal either way
  return (((b >> 23) & 0xFFu) >= 127u - 6u && d > 64u) || (b << 1) == 0u;
}
// (The fp32 -> e4m3 casts are the hardware conversion, saturating to 448,
// which is what Triton's cast compiles to.)
__device__ __forceinline__ uint32_t e4m3_compiled(float x, float s, float r) {
  const float q0 = x * r;
  return e4m3x2_bits(r != 0.f && e4m3_code_settled(q0) ? q0 : div_full(x, s), 0.f) & 0xFFu;
}
// The rare case of full_e4m3x8 (some estimate unsettled): all eight by the
// division, out of line so that the unrolled callers stay small.
static __device__ __noinline__ uint2 full_e4m3x8_div(uint32_t w0, uint32_t w1, uint32_t w2,
                                                    uint32_t w3, float s) {
  const uint32_t w[4] = {w0, w1, w2, w3};
  float q[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) q[e] = div_full(__uint_as_float((w[e >> 1] >> (16 * (e & 1))) << 16), s);
  return make_uint2(e4m3x2_bits(q[0], q[1]) | e4m3x2_bits(q[2], q[3]) << 16,
                    e4m3x2_bits(q[4], q[5]) | e4m3x2_bits(q[6], q[7]) << 16);
}
// Eight bf16 values (four words, low half first) -> two words of codes.
__device__ __forceinline__ void full_e4m3x8(const uint32_t (&w)[4], float s, float r,
                                            uint32_t (&o)[2]) {
  float q[8];
  bool all = r != 0.f;  // no usable reciprocal: divide all
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    q[e] = __uint_as_float((w[e >> 1] >> (16 * (e & 1))) << 16) * r;
    all &= e4m3_code_settled(q[e]);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i)
    o[i] = e4m3x2_bits(q[4 * i], q[4 * i + 1]) | e4m3x2_bits(q[4 * i + 2], q[4 * i + 3]) << 16;
  if (!all) {
    const uint2 d = full_e4m3x8_div(w[0], w[1], w[2], w[3], s);
    o[0] = d.x;
    o[1] = d.y;
  }
}

// Whether the plain estimate x * r (r = 1/s rounded to fp32) gives the
// quantiser's e4m3 code for EVERY bf16 x at this scale -- compiled:
// e4m3(div_full(x, s)); eager: e4m3(bf16(x / s)) -- so that a kernel may
// quantise with the estimate alone (est_e4m3x8).  Proved by exhaustion over
// the bf16 codes that can reach a rounding boundary: with e_s the biased
// exponent of s, a bf16 x of biased exponent E below e_s - 13 has
// |x / s| < 2^-13 (both forms give a signed zero code) and one above
// e_s + 11 has |x / s| > 2^11 (both saturate to +-448), so the 25 binades
// E = e_s - 13 .. e_s + 11, both signs, and E = 255 (inf / NaN) are tested,
// 6656 codes.  A scale whose window leaves bf16's normal exponents (or a
// non-positive, non-finite scale) answers false.  Every thread of the block
// must call it; the answer is uniform over the block.
static __device__ __noinline__ bool e4m3_estimate_exact(float s, float r, bool compiled) {
  const uint32_t es = (__float_as_uint(s) >> 23) & 0xFFu;
  bool ok = s > 0.f && es >= 14u && es <= 243u;
  if (ok) {  // same s in every thread: uniform
    constexpr uint32_t kBinades = 25, kCodes = (kBinades + 1) * 256;
    for (uint32_t i = threadIdx.x; i < kCodes; i += blockDim.x) {
      const uint32_t g = i >> 8, e = g < kBinades ? es - 13u + g : 255u;
      const float x = __uint_as_float((((i & 1u) << 15) | (e << 7) | ((i >> 1) & 127u)) << 16);
      const float q = x * r;
      uint32_t a, b;
      if (compiled) {
        a = e4m3x2_bits(q, 0.f);
        b = e4m3x2_bits(div_full(x, s), 0.f);
      } else {
        const uint32_t h = bf16x2_from_f32(q, __fdiv_rn(x, s));
        a = e4m3x2_bits(bf16_bits_to_f32(h & 0xFFFFu), 0.f);
        b = e4m3x2_bits(bf16_bits_to_f32(h >> 16), 0.f);
      }
      ok &= a == b;
    }
  }
  return __syncthreads_and(ok) != 0;
}

// The quantiser by the estimate alone, on eight bf16 values (four words,
// low half first) -> two words of codes: e4m3(x * r) (compiled) or
// e4m3(bf16(x * r)) (eager).  Exact where e4m3_estimate_exact(s, r, COMPILED)
// holds.
template <bool COMPILED>
__device__ __forceinline__ void est_e4m3x8(const uint32_t (&w)[4], float r, uint32_t (&o)[2]) {
  float q[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    q[2 * i] = __uint_as_float(w[i] << 16) * r;
    q[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u) * r;
    if constexpr (!COMPILED) {
      const uint32_t h = bf16x2_from_f32(q[2 * i], q[2 * i + 1]);
      q[2 * i] = __uint_as_float(h << 16);
      q[2 * i + 1] = __uint_as_float(h & 0xFFFF0000u);
    }
  }
#pragma unroll
  for (int i = 0; i < 2; ++i)
    o[i] = e4m3x2_bits(q[4 * i], q[4 * i + 1]) | e4m3x2_bits(q[4 * i + 2], q[4 * i + 3]) << 16;
}

// The quantiser where the estimate alone is not known exact, out of line
// (the rare path of kernels that check e4m3_estimate_exact): eight bf16
// values -> two words of codes, compiled or eager semantics.
static __device__ __noinline__ uint2 quant8_checked(uint32_t w0, uint32_t w1, uint32_t w2,
                                                    uint32_t w3, float s, float r, bool compiled) {
  const uint32_t w[4] = {w0, w1, w2, w3};
  uint32_t o[2];
  if (compiled) full_e4m3x8(w, s, r, o);
  else div_e4m3x8(w, s, r, o);
  return make_uint2(o[0], o[1]);
}

// Elementwise bf16x2 sum / product, rounded to nearest even.  Equal to
// torch's bf16 arithmetic (the fp32 result rounded to bf16): fp32 carries
// more than 2 * 8 + 2 significant bits, so rounding first to fp32 and then
// to bf16 gives the correctly rounded sum; a product of two bf16 values is
// exact in fp32 wherever it is normal, and in fp32's subnormal range the
// two roundings agree as well.
__device__ __forceinline__ uint32_t bf16x2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// torch.relu on two bf16: strictly negative values (incl. -inf) -> +0;
// -0 and NaN unchanged.
__device__ __forceinline__ uint32_t relu_bf16x2(uint32_t w) {
  const uint32_t v = w & 0x7FFF7FFFu;
  const uint32_t nz = v + 0x7FFF7FFFu;   // bit 15 of a half set iff v != 0
  const uint32_t nan = v + 0x007F007Fu;  // bit 15 set iff v >= 0x7F81 (NaN)
  const uint32_t kill = w & nz & ~nan & 0x80008000u;
  return w & ~((kill >> 15) * 0xFFFFu);
}

// Positive test on raw bits (x > 0.0 as a float; NaN and -0 are not).
template <int DT>
__device__ __forceinline__ bool is_pos(uint32_t b) {
  if constexpr (DT == BS_BF16) return b - 1u < 0x7F80u;   // 1..0x7F80
  else if constexpr (DT == BS_E4M3) return b - 1u < 0x7Eu;  // 1..0x7E
  else if constexpr (DT == BS_E5M2) return b - 1u < 0x7Cu;  // 1..0x7C
  else return b - 1u < 0x7F800000u;                          // fp32
}

template <int DT> struct Elt;
template <> struct Elt<BS_BF16> { static constexpr int bytes = 2; };
template <> struct Elt<BS_E4M3> { static constexpr int bytes = 1; };
template <> struct Elt<BS_E5M2> { static constexpr int bytes = 1; };
template <> struct Elt<BS_F32> { static constexpr int bytes = 4; };

template <int DT>
__device__ __forceinline__ constexpr int pack_bits() {
  return DT == BS_BF16 ? 15 : 7;
}

// ---------------------------------------------------------------------------
// Warp / memory helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    uint32_t n = __shfl_up_sync(0xFFFFFFFFu, v, d);
    if (lane >= d) v += n;
  }
  return v;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint4 ld_nc_v4(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void st_v4(void *p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void status_or(int32_t *status, int bits) {
  if (status) atomicOr(status, bits);
}

}  // namespace bs
