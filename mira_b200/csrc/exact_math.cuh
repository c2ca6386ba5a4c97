// Exact f32 arithmetic shared by the kernels, written so that results are bit-identical to the
// reference's NumPy semantics:
//   dequant      y  = float32(float64(acc) * S)          reference ops.py:619 and ops.py:633
//   quantize     q  = clip(rint(float32(y / s)), -127, 127)   reference ops.py:602-603
//   epilogue     NumPy float32 add/sub/mul/div/maximum/minimum   reference ops.py:192-199
// No contraction: every operation below is an explicitly rounded intrinsic.
#pragma once
#include <cstdint>

#include "../../include/mira_cuda.h"

namespace mira {

// float32(float64(acc) * S) without 64-bit conversions on the fast path.
//
// S (a double) is split as S = hi + lo + r with hi = f32(S), lo = f32(S - hi), |r| <= |S| 2^-48.
// For |acc| < 2^22, a = float(acc) is exact (magic-number conversion) and
//     D = a*hi + f32(a*lo)            (one FFMA: the product a*hi is exact inside the FMA)
// is within |acc*S| 2^-46 of the true product X = acc*S.  float32(float64(X)) equals RN32(X)
// unless an f32 rounding midpoint lies within |X| 2^-53 of X, and RN32(D) equals RN32(X) unless a
// midpoint lies between D and X.  So if RN32(D - d) == RN32(D + d) with d = |a| hi 2^-40 (far
// larger than both distances), no midpoint is near and RN32(D) is the exact answer.  Otherwise
// (about 2 in 10^5 elements, or |acc| >= 2^22) the product must be done in float64 like the
// reference: this branch-free function writes the candidate and returns false in those cases.
__device__ __forceinline__ bool dequant_fast(int32_t acc, float hi, float lo, float& y) {
  const bool in_range = static_cast<uint32_t>(acc) + (1u << 22) < (1u << 23);
  const float a = __fsub_rn(__int_as_float(0x4B400000 + acc), 12582912.0f);
  const float p = __fmul_rn(a, lo);
  const float d = __fmul_rn(fabsf(a), __fmul_rn(hi, 0x1p-40f));
  const float y_lo = __fmaf_rn(a, hi, __fsub_rn(p, d));
  const float y_hi = __fmaf_rn(a, hi, __fadd_rn(p, d));
  y = y_lo;
  return in_range && (y_lo == y_hi);
}

// Row/column scales: S = f64(r) * f64(c) is exact in float64 (24 + 24 significant bits), and
// so is its split hi = f32(r*c), lo = r*c - hi (the FMA residual).
__device__ __forceinline__ void split_rowcol(float r, float c, float& hi, float& lo) {
  hi = __fmul_rn(r, c);
  lo = __fmaf_rn(r, c, -hi);
}

// RN32(y / s) from a precomputed correctly-rounded reciprocal rcp = RN32(1/s): q0 = RN(y*rcp) is
// within one ulp, the residual y - q0*s is exact in one FMA, and RN(q0 + res*rcp) is the correctly
// rounded quotient (Markstein's theorem).  y is first clamped to +-256 s, which cannot change a
// result that is clipped to +-127 afterwards and keeps every intermediate finite.
__device__ __forceinline__ float div_by_scale(float y, float s, float rcp, float lim) {
  y = fminf(fmaxf(y, -lim), lim);
  const float q0 = __fmul_rn(y, rcp);
  const float res = __fmaf_rn(-q0, s, y);
  return __fmaf_rn(res, rcp, q0);
}

// ---- packed f32x2 arithmetic (sm_100): two independent IEEE single-precision operations per
// instruction, each rounded to nearest like the scalar __fadd_rn / __fmul_rn / __fmaf_rn.  Unlike
// the scalar forms, ptxas contracts f2_mul followed by an f2_add/f2_sub of its result into one
// fma.rn.f32x2 (measured on sm_100a): never feed an f2_mul into an f2_add or f2_sub where the
// product must be rounded on its own.
typedef unsigned long long f2_t;

__device__ __forceinline__ f2_t f2(float lo, float hi) {
  f2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_split(f2_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f2_t f2_add(f2_t a, f2_t b) {
  f2_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2_t f2_sub(f2_t a, f2_t b) {
  f2_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2_t f2_mul(f2_t a, f2_t b) {
  f2_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2_t f2_fma(f2_t a, f2_t b, f2_t c) {
  f2_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// The dequant of 4 accumulators, two per instruction: for each lane the same arithmetic as
// dequant_fast with the uncertainty interval P +- A*hi*2^-40 (its sign only swaps the ends).
// Sets bits of `slow` (shifted by `bit`) for elements that need the exact f64 path (|acc| >= 2^22,
// or a result within the interval of an f32 rounding boundary); checked on 3e8 random cases on
// the CPU.
__device__ __forceinline__ void dequant4_x2(const uint32_t* r, const float4& hs, const float4& ls, float* v,
                                            uint32_t& slow, int bit) {
  const f2_t magic = f2(-12582912.0f, -12582912.0f);
  const f2_t e40 = f2(0x1p-40f, 0x1p-40f), ne40 = f2(-0x1p-40f, -0x1p-40f);
  const float hv[4] = {hs.x, hs.y, hs.z, hs.w}, lv[4] = {ls.x, ls.y, ls.z, ls.w};
#pragma unroll
  for (int j = 0; j < 4; j += 2) {
    const f2_t a = f2_add(f2(__int_as_float(0x4B400000 + static_cast<int32_t>(r[j])),
                             __int_as_float(0x4B400000 + static_cast<int32_t>(r[j + 1]))), magic);
    const f2_t h = f2(hv[j], hv[j + 1]);
    const f2_t pl = f2_mul(a, f2(lv[j], lv[j + 1]));
    const f2_t yl = f2_fma(a, h, f2_fma(a, f2_mul(h, ne40), pl));
    const f2_t yh = f2_fma(a, h, f2_fma(a, f2_mul(h, e40), pl));
    float a0, a1, l0, l1, h0, h1;
    f2_split(a, a0, a1);
    f2_split(yl, l0, l1);
    f2_split(yh, h0, h1);
    v[j] = l0;
    v[j + 1] = l1;
    slow |= ((l0 == h0) && (fabsf(a0) < 0x1p22f)) ? 0u : (1u << (bit + j));
    slow |= ((l1 == h1) && (fabsf(a1) < 0x1p22f)) ? 0u : (2u << (bit + j));
  }
}

// dequant4_x2 with its checks folded into two bitwise accumulations (as dequant16_x2 below): a
// value needs the exact f64 path when (bad | (range & 0xFF800000)) != 0 after all are folded in.
__device__ __forceinline__ void dequant4_fold(const uint32_t* r, const float4& hs, const float4& ls, float* v,
                                              uint32_t& bad, uint32_t& range) {
  const f2_t magic = f2(-12582912.0f, -12582912.0f);
  const f2_t e40 = f2(0x1p-40f, 0x1p-40f), ne40 = f2(-0x1p-40f, -0x1p-40f);
  const float hv[4] = {hs.x, hs.y, hs.z, hs.w}, lv[4] = {ls.x, ls.y, ls.z, ls.w};
#pragma unroll
  for (int j = 0; j < 4; j += 2) {
    const uint32_t x0 = 0x4B400000u + r[j], x1 = 0x4B400000u + r[j + 1];
    range |= x0 ^ 0x4B000000u;
    range |= x1 ^ 0x4B000000u;
    const f2_t a = f2_add(f2(__uint_as_float(x0), __uint_as_float(x1)), magic);
    const f2_t h = f2(hv[j], hv[j + 1]);
    const f2_t pl = f2_mul(a, f2(lv[j], lv[j + 1]));
    const f2_t yl = f2_fma(a, h, f2_fma(a, f2_mul(h, ne40), pl));
    const f2_t yh = f2_fma(a, h, f2_fma(a, f2_mul(h, e40), pl));
    float l0, l1, h0, h1;
    f2_split(yl, l0, l1);
    f2_split(yh, h0, h1);
    v[j] = l0;
    v[j + 1] = l1;
    bad |= __float_as_uint(l0) ^ __float_as_uint(h0);
    bad |= __float_as_uint(l1) ^ __float_as_uint(h1);
  }
}

// The dequant of 16 accumulators, the arithmetic of dequant4_x2 two lanes per instruction, with
// the checks folded into two bitwise accumulations per element: the two ends of each value's
// uncertainty interval must round to the same float (their bit patterns XOR to 0), and each
// magic-number conversion 0x4B400000 + acc must keep the exponent of 2^23 (|acc| < 2^22: the bits
// above the mantissa XOR to 0 against 0x4B000000).  Returns false when some value of the 16 needs
// the exact f64 path.
__device__ __forceinline__ bool dequant16_x2(const uint32_t (&r)[16], const float (&hs)[16], const float (&ls)[16],
                                             float (&v)[16]) {
  const f2_t magic = f2(-12582912.0f, -12582912.0f);
  const f2_t e40 = f2(0x1p-40f, 0x1p-40f), ne40 = f2(-0x1p-40f, -0x1p-40f);
  uint32_t bad = 0, range = 0;
#pragma unroll
  for (int j = 0; j < 16; j += 2) {
    const uint32_t x0 = 0x4B400000u + r[j], x1 = 0x4B400000u + r[j + 1];
    range |= x0 ^ 0x4B000000u;
    range |= x1 ^ 0x4B000000u;
    const f2_t a = f2_add(f2(__uint_as_float(x0), __uint_as_float(x1)), magic);
    const f2_t h = f2(hs[j], hs[j + 1]);
    const f2_t pl = f2_mul(a, f2(ls[j], ls[j + 1]));
    const f2_t yl = f2_fma(a, h, f2_fma(a, f2_mul(h, ne40), pl));
    const f2_t yh = f2_fma(a, h, f2_fma(a, f2_mul(h, e40), pl));
    float l0, l1, h0, h1;
    f2_split(yl, l0, l1);
    f2_split(yh, h0, h1);
    v[j] = l0;
    v[j + 1] = l1;
    bad |= __float_as_uint(l0) ^ __float_as_uint(h0);
    bad |= __float_as_uint(l1) ^ __float_as_uint(h1);
  }
  return (bad | (range & 0xFF800000u)) == 0;
}

// Requantization of 16 values, two per instruction: clip(round_half_even(RN(y / s)), -127, 127)
// as bytes.  y is clamped to +-c127 = +-RN(127 s) first, so every quotient lies in [-127, 127]
// after rounding and no clip is needed afterwards (RN(c127 / s) rounds to 127; infinities map to
// +-127); then Markstein's correction of RN(y * RN(1/s)) and the 1.5 * 2^23 rounding add.
// Checked against the reference formula on 3e8 random cases (ties, values next to the clip).
// NONNEG: the values are known to be >= 0 (or NaN), so only the upper clamp is applied.
template <int N, bool NONNEG = false>
__device__ __forceinline__ void requant_x2(const float (&v)[N], float s, float rcp, float c127, uint32_t (&b)[N]) {
  static_assert(N % 2 == 0, "values come in pairs");
  const f2_t r2 = f2(rcp, rcp), ns = f2(-s, -s), magic = f2(12582912.0f, 12582912.0f);
#pragma unroll
  for (int j = 0; j < N; j += 2) {
    const f2_t y = NONNEG ? f2(fminf(v[j], c127), fminf(v[j + 1], c127))
                          : f2(fminf(fmaxf(v[j], -c127), c127), fminf(fmaxf(v[j + 1], -c127), c127));
    const f2_t q0 = f2_mul(y, r2);
    const f2_t z = f2_fma(f2_fma(q0, ns, y), r2, q0);
    float t0, t1;
    f2_split(f2_add(z, magic), t0, t1);
    b[j] = static_cast<uint32_t>(__float_as_int(t0));
    b[j + 1] = static_cast<uint32_t>(__float_as_int(t1));
  }
}
__device__ __forceinline__ void requant16_x2(const float (&v)[16], float s, float rcp, float c127, uint32_t (&b)[16]) {
  requant_x2<16>(v, s, rcp, c127, b);
}

// clip(rint(z), -127, 127) as an int8 in the low byte of the returned word: clipping before
// rounding is equivalent because +-127 are integers; z + 1.5*2^23 rounds z half-to-even into the
// low mantissa bits.
__device__ __forceinline__ uint32_t round_clip_i8(float z) {
  z = fminf(fmaxf(z, -127.0f), 127.0f);
  return static_cast<uint32_t>(__float_as_int(__fadd_rn(z, 12582912.0f)));
}

__device__ __forceinline__ uint32_t pack4_i8(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  const uint32_t ab = __byte_perm(a, b, 0x0040);
  const uint32_t cd = __byte_perm(c, d, 0x0040);
  return __byte_perm(ab, cd, 0x5410);
}

// NumPy float32 maximum/minimum: a NaN on either side propagates (PTX max.NaN / min.NaN).  The
// one difference from NumPy is the sign of a zero result when +0.0 meets -0.0 (NumPy returns the
// first operand); both quantize to 0.
__device__ __forceinline__ float np_maximum(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float np_minimum(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Reference ops.py:94-96 (tanh form of GELU), evaluated in the same order in float32.  tanhf and
// expf are CUDA's; NumPy's own float32 tanh/exp differ in the last bits, so steps that use them
// match the reference within a tolerance, not bit for bit.
__device__ __forceinline__ float gelu_f32(float x) {
  const float x3 = __fmul_rn(__fmul_rn(x, x), x);
  const float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

__device__ __forceinline__ float sigmoid_f32(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
}

__device__ __forceinline__ float apply_unary(int op, float v) {
  switch (op) {
    case MIRA_EPI_RELU: return np_maximum(v, 0.0f);
    case MIRA_EPI_GELU: return gelu_f32(v);
    case MIRA_EPI_SIGMOID: return sigmoid_f32(v);
    case MIRA_EPI_TANH: return tanhf(v);
    default: return v;
  }
}

__device__ __forceinline__ float apply_binary(int op, float a, float b) {
  switch (op) {
    case MIRA_EPI_ADD: return __fadd_rn(a, b);
    case MIRA_EPI_SUB: return __fsub_rn(a, b);
    case MIRA_EPI_MUL: return __fmul_rn(a, b);
    case MIRA_EPI_DIV: return __fdiv_rn(a, b);
    case MIRA_EPI_MAXIMUM: return np_maximum(a, b);
    case MIRA_EPI_MINIMUM: return np_minimum(a, b);
    default: return a;
  }
}

}  // namespace mira
