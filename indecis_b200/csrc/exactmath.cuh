// Float32 functions of the reference's int8 path, evaluated with explicit
// IEEE roundings (every multiply, add and fused multiply-add is spelled out),
// so the device produces the reference's bits, not CUDA's libm results:
//   exp: Cephes expf as linalg/vec_simd.go:216-264 (vector body, FMA) and
//        linalg/fastmath.go:35-51 (scalar tail, no FMA);
//   GELU(erf) x gate: the Eigen/XLA erf rational of linalg/fastmath.go:7-26,
//        in the FMA order of linalg/gelu_amd64.s:165-225;
//   GELU(tanh): x / (1 + exp(-2u)) as linalg/vec_simd.go:166-197 (vector body,
//        FMA) and fastmath.go:28-32 (scalar tail), IEEE division.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace ig {

// Vector-body exp of v = x - m (ExpShift, vec_simd.go:235-248).
__device__ __forceinline__ float exp_body(float v) {
  const bool under = v < -87.3f;
  v = fminf(fmaxf(v, -87.3f), 88.7f);
  float n = __fsub_rn(__fmaf_rn(v, 1.44269504088896341f, 12582912.0f), 12582912.0f);
  float r = __fmaf_rn(n, -0.693359375f, v);
  r = __fmaf_rn(n, 2.12194440e-4f, r);
  float p = __fmaf_rn(r, 1.9875691500e-4f, 1.3981999507e-3f);
  p = __fmaf_rn(r, p, 8.3334519073e-3f);
  p = __fmaf_rn(r, p, 4.1665795894e-2f);
  p = __fmaf_rn(r, p, 1.6666665459e-1f);
  p = __fmaf_rn(r, p, 5.0000001201e-1f);
  float y = __fadd_rn(__fmaf_rn(__fmul_rn(p, r), r, r), 1.0f);
  const int ni = __float2int_rn(n);
  const float pw = __int_as_float((ni + 127) << 23);
  return under ? 0.0f : __fmul_rn(y, pw);
}

// exp_body for two lanes (packed f32x2 steps, each rounding as the scalar one;
// no packed add is fed by a packed multiply).
__device__ __forceinline__ float2 exp_body2(float2 v) {
  const bool ux = v.x < -87.3f, uy = v.y < -87.3f;
  v.x = fminf(fmaxf(v.x, -87.3f), 88.7f);
  v.y = fminf(fmaxf(v.y, -87.3f), 88.7f);
  const float2 t = __ffma2_rn(v, make_float2(1.44269504088896341f, 1.44269504088896341f),
                              make_float2(12582912.0f, 12582912.0f));
  const float2 n = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));
  float2 r = __ffma2_rn(n, make_float2(-0.693359375f, -0.693359375f), v);
  r = __ffma2_rn(n, make_float2(2.12194440e-4f, 2.12194440e-4f), r);
  float2 p = __ffma2_rn(r, make_float2(1.9875691500e-4f, 1.9875691500e-4f), make_float2(1.3981999507e-3f, 1.3981999507e-3f));
  p = __ffma2_rn(r, p, make_float2(8.3334519073e-3f, 8.3334519073e-3f));
  p = __ffma2_rn(r, p, make_float2(4.1665795894e-2f, 4.1665795894e-2f));
  p = __ffma2_rn(r, p, make_float2(1.6666665459e-1f, 1.6666665459e-1f));
  p = __ffma2_rn(r, p, make_float2(5.0000001201e-1f, 5.0000001201e-1f));
  const float2 y = __fadd2_rn(__ffma2_rn(__fmul2_rn(p, r), r, r), make_float2(1.0f, 1.0f));
  // 2^n from t's bits (0x4B400000 + n): (n + 127) << 23.
  const float px = __int_as_float((__float_as_int(t.x) << 23) + ((127 - 0x4B400000) << 23));
  const float py = __int_as_float((__float_as_int(t.y) << 23) + ((127 - 0x4B400000) << 23));
  return make_float2(ux ? 0.0f : __fmul_rn(y.x, px), uy ? 0.0f : __fmul_rn(y.y, py));
}

// Scalar-tail exp (exp32, fastmath.go:35-51): separate roundings throughout.
__device__ __forceinline__ float exp_tail(float x) {
  if (x < -87.3f) return 0.0f;
  x = fminf(x, 88.7f);
  float n = __fsub_rn(__fadd_rn(__fmul_rn(x, 1.44269504088896341f), 12582912.0f), 12582912.0f);
  float r = __fsub_rn(x, __fmul_rn(n, 0.693359375f));
  r = __fsub_rn(r, __fmul_rn(n, -2.12194440e-4f));
  float p = 1.9875691500e-4f;
  p = __fadd_rn(__fmul_rn(p, r), 1.3981999507e-3f);
  p = __fadd_rn(__fmul_rn(p, r), 8.3334519073e-3f);
  p = __fadd_rn(__fmul_rn(p, r), 4.1665795894e-2f);
  p = __fadd_rn(__fmul_rn(p, r), 1.6666665459e-1f);
  p = __fadd_rn(__fmul_rn(p, r), 5.0000001201e-1f);
  float y = __fadd_rn(__fadd_rn(__fmul_rn(__fmul_rn(p, r), r), r), 1.0f);
  const int ni = __float2int_rn(n);
  return __fmul_rn(y, __int_as_float((ni + 127) << 23));
}

// Element t of an ExpShift over `len` values with V lanes: the vector body
// covers t < (len / V) * V, exp32 the rest.
__device__ __forceinline__ float exp_shift_at(float x, float m, int t, int len, int V) {
  const float v = __fsub_rn(x, m);
  return t < (len / V) * V ? exp_body(v) : exp_tail(v);
}

// ---- two lanes at once (f32x2: each lane rounds exactly as the scalar op) ----
// Caution: a packed add fed directly by a packed multiply may be contracted
// into one fused multiply-add by the compiler (the scalar __f*_rn intrinsics
// are never contracted). The helpers below have no multiply-then-add step;
// callers that subtract from a packed product use the scalar __fsub_rn.

__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// max(a, b) that returns NaN when either input is NaN (fmaxf ignores NaN).
// A row maximum taken with it is NaN exactly when the row holds a NaN.
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// Row quantization (linalg/int8.go:157-191 quantizeA): a scale RN(max/127)
// that is a normal float lets every byte take the fast rounding; otherwise
// (NaN rows, subnormal or infinite scales) each byte takes the clamped path.
__device__ __forceinline__ bool row_scale_normal(float s) { return s >= 1.17549435e-38f && s <= 3.40282347e38f; }

// Byte q + 128 of one value of a row whose maximum is not 0 (clamped path:
// any scale).
__device__ __forceinline__ uint32_t quant_byte_slow(float v, float inv) {
  return (uint32_t)(max(-128, min(127, rne_int(__fmul_rn(v, inv)))) + 128);
}

// Integer <-> float without a conversion instruction (those run at an eighth
// of the FP32 rate). For an integer |v| < 2^22 the bits 0x4B400000 + v are the
// float 1.5*2^23 + v exactly; and for a float |x| < 2^22, x + 1.5*2^23 is
// rounded to nearest-even at unit spacing, so its bits minus 0x4B400000 are
// rne(x), the value __float2int_rn gives.
constexpr float kMagic = 12582912.0f;
constexpr int kMagicBits = 0x4B400000;
__device__ __forceinline__ float magic_float(int32_t v) { return __int_as_float(kMagicBits + v); }
__device__ __forceinline__ int magic_rne(float x) { return __float_as_int(__fadd_rn(x, kMagic)) - kMagicBits; }

// The softmax weight bits of ExpShift's vector body for two scores:
// 0x4B400000 + P with P = rne(RN(e * 255)), e = exp_body(v), for v <= 0 (a
// score minus its row's maximum). Every P equals rne(RN(exp_body(v) * 255)):
//   - the upper clamp cannot apply; below -87.3, exp_body's 0 and the value
//     at the clamp both give e*255 < 0.5, so P = 0 either way;
//   - e = y * 2^n (y the polynomial, n from t = v*log2e + 1.5*2^23, whose
//     bits hold 0x4B400000 + n) is exact while normal, so RN(e * 255) = RN(y * 255) * 2^n,
//     and RN(RN(y * 255) * 2^n + 1.5*2^23) (one fused step, the product being
//     exact) holds rne of it in its low bits; where e or e*255 would be
//     subnormal both sides give P = 0.
__device__ __forceinline__ uint2 exp_p_bits2(float2 v) {
  v.x = fmaxf(v.x, -87.3f);
  v.y = fmaxf(v.y, -87.3f);
  const float2 t = __ffma2_rn(v, f2(1.44269504088896341f), f2(kMagic));
  const float2 n = __fadd2_rn(t, f2(-kMagic));
  float2 r = __ffma2_rn(n, f2(-0.693359375f), v);
  r = __ffma2_rn(n, f2(2.12194440e-4f), r);
  float2 p = __ffma2_rn(r, f2(1.9875691500e-4f), f2(1.3981999507e-3f));
  p = __ffma2_rn(r, p, f2(8.3334519073e-3f));
  p = __ffma2_rn(r, p, f2(4.1665795894e-2f));
  p = __ffma2_rn(r, p, f2(1.6666665459e-1f));
  p = __ffma2_rn(r, p, f2(5.0000001201e-1f));
  const float2 y = __fadd2_rn(__ffma2_rn(__fmul2_rn(p, r), r, r), f2(1.0f));
  const float2 z = __fmul2_rn(y, f2(255.0f));
  // 2^n from t's bits (0x4B400000 + n): (n + 127) << 23.
  const float2 pw = make_float2(__int_as_float((__float_as_int(t.x) << 23) + ((127 - kMagicBits) << 23)),
                                __int_as_float((__float_as_int(t.y) << 23) + ((127 - kMagicBits) << 23)));
  const float2 b = __ffma2_rn(z, pw, f2(kMagic));
  return make_uint2(__float_as_uint(b.x), __float_as_uint(b.y));
}

// dequant2 for |acc| < 2^22 with zcm = zc + 1.5*2^23 (exact while
// |zc| < 2^22): (1.5*2^23 + acc) - zcm is acc - zc, an integer below 2^23 in
// magnitude, so it is exact, as float(acc) - zc is.
__device__ __forceinline__ float2 dequant2m(int32_t a0, int32_t a1, float2 zcm, float2 sb, float sa) {
  float2 v = __fadd2_rn(make_float2(magic_float(a0), magic_float(a1)), make_float2(-zcm.x, -zcm.y));
  v = __fmul2_rn(v, sb);
  return __fmul2_rn(v, f2(sa));
}

// ((float(acc) - zc) * sb) * sa for two columns.
__device__ __forceinline__ float2 dequant2(int32_t a0, int32_t a1, float2 zc, float2 sb, float sa) {
  float2 v = __fadd2_rn(make_float2(__int2float_rn(a0), __int2float_rn(a1)), make_float2(-zc.x, -zc.y));
  v = __fmul2_rn(v, sb);
  return __fmul2_rn(v, f2(sa));
}

// p / q rounded to nearest for the erf rational of the GELU vector body,
// without the IEEE division's special-case path: a hardware reciprocal
// estimate, one Newton-Raphson step r = r + r(1 - qr), the quotient y = RN(p r)
// and Markstein's remainder correction y + (p - q y) r with exact FMA
// remainders (P. Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990; J.-M. Muller et
// al., Handbook of Floating-Point Arithmetic, division by FMA). Used only
// where q is the erf denominator of gelu_mul_fma(2): t in [-4, 4] gives
// q in [-2.4, -0.0142] and |p| <= |q|, so every intermediate is a normal
// number or zero. ig_check_gelu_division compares it with the IEEE quotient
// for every float t in [-4, 4] (tests/test_gpu_gelu_division.py): equal bits.
__device__ __forceinline__ float div_erf(float p, float q) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(q));
  r = __fmaf_rn(r, __fmaf_rn(-q, r, 1.0f), r);
  const float y = __fmul_rn(p, r);
  return __fmaf_rn(__fmaf_rn(-q, y, p), r, y);
}
__device__ __forceinline__ float2 div_erf2(float2 p, float2 q) {
  float2 r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(q.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(q.y));
  const float2 nq = make_float2(-q.x, -q.y);
  r = __ffma2_rn(r, __ffma2_rn(nq, r, make_float2(1.0f, 1.0f)), r);
  const float2 y = __fmul2_rn(p, r);
  return __ffma2_rn(__ffma2_rn(nq, y, p), r, y);
}

// The erf rational's numerator and denominator of gelu_mul_fma for a clamped
// t (gelu_amd64.s:176-195).
__device__ __forceinline__ void erf_pq_fma(float t, float &p, float &q) {
  const float t2 = __fmul_rn(t, t);
  p = __fmaf_rn(t2, -2.72614225801306e-10f, 2.77068142495902e-08f);
  p = __fmaf_rn(t2, p, -2.10102402082508e-06f);
  p = __fmaf_rn(t2, p, -5.69250639462346e-05f);
  p = __fmaf_rn(t2, p, -7.34990630326855e-04f);
  p = __fmaf_rn(t2, p, -2.95459980854025e-03f);
  p = __fmaf_rn(t2, p, -1.60960333262415e-02f);
  p = __fmul_rn(p, t);
  q = __fmaf_rn(t2, -1.45660718464996e-05f, -2.13374055278905e-04f);
  q = __fmaf_rn(t2, q, -1.68282697438203e-03f);
  q = __fmaf_rn(t2, q, -7.37332916720468e-03f);
  q = __fmaf_rn(t2, q, -1.42647390514189e-02f);
}

// gelu_mul_fma for two elements.
__device__ __forceinline__ float2 gelu_mul_fma2(float2 x, float2 gate) {
  float2 t = __fmul2_rn(x, f2(0.7071067811865476f));
  t.x = fminf(fmaxf(t.x, -4.0f), 4.0f);
  t.y = fminf(fmaxf(t.y, -4.0f), 4.0f);
  const float2 t2 = __fmul2_rn(t, t);
  float2 p = __ffma2_rn(t2, f2(-2.72614225801306e-10f), f2(2.77068142495902e-08f));
  p = __ffma2_rn(t2, p, f2(-2.10102402082508e-06f));
  p = __ffma2_rn(t2, p, f2(-5.69250639462346e-05f));
  p = __ffma2_rn(t2, p, f2(-7.34990630326855e-04f));
  p = __ffma2_rn(t2, p, f2(-2.95459980854025e-03f));
  p = __ffma2_rn(t2, p, f2(-1.60960333262415e-02f));
  p = __fmul2_rn(p, t);
  float2 q = __ffma2_rn(t2, f2(-1.45660718464996e-05f), f2(-2.13374055278905e-04f));
  q = __ffma2_rn(t2, q, f2(-1.68282697438203e-03f));
  q = __ffma2_rn(t2, q, f2(-7.37332916720468e-03f));
  q = __ffma2_rn(t2, q, f2(-1.42647390514189e-02f));
  float2 r = div_erf2(p, q);
  r = __fadd2_rn(r, f2(1.0f));
  const float2 g = __fmul2_rn(r, __fmul2_rn(x, f2(0.5f)));
  return __fmul2_rn(g, gate);
}

// geluMulAVX2 for one element (gelu_amd64.s:176-200).
__device__ __forceinline__ float gelu_mul_fma(float x, float gate) {
  float t = __fmul_rn(x, 0.7071067811865476f);
  t = fmaxf(t, -4.0f);
  t = fminf(t, 4.0f);
  const float t2 = __fmul_rn(t, t);
  float p = __fmaf_rn(t2, -2.72614225801306e-10f, 2.77068142495902e-08f);
  p = __fmaf_rn(t2, p, -2.10102402082508e-06f);
  p = __fmaf_rn(t2, p, -5.69250639462346e-05f);
  p = __fmaf_rn(t2, p, -7.34990630326855e-04f);
  p = __fmaf_rn(t2, p, -2.95459980854025e-03f);
  p = __fmaf_rn(t2, p, -1.60960333262415e-02f);
  p = __fmul_rn(p, t);
  float q = __fmaf_rn(t2, -1.45660718464996e-05f, -2.13374055278905e-04f);
  q = __fmaf_rn(t2, q, -1.68282697438203e-03f);
  q = __fmaf_rn(t2, q, -7.37332916720468e-03f);
  q = __fmaf_rn(t2, q, -1.42647390514189e-02f);
  float r = div_erf(p, q);
  r = __fadd_rn(r, 1.0f);
  const float g = __fmul_rn(r, __fmul_rn(x, 0.5f));
  return __fmul_rn(g, gate);
}

// geluScalar(x) * gate (fastmath.go:9-26): the tail of GeluMul when the row
// length is not a multiple of 16.
__device__ __forceinline__ float gelu_mul_scalar(float x, float gate) {
  float e = __fmul_rn(x, 0.7071067811865476f);
  e = fminf(fmaxf(e, -4.0f), 4.0f);
  const float x2 = __fmul_rn(e, e);
  float p = __fadd_rn(__fmul_rn(x2, -2.72614225801306e-10f), 2.77068142495902e-08f);
  p = __fadd_rn(__fmul_rn(x2, p), -2.10102402082508e-06f);
  p = __fadd_rn(__fmul_rn(x2, p), -5.69250639462346e-05f);
  p = __fadd_rn(__fmul_rn(x2, p), -7.34990630326855e-04f);
  p = __fadd_rn(__fmul_rn(x2, p), -2.95459980854025e-03f);
  p = __fadd_rn(__fmul_rn(x2, p), -1.60960333262415e-02f);
  p = __fmul_rn(p, e);
  float q = __fadd_rn(__fmul_rn(x2, -1.45660718464996e-05f), -2.13374055278905e-04f);
  q = __fadd_rn(__fmul_rn(x2, q), -1.68282697438203e-03f);
  q = __fadd_rn(__fmul_rn(x2, q), -7.37332916720468e-03f);
  q = __fadd_rn(__fmul_rn(x2, q), -1.42647390514189e-02f);
  const float erf = __fdiv_rn(p, q);
  const float g = __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erf));
  return __fmul_rn(g, gate);
}

// GeluMul element i of a row of n values (vec_simd.go:121-160 on amd64:
// the first n &^ 15 go through the AVX2 kernel).
__device__ __forceinline__ float gelu_mul_at(float x, float gate, int i, int n) {
  return i < (n & ~15) ? gelu_mul_fma(x, gate) : gelu_mul_scalar(x, gate);
}

// ---- GELU, tanh form: x * sigmoid(2u), u = sqrt(2/pi) * (x + 0.044715 x^3) ----

// The vector body of linalg.GeluTanh (vec_simd.go:166-197), one lane: the
// exponent of Cephes' expf with FMA, then an IEEE division.
__device__ __forceinline__ float gelu_tanh_body(float x) {
  float v = __fmul_rn(x, x);
  v = __fmaf_rn(v, 0.044715f, 1.0f);
  v = __fmul_rn(v, x);
  v = __fmul_rn(v, -1.5957691216057308f);  // -2*sqrt(2/pi), rounded once to float32
  v = fminf(fmaxf(v, -87.3f), 88.7f);
  const float n = __fsub_rn(__fmaf_rn(v, 1.44269504088896341f, 12582912.0f), 12582912.0f);
  float r = __fmaf_rn(n, -0.693359375f, v);
  r = __fmaf_rn(n, 2.12194440e-4f, r);
  float p = __fmaf_rn(r, 1.9875691500e-4f, 1.3981999507e-3f);
  p = __fmaf_rn(r, p, 8.3334519073e-3f);
  p = __fmaf_rn(r, p, 4.1665795894e-2f);
  p = __fmaf_rn(r, p, 1.6666665459e-1f);
  p = __fmaf_rn(r, p, 5.0000001201e-1f);
  const float y = __fadd_rn(__fmaf_rn(__fmul_rn(p, r), r, r), 1.0f);
  const float pw = __int_as_float((__float2int_rn(n) + 127) << 23);
  return __fdiv_rn(x, __fadd_rn(1.0f, __fmul_rn(y, pw)));
}

// gelu_tanh_body for two lanes: the same roundings with paired f32x2
// operations wherever a packed add is not fed by a packed multiply; the
// final 1 + y*2^n and the division stay scalar.
__device__ __forceinline__ float2 gelu_tanh_body2(float2 x) {
  float2 v = __fmul2_rn(x, x);
  v = __ffma2_rn(v, f2(0.044715f), f2(1.0f));
  v = __fmul2_rn(v, x);
  v = __fmul2_rn(v, f2(-1.5957691216057308f));
  v.x = fminf(fmaxf(v.x, -87.3f), 88.7f);
  v.y = fminf(fmaxf(v.y, -87.3f), 88.7f);
  const float2 t = __ffma2_rn(v, f2(1.44269504088896341f), f2(kMagic));
  const float2 n = __fadd2_rn(t, f2(-kMagic));
  float2 r = __ffma2_rn(n, f2(-0.693359375f), v);
  r = __ffma2_rn(n, f2(2.12194440e-4f), r);
  float2 p = __ffma2_rn(r, f2(1.9875691500e-4f), f2(1.3981999507e-3f));
  p = __ffma2_rn(r, p, f2(8.3334519073e-3f));
  p = __ffma2_rn(r, p, f2(4.1665795894e-2f));
  p = __ffma2_rn(r, p, f2(1.6666665459e-1f));
  p = __ffma2_rn(r, p, f2(5.0000001201e-1f));
  const float2 y = __fadd2_rn(__ffma2_rn(__fmul2_rn(p, r), r, r), f2(1.0f));
  // 2^n from t's bits (0x4B400000 + n): (n + 127) << 23.
  const float pwx = __int_as_float((__float_as_int(t.x) << 23) + ((127 - kMagicBits) << 23));
  const float pwy = __int_as_float((__float_as_int(t.y) << 23) + ((127 - kMagicBits) << 23));
  return make_float2(__fdiv_rn(x.x, __fadd_rn(1.0f, __fmul_rn(y.x, pwx))),
                     __fdiv_rn(x.y, __fadd_rn(1.0f, __fmul_rn(y.y, pwy))));
}

// geluTanhScalar (fastmath.go:28-32): separate roundings, exp32.
__device__ __forceinline__ float gelu_tanh_tail(float x) {
  const float t = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  const float u = __fmul_rn(0.7978845608028654f, __fadd_rn(x, t));
  return __fdiv_rn(x, __fadd_rn(1.0f, exp_tail(__fmul_rn(-2.0f, u))));
}

// Element i of a GeluTanh call over len values with V lanes.
__device__ __forceinline__ float gelu_tanh_at(float x, long long i, long long len, int V) {
  return i < len - len % V ? gelu_tanh_body(x) : gelu_tanh_tail(x);
}

// ---- per-row int8 quantization pieces (attention8.go:210-269) ----------------

// max(0, |v[0]|, ..., |v[31]|), NaN-propagating (PROP) or NaN-ignoring, as a
// tree of four chains: both maxima are associative (max.NaN returns the
// canonical NaN), so the value is the one chain's.
template <bool PROP>
__device__ __forceinline__ float absmax32(const float (&v)[32]) {
  float m[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int u = 0; u < 32; u++) m[u & 3] = PROP ? fmax_nan(m[u & 3], fabsf(v[u])) : fmaxf(m[u & 3], fabsf(v[u]));
  return PROP ? fmax_nan(fmax_nan(m[0], m[1]), fmax_nan(m[2], m[3])) : fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}

// x with its sign bit set.
__device__ __forceinline__ float neg_bits(float x) { return __int_as_float(__float_as_int(x) | 0x80000000); }

// The low bytes of four words as one word (byte k from word k).
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Byte of clamp(rne(x)) (two's complement) in the low byte of the result
// (rne as the reference's VCVTPS2DQ; any scale).
__device__ __forceinline__ uint32_t quant_bits(float x) { return (uint32_t)max(-128, min(127, rne_int(x))); }

// For a row (or column) maximum m > 0 whose scale RN(m/127) is a normal
// float, every |x * inv| with |x| <= m is below 127 + 2^-20, so rne(x * inv)
// stays in [-127, 127] and the int8 clamp never applies.
__device__ __forceinline__ bool scale_is_normal(float scale) {
  return scale >= 1.17549435e-38f && scale <= 3.40282347e38f;
}

// Four bytes q + 128, q = rne(x * inv), for a normal scale and finite
// values: the product rounded, then + (1.5*2^23 + 128), whose low byte is
// q + 128.
__device__ __forceinline__ uint32_t quant4_fast(float a, float b, float c, float d, float2 inv01, float2 inv23) {
  const float2 p0 = __fmul2_rn(make_float2(a, b), inv01), p1 = __fmul2_rn(make_float2(c, d), inv23);
  constexpr float m = kMagic + 128.0f;
  return pack_low_bytes(__float_as_uint(__fadd_rn(p0.x, m)), __float_as_uint(__fadd_rn(p0.y, m)),
                        __float_as_uint(__fadd_rn(p1.x, m)), __float_as_uint(__fadd_rn(p1.y, m)));
}
// The same bytes as int8 q (two's complement): q + 128 with the top bit
// flipped.
__device__ __forceinline__ uint32_t quant4_fast_s8(float a, float b, float c, float d, float2 inv01, float2 inv23) {
  return quant4_fast(a, b, c, d, inv01, inv23) ^ 0x80808080u;
}

}  // namespace ig
