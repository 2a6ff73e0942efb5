// Bit-level restatements of the reference's CPU numerics, shared by every
// kernel.  The engine is compiled with -fmad=false so that no multiply/add
// pair is contracted; every fused multiply-add below is an explicit
// __fmaf_rn that restates an FMA instruction of the reference.
#pragma once
#include <stdint.h>

namespace ocrvl {

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }

// fastRsqrtF32 (internal/tensor/ops.go:1374-1381): magic-constant guess and
// two Newton steps, unfused.
__device__ __forceinline__ float fast_rsqrt(float x) {
  float half = __fmul_rn(x, 0.5f);
  float y = u2f(0x5f3759dfu - (f2u(x) >> 1));
  y = __fmul_rn(y, __fsub_rn(1.5f, __fmul_rn(__fmul_rn(half, y), y)));
  return __fmul_rn(y, __fsub_rn(1.5f, __fmul_rn(__fmul_rn(half, y), y)));
}

#define OCRVL_LOG2E 0x3FB8AA3Bu
#define OCRVL_C1 0x3F317218u
#define OCRVL_C2 0x3E75FDF0u
#define OCRVL_C3 0x3D635847u
#define OCRVL_C4 0x3C1D955Bu
#define OCRVL_C5 0x3AAF0217u

// FastExpF32 (internal/tensor/ops.go:1099-1112): magic-number rounding,
// unfused degree-5 polynomial, exponent added to the bit pattern.
__device__ __forceinline__ float fast_exp(float x) {
  const float magic = 12582912.0f;
  float t = __fmul_rn(x, u2f(OCRVL_LOG2E));
  int32_t n = (int32_t)__fsub_rn(__fadd_rn(t, magic), magic);
  float f = __fsub_rn(t, (float)n);
  float f2 = __fmul_rn(f, f);
  float a = __fadd_rn(1.0f, __fmul_rn(u2f(OCRVL_C1), f));
  float b = __fadd_rn(u2f(OCRVL_C2), __fmul_rn(u2f(OCRVL_C3), f));
  float d = __fadd_rn(u2f(OCRVL_C4), __fmul_rn(u2f(OCRVL_C5), f));
  float poly = __fadd_rn(a, __fmul_rn(f2, __fadd_rn(b, __fmul_rn(f2, d))));
  return u2f(f2u(poly) + ((uint32_t)n << 23));
}

// Vector exp of expF32VecFMA / siluMulInPlaceFMA (internal/tensor/
// dot_amd64.s:6134-6151, 5670-5687).
__device__ __forceinline__ float exp_fma(float d) {
  float t = __fmul_rn(d, u2f(OCRVL_LOG2E));
  float n = rintf(t);
  float f = __fsub_rn(t, n);
  float f2 = __fmul_rn(f, f);
  float p1 = __fmaf_rn(f, u2f(OCRVL_C1), 1.0f);
  float p2 = __fmaf_rn(f, u2f(OCRVL_C3), u2f(OCRVL_C2));
  float p3 = __fmaf_rn(f, u2f(OCRVL_C5), u2f(OCRVL_C4));
  p2 = __fmaf_rn(f2, p3, p2);
  p1 = __fmaf_rn(f2, p2, p1);
  int32_t ni = (int32_t)n;
  return __fmul_rn(p1, u2f((uint32_t)(ni + 127) << 23));
}

// siluMulInPlaceFMA: (g / (exp(-g) + 1)) * u.
__device__ __forceinline__ float silu_mul(float g, float u) {
  float e = exp_fma(__fsub_rn(0.0f, g));
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(e, 1.0f)), u);
}

// finalizeDotQ8VNNI vector lane (dot_vnni_amd64.s:1043-1090).
__device__ __forceinline__ float vnni_finalize(int32_t dot, int32_t rowsum, float sx, float sw) {
  float d = __fsub_rn((float)dot, __fmul_rn(128.0f, (float)rowsum));
  return __fmul_rn(__fmul_rn(d, sx), sw);
}

// 16-lane ZMM horizontal tree (every reduction tail in the reference asm).
__device__ __forceinline__ float tree16(const float *v) {
  float a[8], b[4];
#pragma unroll
  for (int i = 0; i < 8; i++) a[i] = __fadd_rn(v[i], v[i + 8]);
#pragma unroll
  for (int i = 0; i < 4; i++) b[i] = __fadd_rn(a[i], a[i + 4]);
  return __fadd_rn(__fadd_rn(b[0], b[2]), __fadd_rn(b[1], b[3]));
}

// Order-preserving key for argmax: larger score -> larger key; equal scores
// -> the lower row wins (first maximum, argmax_quant.go).
__device__ __forceinline__ unsigned long long argmax_key(float s, int row) {
  uint32_t u = f2u(s);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)row);
}
__device__ __forceinline__ int argmax_key_row(unsigned long long k) {
  return (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
}

}  // namespace ocrvl
