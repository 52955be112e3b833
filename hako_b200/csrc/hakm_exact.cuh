// hakm_exact.cuh — the reference's floating-point steps as its own build
// performs them, for the device.
//
// The reference is compiled with -O3 -ffast-math for x86-64 with AVX2 and
// FMA (its Makefile:8 flags). That build fixes every rounding of the hot
// path: how the dot products are split over the 8 lanes of a 256-bit
// vector and folded, which products are fused, that 1.0f/sqrtf becomes the
// rsqrtss estimate plus one Newton step, and which exp routine each softmax
// element goes through (glibc's scalar expf, or libmvec's 8- or 4-wide
// vector expf). The helpers below restate those steps with explicit IEEE
// operations (__fadd_rn, __fmul_rn, __fmaf_rn: nothing is left to the
// compiler's contraction), so the kernels reproduce the reference's
// results bit for bit.
#pragma once
#include "hakm_device.cuh"

namespace hakm {

// ------------------------------------------------------------ packed fp32
// Two independent IEEE fp32 operations in one instruction (sm_100): the
// same roundings as two scalar operations. Unlike the scalar __fmul_rn /
// __fadd_rn, a packed add whose operand comes straight from a packed
// multiply can be contracted into a packed FMA by the assembler (measured
// on this toolchain): a sum of rounded products adds them with __fadd_rn.
__device__ __forceinline__ uint64_t f2_bits(float2 a) {
  return (uint64_t)__float_as_uint(a.x) | ((uint64_t)__float_as_uint(a.y) << 32);
}
__device__ __forceinline__ float2 f2_of(uint64_t r) {
  return make_float2(__uint_as_float((uint32_t)r), __uint_as_float((uint32_t)(r >> 32)));
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_of(r);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_of(r);
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return f2_of(r);
}

// ------------------------------------------------------------ reductions
// Fold of an 8-lane accumulator as gcc emits it for a vectorized reduction
// (vextractf128 / movhlps / shufps): ((a1+a5)+(a3+a7)) + ((a0+a4)+(a2+a6)).
// Lanes 8g..8g+7 of a warp hold a0..a7 of group g; every lane of the group
// gets the fold (IEEE addition is commutative, so both partners of each
// shuffle compute the same value).
__device__ __forceinline__ float fold8_lanes(float a) {
  const float s = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));
  const float u = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
  return __fadd_rn(u, __shfl_xor_sync(0xffffffffu, u, 1));
}
__device__ __forceinline__ float fold8(const float a[8]) {
  const float s0 = __fadd_rn(a[0], a[4]), s1 = __fadd_rn(a[1], a[5]);
  const float s2 = __fadd_rn(a[2], a[6]), s3 = __fadd_rn(a[3], a[7]);
  return __fadd_rn(__fadd_rn(s0, s2), __fadd_rn(s1, s3));
}

// ------------------------------------------------------------ 1/sqrtf
// rsqrtss: an estimate fixed by the exponent's parity and the top 10
// mantissa bits. `tab` holds the host instruction's 2048 results for [1, 4)
// (tab[par * 1024 + m10] for 2^par * 1.m); other inputs scale the exponent
// by one per factor of four. Positive normal inputs (the reference's).
__device__ __forceinline__ float rsqrt_est(float v, const uint32_t* tab) {
  const uint32_t u = __float_as_uint(v);
  const int E = (int)(u >> 23) - 127, par = E & 1, k = (E - par) / 2;
  const uint32_t r = __ldg(tab + par * 1024 + ((u >> 13) & 1023));
  return __uint_as_float(r - ((uint32_t)k << 23));
}
// 1.0f/sqrtf(v) as built: r = rsqrtss(v); (r * -0.5) * fma(r, v * r, -3).
__device__ __forceinline__ float rsqrt_nr(float v, const uint32_t* tab) {
  const float r = rsqrt_est(v, tab);
  const float t = __fmaf_rn(r, __fmul_rn(v, r), -3.0f);
  return __fmul_rn(__fmul_rn(r, -0.5f), t);
}

// ------------------------------------------------------------ expf
// glibc's scalar expf: the published exp2f-table method. x*32/ln2 = k + r
// (|r| <= 1/2, k rounded to nearest by the 1.5*2^52 shifter), 2^(k/32) from
// a 32-entry table, a cubic in r, everything in double and one rounding to
// float at the end. Table entry i is 2^(i/32) rounded to double, stored
// minus i << 47 (the exponent bits the index adds back).
__device__ __constant__ uint64_t kExp2Tab[32] = {
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL,
    0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL,
    0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL,
    0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL,
    0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL,
    0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL,
    0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL,
    0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL};

__device__ __forceinline__ float exp_scalar(float x) {
  const uint32_t ax = __float_as_uint(x) & 0x7FFFFFFFu;
  if (ax >= 0x42B00000u) {  // |x| >= 88, inf, nan
    if (__float_as_uint(x) == 0xFF800000u) return 0.0f;
    if (ax >= 0x7F800000u) return __fadd_rn(x, x);
    if (x > 0x1.62e42ep6f) return __uint_as_float(0x7F800000u);
    if (x < -0x1.9fe368p6f) return 0.0f;
  }
  const double kInvLn2N = 0x1.71547652b82fep+0 * 32, kShift = 0x1.8p+52;
  const double kC0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, kC1 = 0x1.ebfce50fac4f3p-3 / 32 / 32,
               kC2 = 0x1.62e42ff0c52d6p-1 / 32;
  const double xd = (double)x, z = __dmul_rn(kInvLn2N, xd);
  double kd = __dadd_rn(z, kShift);
  const uint64_t ki = (uint64_t)__double_as_longlong(kd);
  kd = __dsub_rn(kd, kShift);
  const double r = __fma_rn(kInvLn2N, xd, -kd);
  const uint64_t t = kExp2Tab[ki & 31] + (ki << 47);
  const double s = __longlong_as_double((long long)t);
  const double zz = __fma_rn(kC0, r, kC1), r2 = __dmul_rn(r, r);
  double y = __fma_rn(kC2, r, 1.0);
  y = __fma_rn(zz, r2, y);
  return __double2float_rn(__dmul_rn(y, s));
}

// libmvec's vector expf, which gcc calls for vectorized exp loops: n =
// rint(x/ln2) through the 1.5*2^23 shifter, r = x - n*ln2 in two parts, a
// degree-5 polynomial for e^r, times 2^n built in the exponent field. The
// 8-wide (AVX2) entry point fuses every step; the 4-wide (SSE4) one rounds
// every product and sum. Lanes with |x| > 87.3365 take the scalar expf.
constexpr uint32_t VX_INVLN2 = 0x3fb8aa3bu, VX_SHIFT = 0x4b400000u, VX_LN2HI = 0x3f317200u,
                   VX_LN2LO = 0x35bfbe8eu, VX_DOM = 0x42aeac4fu;
constexpr uint32_t VX_P0 = 0x3f800000u, VX_P1 = 0x3f7ffffeu, VX_P2 = 0x3effff34u, VX_P3 = 0x3e2aacacu,
                   VX_P4 = 0x3d2b8392u, VX_P5 = 0x3c07d9feu;
__device__ __forceinline__ float U2F(uint32_t u) { return __uint_as_float(u); }

__device__ __forceinline__ float exp_v8(float x) {
  if ((__float_as_uint(x) & 0x7FFFFFFFu) > VX_DOM) return exp_scalar(x);
  const float m = __fmaf_rn(x, U2F(VX_INVLN2), U2F(VX_SHIFT));
  const float n = __fsub_rn(m, U2F(VX_SHIFT));
  float r = __fmaf_rn(-n, U2F(VX_LN2HI), x);
  r = __fmaf_rn(-n, U2F(VX_LN2LO), r);
  float p = __fmaf_rn(U2F(VX_P5), r, U2F(VX_P4));
  p = __fmaf_rn(p, r, U2F(VX_P3));
  p = __fmaf_rn(p, r, U2F(VX_P2));
  p = __fmaf_rn(p, r, U2F(VX_P1));
  p = __fmaf_rn(p, r, U2F(VX_P0));
  return __fmul_rn(p, __uint_as_float((__float_as_uint(m) + 127u) << 23));
}

__device__ __forceinline__ float exp_v4(float x) {
  if ((__float_as_uint(x) & 0x7FFFFFFFu) > VX_DOM) return exp_scalar(x);
  const float m = __fadd_rn(__fmul_rn(x, U2F(VX_INVLN2)), U2F(VX_SHIFT));
  const float n = __fsub_rn(m, U2F(VX_SHIFT));
  float r = __fsub_rn(x, __fmul_rn(n, U2F(VX_LN2HI)));
  r = __fsub_rn(r, __fmul_rn(n, U2F(VX_LN2LO)));
  float p = __fadd_rn(__fmul_rn(U2F(VX_P5), r), U2F(VX_P4));
  p = __fadd_rn(__fmul_rn(p, r), U2F(VX_P3));
  p = __fadd_rn(__fmul_rn(p, r), U2F(VX_P2));
  p = __fadd_rn(__fmul_rn(p, r), U2F(VX_P1));
  p = __fadd_rn(__fmul_rn(p, r), U2F(VX_P0));
  return __fmul_rn(p, __uint_as_float((__float_as_uint(m) + 127u) << 23));
}

// exp(x) of softmax element t of n (src/nn.c:24 as vectorized): the 8-wide
// routine for t < 8*floor(n/8), the 4-wide one for the next 4 when at least
// 4 remain, the scalar expf for the rest.
__device__ __forceinline__ float exp_softmax(float x, int t, int n) {
  const int n8 = n & ~7;
  if (t < n8) return exp_v8(x);
  if (n - n8 >= 4 && t < n8 + 4) return exp_v4(x);
  return exp_scalar(x);
}

// silu(g) * u (src/model.c:154, silu_f src/nn.c:29): scalar expf, one IEEE
// division, one product.
__device__ __forceinline__ float swiglu_exact(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_scalar(-g))), u);
}

}  // namespace hakm
