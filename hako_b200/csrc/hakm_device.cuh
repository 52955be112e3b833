// hakm_device.cuh — device helpers shared by the kernels of libhakm_cuda.
#pragma once
#include <cuda_fp16.h>
#include <math_constants.h>

#include "hakm_internal.h"

namespace hakm {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_isum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
  return __half2float(__ushort_as_half((unsigned short)(h16 & 0xFFFFu)));
}

// Float -> int8 as the reference's (int)lrintf + clamp compiles with its own
// flags (src/quant.c:138-141): round half to even through a 64-bit
// conversion truncated to 32 bits; NaN and infinities give 0 (the 64-bit
// result is INT64_MIN). Here r = x * (127/amax) with |x| <= amax, so r is
// either within 127 * (1 + 2^-22), or infinite (127/amax overflowed for
// amax < 2^-121), or NaN: on that set a 32-bit round-to-nearest-even
// conversion behind a range check gives the same integers.
__device__ __forceinline__ int q8_round(float r) {
  const int v = fabsf(r) < 2147483648.0f ? __float2int_rn(r) : 0;
  return v > 127 ? 127 : (v < -127 ? -127 : v);
}

// Per-32 quantization step of quantize_row_q8_32 as built with -ffast-math:
// xs = amax * fl(1/127), inv = 127 / amax (one IEEE division).
__device__ __forceinline__ float q8_inv(float amax, float scale) {
  return scale > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
}

// NeoX RoPE rotation of the pair (a, b) with the roundings of the reference
// as built (src/nn.c:38-40 under gcc -O3 -ffast-math with FMA): the b
// products are rounded on their own, the a products fused:
//   a' = fma(a, c, -(b*s)),  b' = fma(a, s, b*c).
__device__ __forceinline__ float2 rope_rotate(float a, float b, float c, float s) {
  return make_float2(__fmaf_rn(a, c, -__fmul_rn(b, s)), __fmaf_rn(a, s, __fmul_rn(b, c)));
}

// Monotonic key for argmax: larger value wins, equal values -> lower index.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ int argmax_key_index(unsigned long long k) {
  return (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
}

// Six-bit code -> float (q - 32) without an int->float conversion: byte k of
// `packed` becomes the low mantissa byte of 2^23, then 2^23 + 32 is removed.
__device__ __forceinline__ float q6_val(uint32_t packed, int k) {
  return __uint_as_float(__byte_perm(packed, 0x4B000000u, 0x7650u | (uint32_t)k)) - 8388640.0f;
}

// One element of a packed Q6_K row (device layout of hakm_internal.h).
__device__ __forceinline__ float q6k_dequant_packed(const uint8_t* row, int nb, int e) {
  const int b = e / QK, i = e % QK;
  const int c = b >> 3, j = b & 7, m = q6_chunk_blocks(nb, c);
  const uint8_t* chunk = row + (size_t)c * Q6K_CHUNK;
  const uint8_t* body = chunk + j * Q6K_BODY;
  const uint16_t dh = (uint16_t)(chunk[m * Q6K_BODY + 2 * j] | (chunk[m * Q6K_BODY + 2 * j + 1] << 8));
  const float d = __half2float(__ushort_as_half(dh));
  const int nh = i >> 7, k = (i >> 5) & 3, l = i & 31;
  // verbatim ql[64nh + 32(k&1) + l] and qh[32nh + l], at their device places
  const int lb = body[q6k_body_pos(64 * nh + 32 * (k & 1) + l)];
  const int nib = k < 2 ? (lb & 15) : (lb >> 4);
  const int hb = (body[q6k_body_pos(128 + 32 * nh + l)] >> (2 * k)) & 3;
  const int q = (nib | (hb << 4)) - 32;
  // d * sc * q is exact in fp32 (src/quant.c:104-107)
  return __fmul_rn(__fmul_rn(d, (float)(int8_t)body[192 + (i >> 4)]), (float)q);
}

}  // namespace hakm
