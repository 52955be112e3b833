// hakm_kernels.cu — sm_100a kernels of the hako decode path.
//
// The decode step is a chain of "phases". Every GEMV phase runs one kernel,
// phase_kernel, over one or more row segments that share the activation:
//
//   prologue  each CTA rebuilds the whole activation in shared memory:
//             fp32 x (optionally rmsnorm'ed, src/nn.c:13-18) and, when a
//             segment holds Q4_K rows, its per-32 int8 quantization
//             (quantize_row_q8_32, src/quant.c:127-144) with the per-block
//             sum of xq that the Q4_K min term needs.
//   body      each warp owns chunks of 4 output rows; lanes split K so every
//             lane keeps its slice of the activation in registers across the
//             4 rows, and weights stream from HBM as 128-bit non-allocating
//             loads. Q4_K: dp4a over 32-element sub-blocks (q4k_vec_dot,
//             src/quant.c:150-232). Q6_K: fp32 dot on the fly (the generic
//             dequant-and-dot path, src/nn.c:84-95) with 6-bit codes turned
//             into floats by exponent-bias construction (no int->float
//             conversion instruction).
//   epilogue bias, residual add, NeoX RoPE + K-cache append, V-cache append,
//             SwiGLU, or logits + greedy argmax — fused per row pair.
//
// The lm_head phase's last CTA also finalises the step (next token, token log,
// position + 1), so a whole decode step replays as one CUDA graph.
#include "hakm_internal.h"

#include <cuda_fp16.h>
#include <math_constants.h>

namespace hakm {

// ------------------------------------------------------------------ helpers

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}
__device__ __forceinline__ uint16_t ld_stream_u16(const uint16_t* p) {
  uint16_t r;
  asm("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
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
// conversion truncated to 32 bits, so NaN / out-of-range (INT64_MIN) give 0.
__device__ __forceinline__ int q8_round(float r) {
  if (!(fabsf(r) < 9223372036854775808.0f)) return 0;
  const long long v = __float2ll_rn(r);
  const int v32 = (int)(unsigned)((unsigned long long)v & 0xFFFFFFFFull);
  return v32 > 127 ? 127 : (v32 < -127 ? -127 : v32);
}

// Per-32 quantization step of quantize_row_q8_32 as built with -ffast-math:
// xs = amax * fl(1/127), inv = 127 / amax (one IEEE division).
__device__ __forceinline__ float q8_inv(float amax, float scale) {
  return scale > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
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

// Block-wide sum over blockDim.x threads (<= 1024). `red` holds 32 floats.
__device__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

// ------------------------------------------------------------ prologue

// Builds the activation in shared memory. Layout (K = n_in):
//   float xf[K] | int8 xq[K] | float xs[K/32] | int xsum[K/32] | float red[32]
__device__ void build_activation(const PhaseParams& p, float* xf, int8_t* xq, float* xs,
                                 int* xsum, float* red) {
  const int K = p.n_in, nsb = K >> 5;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  if (p.act == ACT_Q8) {
    const int4* src = reinterpret_cast<const int4*>(p.xq);
    int4* dst = reinterpret_cast<int4*>(xq);
    for (int i = tid; i < K / 16; i += nt) dst[i] = src[i];
    for (int i = tid; i < nsb; i += nt) xs[i] = p.xs[i];
    __syncthreads();
    for (int b = warp; b < nsb; b += nw) {
      int s = warp_isum((int)xq[32 * b + lane]);
      if (lane == 0) xsum[b] = s;
    }
    __syncthreads();
    return;
  }
  const float4* x4 = reinterpret_cast<const float4*>(p.x);
  float4* xf4 = reinterpret_cast<float4*>(xf);
  float ss = 0.f;
  for (int i = tid; i < K / 4; i += nt) {
    float4 v = x4[i];
    xf4[i] = v;
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  if (p.act == ACT_RMS) {
    float tot = block_sum(ss, red);
    // src/nn.c:16-17: scale = 1/sqrtf(ss/n + eps); y = x * scale * w
    const float scale = 1.0f / sqrtf(tot / (float)K + p.eps);
    const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
    for (int i = tid; i < K / 4; i += nt) {
      float4 v = xf4[i], w = w4[i];
      v.x = v.x * scale * w.x; v.y = v.y * scale * w.y;
      v.z = v.z * scale * w.z; v.w = v.w * scale * w.w;
      xf4[i] = v;
    }
  }
  __syncthreads();
  if (p.need_q8) {
    // src/quant.c:127-144 as built: scale = amax * fl(1/127), inv = 127/amax
    for (int b = warp; b < nsb; b += nw) {
      float v = xf[32 * b + lane];
      float amax = warp_max(fabsf(v));
      float scale = amax * (1.0f / 127.0f);
      float inv = q8_inv(amax, scale);
      int q = q8_round(v * inv);
      xq[32 * b + lane] = (int8_t)q;
      int s = warp_isum(q);
      if (lane == 0) { xs[b] = scale; xsum[b] = s; }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------ Q4_K body

// Partial dots of up to ROWS_PER_CHUNK Q4_K rows. Lane (bl = lane/4, g = lane%4)
// owns qs bytes [32g, 32g+32) of block bl of each 8-block slice: the low
// nibbles are sub-block 2g, the high nibbles sub-block 2g+1 (src/quant.c:
// 239-259). Per sub-block: xs * (d*s*sum(q*xq) - dmin*m*sum(xq)).
__device__ __forceinline__ void q4k_chunk(const uint8_t* __restrict__ w, int row0, int nrows, int nb,
                                          const int8_t* xq, const float* xs, const int* xsum,
                                          float acc[ROWS_PER_CHUNK]) {
  const int lane = threadIdx.x & 31;
  const int bl = lane >> 2, g = lane & 3;
  const size_t row_bytes = (size_t)nb * Q4K_BYTES;
  // sub-block indices j = 2g, 2g+1 inside a block; byte shifts for the
  // 6-bit scale/min unpack (src/quant.c:57-66)
  const int ja = 2 * g, jb = 2 * g + 1;
#pragma unroll
  for (int r = 0; r < ROWS_PER_CHUNK; r++) acc[r] = 0.f;
  for (int s0 = 0; s0 < nb; s0 += 8) {
    const int b = s0 + bl;
    if (b >= nb) continue;
    const int4* xa = reinterpret_cast<const int4*>(xq + 256 * b + 64 * g);
    const int4 xa0 = xa[0], xa1 = xa[1], xb0 = xa[2], xb1 = xa[3];
    const float xsa = xs[8 * b + ja], xsb = xs[8 * b + jb];
    const int sma = xsum[8 * b + ja], smb = xsum[8 * b + jb];
    uint4 hd[ROWS_PER_CHUNK], q0[ROWS_PER_CHUNK], q1[ROWS_PER_CHUNK];
#pragma unroll
    for (int r = 0; r < ROWS_PER_CHUNK; r++) {
      if (r < nrows) {
        const uint8_t* blk = w + (size_t)(row0 + r) * row_bytes + (size_t)b * Q4K_BYTES;
        hd[r] = ld_stream16(blk);
        q0[r] = ld_stream16(blk + 16 + 32 * g);
        q1[r] = ld_stream16(blk + 32 + 32 * g);
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS_PER_CHUNK; r++) {
      if (r < nrows) {
        const uint32_t qw[8] = {q0[r].x, q0[r].y, q0[r].z, q0[r].w, q1[r].x, q1[r].y, q1[r].z, q1[r].w};
        const int xw_a[8] = {xa0.x, xa0.y, xa0.z, xa0.w, xa1.x, xa1.y, xa1.z, xa1.w};
        const int xw_b[8] = {xb0.x, xb0.y, xb0.z, xb0.w, xb1.x, xb1.y, xb1.z, xb1.w};
        int ia = 0, ib = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
          ia = __dp4a((int)(qw[i] & 0x0F0F0F0Fu), xw_a[i], ia);
          ib = __dp4a((int)((qw[i] >> 4) & 0x0F0F0F0Fu), xw_b[i], ib);
        }
        const float d = half_bits_to_float(hd[r].x), dmin = half_bits_to_float(hd[r].x >> 16);
        // scales[0..3] = hd.y, [4..7] = hd.z, [8..11] = hd.w
        int sa, ma, sb, mb;
        {
          const int jj = ja & 3, shf = 8 * jj;
          const uint32_t Y = hd[r].y >> shf, Z = hd[r].z >> shf, W = hd[r].w >> shf;
          if (ja < 4) { sa = Y & 63; ma = Z & 63; }
          else { sa = (W & 15) | ((Y >> 2) & 0x30); ma = ((W >> 4) & 15) | ((Z >> 2) & 0x30); }
        }
        {
          const int jj = jb & 3, shf = 8 * jj;
          const uint32_t Y = hd[r].y >> shf, Z = hd[r].z >> shf, W = hd[r].w >> shf;
          if (jb < 4) { sb = Y & 63; mb = Z & 63; }
          else { sb = (W & 15) | ((Y >> 2) & 0x30); mb = ((W >> 4) & 15) | ((Z >> 2) & 0x30); }
        }
        acc[r] += xsa * (d * (float)sa * (float)ia - dmin * (float)ma * (float)sma);
        acc[r] += xsb * (d * (float)sb * (float)ib - dmin * (float)mb * (float)smb);
      }
    }
  }
}

// ------------------------------------------------------------ Q6_K body

// Six-bit code -> float (q - 32) without an int->float conversion: byte k of
// `packed` becomes the low mantissa byte of 2^23, then 2^23 + 32 is removed.
__device__ __forceinline__ float q6_val(uint32_t packed, int k) {
  return __uint_as_float(__byte_perm(packed, 0x4B000000u, 0x7650u | (uint32_t)k)) - 8388640.0f;
}

// Partial dots of up to ROWS_PER_CHUNK Q6_K rows against fp32 x in smem.
// Packed layout per row: nb bodies of 208 B {ql[128], qh[64], sc[16]} then a
// separate fp16 d plane. Lane (bl = lane/8, n = half, k = quarter) owns
// ql[64n + 16k .. +16]: low nibbles are elements 128n + 16k + i (scale group
// 8n + k), high nibbles elements 128n + 64 + 16k + i (group 8n + 4 + k); the
// two high bits come from qh[32n + 16(k&1) + i] at bit 0/2 (low) and 4/6 (high)
// — the element map of dequant_q6_K (src/quant.c:94-123).
__device__ __forceinline__ void q6k_chunk(const uint8_t* __restrict__ wb, const uint16_t* __restrict__ wd,
                                          int row0, int nrows, int nb, const float* xf,
                                          float acc[ROWS_PER_CHUNK]) {
  const int lane = threadIdx.x & 31;
  const int bl = lane >> 3, n = (lane >> 2) & 1, k = lane & 3;
  const int sh_lo = (k < 2) ? 0 : 2, sh_hi = (k < 2) ? 4 : 6;
  const size_t row_bytes = (size_t)nb * Q6K_BODY;
#pragma unroll
  for (int r = 0; r < ROWS_PER_CHUNK; r++) acc[r] = 0.f;
  for (int s0 = 0; s0 < nb; s0 += 4) {
    const int b = s0 + bl;
    if (b >= nb) continue;
    const float4* xl4 = reinterpret_cast<const float4*>(xf + 256 * b + 128 * n + 16 * k);
    const float4* xh4 = reinterpret_cast<const float4*>(xf + 256 * b + 128 * n + 64 + 16 * k);
    float xl[16], xh[16];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float4 a = xl4[i], c = xh4[i];
      xl[4 * i] = a.x; xl[4 * i + 1] = a.y; xl[4 * i + 2] = a.z; xl[4 * i + 3] = a.w;
      xh[4 * i] = c.x; xh[4 * i + 1] = c.y; xh[4 * i + 2] = c.z; xh[4 * i + 3] = c.w;
    }
    uint4 ql[ROWS_PER_CHUNK], qh[ROWS_PER_CHUNK], sc[ROWS_PER_CHUNK];
    uint16_t dd[ROWS_PER_CHUNK];
#pragma unroll
    for (int r = 0; r < ROWS_PER_CHUNK; r++) {
      if (r < nrows) {
        const uint8_t* body = wb + (size_t)(row0 + r) * row_bytes + (size_t)b * Q6K_BODY;
        ql[r] = ld_stream16(body + 64 * n + 16 * k);
        qh[r] = ld_stream16(body + 128 + 32 * n + 16 * (k & 1));
        sc[r] = ld_stream16(body + 192);
        dd[r] = ld_stream_u16(wd + (size_t)(row0 + r) * nb + b);
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS_PER_CHUNK; r++) {
      if (r < nrows) {
        const uint32_t lw[4] = {ql[r].x, ql[r].y, ql[r].z, ql[r].w};
        const uint32_t hw[4] = {qh[r].x, qh[r].y, qh[r].z, qh[r].w};
        float slo = 0.f, shi = 0.f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint32_t lo = (lw[i] & 0x0F0F0F0Fu) | (((hw[i] >> sh_lo) & 0x03030303u) << 4);
          const uint32_t hi = ((lw[i] >> 4) & 0x0F0F0F0Fu) | (((hw[i] >> sh_hi) & 0x03030303u) << 4);
#pragma unroll
          for (int t = 0; t < 4; t++) {
            slo = fmaf(q6_val(lo, t), xl[4 * i + t], slo);
            shi = fmaf(q6_val(hi, t), xh[4 * i + t], shi);
          }
        }
        // scales: sc[8n + k] is byte k of word 2n; sc[8n + 4 + k] byte k of word 2n+1
        const uint32_t wlo = n ? sc[r].z : sc[r].x, whi = n ? sc[r].w : sc[r].y;
        const float sl = (float)(int8_t)(wlo >> (8 * k)), sh = (float)(int8_t)(whi >> (8 * k));
        const float d = __half2float(__ushort_as_half(dd[r]));
        acc[r] += d * sl * slo + d * sh * shi;
      }
    }
  }
}

// ------------------------------------------------------------ phase kernel

__device__ __forceinline__ Seg pick_seg(const PhaseParams& p, int c, int& si) {
  si = 0;
  if (p.n_seg > 1 && c >= p.seg[1].chunk_begin) si = 1;
  if (p.n_seg > 2 && c >= p.seg[2].chunk_begin) si = 2;
  return si == 0 ? p.seg[0] : (si == 1 ? p.seg[1] : p.seg[2]);
}

// KINDS: bit 0 = Q4_K segments possible, bit 1 = Q6_K segments possible.
template <int KINDS>
__global__ void __launch_bounds__(256, 1) phase_kernel(const __grid_constant__ PhaseParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = p.n_in, nb = K / QK, nsb = K / 32;
  float* xf = reinterpret_cast<float*>(smem);
  int8_t* xq = reinterpret_cast<int8_t*>(xf + K);
  float* xs = reinterpret_cast<float*>(xq + K);
  int* xsum = reinterpret_cast<int*>(xs + nsb);
  float* red = reinterpret_cast<float*>(xsum + nsb);

  pdl_wait();
  build_activation(p, xf, xq, xs, xsum, red);
  pdl_launch_dependents();

  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int gw = blockIdx.x * wpb + (threadIdx.x >> 5);
  const int nwt = gridDim.x * wpb;
  const int pos = p.pos_dev ? *p.pos_dev : 0;
  unsigned long long best = 0ull;

  for (int c = gw; c < p.total_chunks; c += nwt) {
    int si;
    const Seg S = pick_seg(p, c, si);
    const int row0 = (c - S.chunk_begin) * ROWS_PER_CHUNK;
    const int nrows = min(ROWS_PER_CHUNK, S.n_rows - row0);
    float acc[ROWS_PER_CHUNK];
    if constexpr (KINDS == 1) {
      q4k_chunk(S.w, row0, nrows, nb, xq, xs, xsum, acc);
    } else if constexpr (KINDS == 2) {
      q6k_chunk(S.w, S.wd, row0, nrows, nb, xf, acc);
    } else {
      if (S.type == W_Q4K) q4k_chunk(S.w, row0, nrows, nb, xq, xs, xsum, acc);
      else q6k_chunk(S.w, S.wd, row0, nrows, nb, xf, acc);
    }
#pragma unroll
    for (int r = 0; r < ROWS_PER_CHUNK; r++) acc[r] = warp_sum(acc[r]);

    // every lane now holds all ROWS_PER_CHUNK sums
    float mine = acc[0];
#pragma unroll
    for (int r = 1; r < ROWS_PER_CHUNK; r++) if (lane == r) mine = acc[r];
    switch (S.epi) {
      case EPI_STORE:
        if (lane < nrows) S.out[row0 + lane] = S.bias ? mine + S.bias[row0 + lane] : mine;
        break;
      case EPI_RESID:
        if (lane < nrows) S.out[row0 + lane] += mine;
        break;
      case EPI_V_CACHE:
        if (lane < nrows) {
          const float v = S.bias ? mine + S.bias[row0 + lane] : mine;
          S.out[row0 + lane] = v;
          S.cache[(size_t)pos * p.kv_dim + row0 + lane] = v;
        }
        break;
      case EPI_ARGMAX:
        if (lane < nrows) {
          if (S.out) S.out[row0 + lane] = mine;
          const unsigned long long kk = argmax_key(mine, row0 + lane);
          best = kk > best ? kk : best;
        }
        break;
      case EPI_ROPE_QK:
      case EPI_SWIGLU: {
        // lanes 0 and 1 take the row pairs (0,1) and (2,3) of the chunk
        const int j = lane;
        if (j < 2 && 2 * j + 1 < nrows) {
          const float a0 = (j == 0) ? acc[0] : acc[2];
          const float a1 = (j == 0) ? acc[1] : acc[3];
          const int dr = row0 + 2 * j;  // device row of the pair's first element
          if (S.epi == EPI_SWIGLU) {
            // src/model.c:154 with silu_f src/nn.c:29
            const float gv = a0, uv = a1;
            S.out[dr >> 1] = gv / (1.0f + expf(-gv)) * uv;
          } else {
            const float x0 = S.bias ? a0 + S.bias[dr] : a0;
            const float x1 = S.bias ? a1 + S.bias[dr + 1] : a1;
            const bool is_k = dr >= S.split;
            const int lr = is_k ? dr - S.split : dr;  // device row within q or k
            const int hd = p.head_dim, half = hd >> 1;
            const int head = lr / hd, pi = (lr % hd) >> 1;
            const float2 cs = reinterpret_cast<const float2*>(p.rope_cs)[(size_t)pos * half + pi];
            // src/nn.c:38-40
            const float r0 = x0 * cs.x - x1 * cs.y;
            const float r1 = x0 * cs.y + x1 * cs.x;
            const int o0 = head * hd + pi, o1 = o0 + half;
            float* dst = is_k ? S.out2 : S.out;
            dst[o0] = r0;
            dst[o1] = r1;
            if (is_k) {
              S.cache[(size_t)pos * p.kv_dim + o0] = r0;
              S.cache[(size_t)pos * p.kv_dim + o1] = r1;
            }
          }
        }
        break;
      }
    }
  }

  if (p.argmax_key) {
    // warp max of the 64-bit keys, one atomic per warp
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0 && best) atomicMax(p.argmax_key, best);
  }
  if (p.done_counter) {
    __shared__ bool last;
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(p.done_counter, 1u);
      last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
      __threadfence();
      const unsigned long long k = atomicExch(p.argmax_key, 0ull);
      const int tok = argmax_key_index(k);
      if (p.next_token) *p.next_token = tok;
      if (p.token_log && p.step_dev) {
        const int st = *p.step_dev;
        if (st >= 0 && st < p.token_log_cap) p.token_log[st] = tok;
      }
      if (p.step_dev) *p.step_dev += 1;
      if (p.pos_inc) *p.pos_inc += 1;
      *p.done_counter = 0u;
    }
  }
}

size_t phase_smem_bytes(const PhaseParams& p) {
  const size_t K = (size_t)p.n_in;
  return K * 4 + K + (K / 32) * 8 + 32 * 4;
}

static int phase_kinds(const PhaseParams& p) {
  int k = 0;
  for (int i = 0; i < p.n_seg; i++) k |= (p.seg[i].type == W_Q4K) ? 1 : 2;
  return k;
}

constexpr int PHASE_SMEM_MAX = 110 * 1024;

template <int KINDS>
static cudaError_t prepare_kernel(int* ctas_per_sm, size_t smem) {
  // per device: the attribute and the occupancy both depend on the device
  static int done_mask = 0;
  static int occ[64][4];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!(done_mask & (1 << (dev & 31))) || dev >= 32) {
    cudaError_t e = cudaFuncSetAttribute(phase_kernel<KINDS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         PHASE_SMEM_MAX);
    if (e != cudaSuccess) return e;
    done_mask |= 1 << (dev & 31);
    for (int i = 0; i < 4; i++) occ[dev][i] = 0;
  }
  // occupancy bucket by smem size (small / medium / large / max)
  const int bucket = smem <= 16384 ? 0 : smem <= 49152 ? 1 : smem <= 81920 ? 2 : 3;
  if (!occ[dev][bucket]) {
    const size_t probe = bucket == 0 ? 16384 : bucket == 1 ? 49152 : bucket == 2 ? 81920 : PHASE_SMEM_MAX;
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, phase_kernel<KINDS>, 256, probe);
    if (e != cudaSuccess) return e;
    occ[dev][bucket] = n < 1 ? 1 : n;
  }
  *ctas_per_sm = occ[dev][bucket];
  return cudaSuccess;
}

int phase_grid(const PhaseParams& p, int num_sms) {
  int per_sm = 1;
  const size_t smem = phase_smem_bytes(p);
  const int kinds = phase_kinds(p);
  if (kinds == 1) prepare_kernel<1>(&per_sm, smem);
  else if (kinds == 2) prepare_kernel<2>(&per_sm, smem);
  else prepare_kernel<3>(&per_sm, smem);
  int ctas = (p.total_chunks + 7) / 8;
  const int cap = per_sm * num_sms;  // one wave
  return ctas < cap ? (ctas < 1 ? 1 : ctas) : cap;
}

template <int KINDS>
static cudaError_t launch_phase_k(const PhaseParams& p, int grid, cudaStream_t s, bool pdl) {
  const size_t smem = phase_smem_bytes(p);
  int per_sm = 1;
  cudaError_t e = prepare_kernel<KINDS>(&per_sm, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, phase_kernel<KINDS>, p);
}

cudaError_t launch_phase(const PhaseParams& p, int grid, cudaStream_t s, bool pdl) {
  if (phase_smem_bytes(p) > PHASE_SMEM_MAX) return cudaErrorInvalidValue;
  const int kinds = phase_kinds(p);
  if (kinds == 1) return launch_phase_k<1>(p, grid, s, pdl);
  if (kinds == 2) return launch_phase_k<2>(p, grid, s, pdl);
  return launch_phase_k<3>(p, grid, s, pdl);
}

// ------------------------------------------------------------ small kernels

__global__ void quantize_q8_kernel(const float* __restrict__ x, int n, int8_t* __restrict__ xq,
                                   float* __restrict__ xs) {
  const int lane = threadIdx.x & 31;
  const int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (32 * b >= n) return;
  const float v = x[32 * b + lane];
  const float amax = warp_max(fabsf(v));
  const float scale = amax * (1.0f / 127.0f);
  const float inv = q8_inv(amax, scale);
  xq[32 * b + lane] = (int8_t)q8_round(v * inv);
  if (lane == 0) xs[b] = scale;
}

cudaError_t launch_quantize_q8(const float* x, int n, int8_t* xq, float* xs, cudaStream_t s) {
  const int blocks = (n / 32 + 7) / 8;
  quantize_q8_kernel<<<blocks, 256, 0, s>>>(x, n, xq, xs);
  return cudaGetLastError();
}

// One thread per (row, sub-block): exact integer sums of q4k_vec_dot.
__global__ void q4k_subsums_kernel(int32_t* iqx, int32_t* ix, const uint8_t* __restrict__ w,
                                   const int8_t* __restrict__ xq, int n_out, int n_in) {
  const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int nsb = n_in / 32;
  if (t >= (long)n_out * nsb) return;
  const int r = (int)(t / nsb), j = (int)(t % nsb);
  const int b = j / 8, sb = j % 8, g = sb >> 1, hi = sb & 1;
  const uint8_t* qs = w + ((size_t)r * (n_in / QK) + b) * Q4K_BYTES + 16 + 32 * g;
  int a = 0, c = 0;
  for (int l = 0; l < 32; l++) {
    const int q = hi ? (qs[l] >> 4) : (qs[l] & 15);
    const int xv = xq[32 * j + l];
    a += q * xv;
    c += xv;
  }
  iqx[t] = a;
  ix[t] = c;
}

cudaError_t launch_q4k_subsums(int32_t* iqx, int32_t* ix, const uint8_t* w, const int8_t* xq,
                               int n_out, int n_in, cudaStream_t s) {
  const long n = (long)n_out * (n_in / 32);
  q4k_subsums_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(iqx, ix, w, xq, n_out, n_in);
  return cudaGetLastError();
}

// Verbatim 210-byte blocks -> {208-byte bodies per row} + fp16 d plane.
__global__ void q6k_pack_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, long n_blocks) {
  const long b = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= n_blocks) return;
  const uint8_t* s = src + b * Q6K_BYTES;
  uint8_t* d = dst + b * Q6K_BODY;
  for (int i = lane; i < Q6K_BODY; i += 32) d[i] = s[i];
  if (lane == 0) {
    uint8_t* dp = dst + n_blocks * Q6K_BODY + 2 * b;
    dp[0] = s[208];
    dp[1] = s[209];
  }
}

cudaError_t launch_q6k_pack(uint8_t* dst, const uint8_t* src, int n_rows, int n_in, cudaStream_t s) {
  const long nbk = (long)n_rows * (n_in / QK);
  q6k_pack_kernel<<<(unsigned)((nbk + 7) / 8), 256, 0, s>>>(dst, src, nbk);
  return cudaGetLastError();
}

// Element-wise dequant of verbatim blocks (src/quant.c:68-123).
__global__ void dequant_kernel(float* __restrict__ out, const uint8_t* __restrict__ w, int type, long n) {
  const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  const long blk = e / QK;
  const int i = (int)(e % QK);
  if (type == W_Q4K) {
    const uint8_t* b = w + blk * Q4K_BYTES;
    const float d = __half2float(__ushort_as_half((unsigned short)(b[0] | (b[1] << 8))));
    const float dm = __half2float(__ushort_as_half((unsigned short)(b[2] | (b[3] << 8))));
    const int sb = i / 32, l = i % 32, g = sb >> 1;
    const uint8_t* sc = b + 4;
    int s, m;
    if (sb < 4) { s = sc[sb] & 63; m = sc[sb + 4] & 63; }
    else { s = (sc[sb + 4] & 15) | ((sc[sb - 4] >> 6) << 4); m = (sc[sb + 4] >> 4) | ((sc[sb] >> 6) << 4); }
    const int q = (sb & 1) ? (b[16 + 32 * g + l] >> 4) : (b[16 + 32 * g + l] & 15);
    const float d1 = d * (float)s, m1 = dm * (float)m;
    out[e] = __fsub_rn(__fmul_rn(d1, (float)q), m1);
  } else {
    const uint8_t* b = w + blk * Q6K_BYTES;
    const float d = __half2float(__ushort_as_half((unsigned short)(b[208] | (b[209] << 8))));
    const int nh = i >> 7, k = (i >> 5) & 3, l = i & 31;
    const int lb = b[64 * nh + 32 * (k & 1) + l];
    const int nib = k < 2 ? (lb & 15) : (lb >> 4);
    const int hb = (b[128 + 32 * nh + l] >> (2 * k)) & 3;
    const int q = (nib | (hb << 4)) - 32;
    out[e] = __fmul_rn(__fmul_rn(d, (float)(int8_t)b[192 + (i >> 4)]), (float)q);
  }
}

cudaError_t launch_dequant(float* out, const uint8_t* w, int type, int n_rows, int n_in, cudaStream_t s) {
  const long n = (long)n_rows * n_in;
  dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(out, w, type, n);
  return cudaGetLastError();
}

__global__ void rmsnorm_kernel(float* y, const float* x, const float* w, int n, float eps) {
  __shared__ float red[32];
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
  const float tot = block_sum(ss, red);
  const float scale = 1.0f / sqrtf(tot / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = x[i] * scale * w[i];
}

cudaError_t launch_rmsnorm(float* y, const float* x, const float* w, int n, float eps, cudaStream_t s) {
  rmsnorm_kernel<<<1, 1024, 0, s>>>(y, x, w, n, eps);
  return cudaGetLastError();
}

// Embedding lookup of a packed Q6_K row (deq_row, src/nn.c:55-59): the
// products are formed in the reference's order, (d * sc) * (q - 32), so the
// row is bit-exact.
__global__ void embed_q6k_kernel(float* __restrict__ xb, const uint8_t* __restrict__ wb,
                                 const uint16_t* __restrict__ wd, const int* token, int n_in,
                                 unsigned long long* argmax_key) {
  pdl_wait();
  const int nb = n_in / QK;
  const int t = *token;
  for (int e = threadIdx.x + blockIdx.x * blockDim.x; e < n_in; e += blockDim.x * gridDim.x) {
    const int b = e / QK, i = e % QK;
    const uint8_t* body = wb + ((size_t)t * nb + b) * Q6K_BODY;
    const float d = __half2float(__ushort_as_half(wd[(size_t)t * nb + b]));
    const int nh = i >> 7, k = (i >> 5) & 3, l = i & 31;
    const int lb = body[64 * nh + 32 * (k & 1) + l];
    const int nib = k < 2 ? (lb & 15) : (lb >> 4);
    const int hb = (body[128 + 32 * nh + l] >> (2 * k)) & 3;
    const int q = (nib | (hb << 4)) - 32;
    xb[e] = __fmul_rn(__fmul_rn(d, (float)(int8_t)body[192 + (i >> 4)]), (float)q);
  }
  (void)argmax_key;
  pdl_launch_dependents();
}

cudaError_t launch_embed_q6k(float* xb, const uint8_t* wb, const uint16_t* wd, const int* token,
                             int n_in, unsigned long long* argmax_key, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((n_in + 255) / 256);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, embed_q6k_kernel, xb, wb, wd, token, n_in, argmax_key);
}

// NeoX RoPE in place from a (cos, sin) table row (src/nn.c:32-42).
__global__ void rope_kernel(float* x, const float* rope_cs, const int* pos_dev, int n_heads, int hd) {
  const int half = hd / 2;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n_heads * half) return;
  const int h = t / half, i = t % half;
  const int pos = pos_dev ? *pos_dev : 0;
  const float2 cs = reinterpret_cast<const float2*>(rope_cs)[(size_t)pos * half + i];
  const float a = x[h * hd + i], b = x[h * hd + i + half];
  x[h * hd + i] = a * cs.x - b * cs.y;
  x[h * hd + i + half] = a * cs.y + b * cs.x;
}

cudaError_t launch_rope(float* x, const float* rope_cs, const int* pos_dev, int n_heads, int head_dim,
                        cudaStream_t s) {
  const int n = n_heads * head_dim / 2;
  rope_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, rope_cs, pos_dev, n_heads, head_dim);
  return cudaGetLastError();
}

// ------------------------------------------------------------ attention

// GQA decode attention (src/model.c:124-142, softmax src/nn.c:20-27). One CTA
// per (kv head, chunk of ATTN_CHUNK positions) serves the G query heads that
// share the kv head, so K and V stream once. Scores: one thread per position
// (its K row as 128-bit loads, q broadcast from smem). Softmax per head. Out:
// each warp sums a stride of positions for all G heads, then a cross-warp
// reduction. Chunks combine flash-decode style (max / sum rescale); the last
// CTA of a kv head (atomic ticket) merges them, so one launch suffices.
template <int HD>
__global__ void __launch_bounds__(256) attention_kernel(const AttnParams a) {
  extern __shared__ __align__(16) float sm[];
  constexpr int MAXG = 8;
  const int G = a.n_heads / a.n_kv;
  const int kvh = blockIdx.x, split = blockIdx.y;
  const int kv_dim = a.n_kv * HD;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  float* qs = sm;                       // [G][HD]
  float* sc = qs + MAXG * HD;           // [G][ATTN_CHUNK]
  float* red = sc + MAXG * ATTN_CHUNK;  // [nw][G][HD]
  __shared__ float stat_m[MAXG], stat_l[MAXG];
  __shared__ bool last;

  pdl_wait();
  const int pos = *a.pos_dev;
  const int s0 = split * ATTN_CHUNK;
  const int s1 = min(s0 + ATTN_CHUNK, pos + 1);
  const int ns = s1 - s0;  // may be <= 0 for chunks past pos

  for (int i = tid; i < G * HD; i += blockDim.x) qs[i] = a.q[(kvh * G) * HD + i];
  __syncthreads();

  if (tid < ns) {
    const float4* kr = reinterpret_cast<const float4*>(a.k_cache + (size_t)(s0 + tid) * kv_dim + kvh * HD);
    float dot[MAXG];
#pragma unroll
    for (int g = 0; g < MAXG; g++) dot[g] = 0.f;
#pragma unroll 4
    for (int d4 = 0; d4 < HD / 4; d4++) {
      const float4 kv = kr[d4];
#pragma unroll
      for (int g = 0; g < MAXG; g++) {
        if (g < G) {
          const float4 qv = reinterpret_cast<const float4*>(qs + g * HD)[d4];
          dot[g] = fmaf(qv.x, kv.x, dot[g]);
          dot[g] = fmaf(qv.y, kv.y, dot[g]);
          dot[g] = fmaf(qv.z, kv.z, dot[g]);
          dot[g] = fmaf(qv.w, kv.w, dot[g]);
        }
      }
    }
#pragma unroll
    for (int g = 0; g < MAXG; g++)
      if (g < G) sc[g * ATTN_CHUNK + tid] = dot[g] * a.scale;
  }
  __syncthreads();

  // per-head max and exp-sum (warp g handles head g)
  for (int g = warp; g < G; g += nw) {
    float m = -CUDART_INF_F;
    for (int i = lane; i < ns; i += 32) m = fmaxf(m, sc[g * ATTN_CHUNK + i]);
    m = warp_max(m);
    float l = 0.f;
    for (int i = lane; i < ns; i += 32) {
      const float e = expf(sc[g * ATTN_CHUNK + i] - m);
      sc[g * ATTN_CHUNK + i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) { stat_m[g] = m; stat_l[g] = l; }
  }
  __syncthreads();

  // weighted V: lane owns HD/32 consecutive dims
  constexpr int DPL = HD / 32;
  float acc[MAXG][DPL];
#pragma unroll
  for (int g = 0; g < MAXG; g++)
#pragma unroll
    for (int j = 0; j < DPL; j++) acc[g][j] = 0.f;
  for (int i = warp; i < ns; i += nw) {
    const float* vr = a.v_cache + (size_t)(s0 + i) * kv_dim + kvh * HD + lane * DPL;
    float v[DPL];
    if constexpr (DPL == 4) {
      const float4 t = *reinterpret_cast<const float4*>(vr);
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[DPL - 1] = t.w;
    } else {
#pragma unroll
      for (int j = 0; j < DPL; j++) v[j] = vr[j];
    }
#pragma unroll
    for (int g = 0; g < MAXG; g++) {
      if (g < G) {
        const float e = sc[g * ATTN_CHUNK + i];
#pragma unroll
        for (int j = 0; j < DPL; j++) acc[g][j] = fmaf(e, v[j], acc[g][j]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < MAXG; g++)
    if (g < G)
#pragma unroll
      for (int j = 0; j < DPL; j++) red[(warp * MAXG + g) * HD + lane * DPL + j] = acc[g][j];
  __syncthreads();

  const bool single = (a.n_split == 1);
  for (int i = tid; i < G * HD; i += blockDim.x) {
    const int g = i / HD, d = i % HD;
    float s = 0.f;
    for (int w = 0; w < nw; w++) s += red[(w * MAXG + g) * HD + d];
    if (single) {
      a.out[(kvh * G + g) * HD + d] = s / stat_l[g];
    } else {
      float* pp = a.part + ((size_t)(kvh * a.n_split + split) * G + g) * (HD + 2);
      pp[2 + d] = s;
      if (d == 0) { pp[0] = ns > 0 ? stat_m[g] : -CUDART_INF_F; pp[1] = ns > 0 ? stat_l[g] : 0.f; }
    }
  }
  if (!single) {
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(&a.counters[kvh], 1u);
      last = (prev == (unsigned)a.n_split - 1);
    }
    __syncthreads();
    if (last) {
      __threadfence();
      for (int i = tid; i < G * HD; i += blockDim.x) {
        const int g = i / HD, d = i % HD;
        float m = -CUDART_INF_F;
        for (int sp = 0; sp < a.n_split; sp++) {
          const volatile float* pp = a.part + ((size_t)(kvh * a.n_split + sp) * G + g) * (HD + 2);
          m = fmaxf(m, pp[0]);
        }
        float l = 0.f, s = 0.f;
        for (int sp = 0; sp < a.n_split; sp++) {
          const volatile float* pp = a.part + ((size_t)(kvh * a.n_split + sp) * G + g) * (HD + 2);
          if (pp[1] > 0.f) {
            const float f = expf(pp[0] - m);
            l += pp[1] * f;
            s += pp[2 + d] * f;
          }
        }
        a.out[(kvh * G + g) * HD + d] = s / l;
      }
      if (tid == 0) a.counters[kvh] = 0u;
    }
  }
  pdl_launch_dependents();
}

size_t attention_scratch_floats(int n_kv, int n_split, int group, int head_dim) {
  return (size_t)n_kv * n_split * group * (head_dim + 2);
}

cudaError_t launch_attention(const AttnParams& a, cudaStream_t s, bool pdl) {
  constexpr int MAXG = 8;
  if (a.n_heads % a.n_kv || a.n_heads / a.n_kv > MAXG) return cudaErrorInvalidValue;
  const int hd = a.head_dim;
  const size_t smem = (size_t)(MAXG * hd + MAXG * ATTN_CHUNK + 8 * MAXG * hd) * sizeof(float);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_kv, a.n_split);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (hd == 128) {
    static bool done = false;
    if (!done) {
      cudaFuncSetAttribute(attention_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      done = true;
    }
    return cudaLaunchKernelEx(&cfg, attention_kernel<128>, a);
  }
  if (hd == 64) {
    static bool done = false;
    if (!done) {
      cudaFuncSetAttribute(attention_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      done = true;
    }
    return cudaLaunchKernelEx(&cfg, attention_kernel<64>, a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace hakm
