// hakm_sample.cu — sampling for temperature > 0 on the device
// (sample_token, src/sample.c:27-58), with the roundings of the reference's
// own build, so the pick and the generator state match it bit for bit.
//
// The reference, as gcc -O3 -ffast-math builds it for x86-64-v3:
//  1. logits[i] /= temp: element 0 by an IEEE division, then 8-wide
//     multiplies by fl(1/temp) for elements 1 .. 8q (q = (n-1)/8), one
//     4-wide step by the rcpps estimate of 1/temp with a Newton step
//     (2r - (temp*r)*r) when at least 4 remain, IEEE divisions for the rest;
//  2. softmax in place (src/nn.c:20-27, the vectorized form of
//     hakm_attn.cuh);
//  3. the candidates sorted by probability, largest first, by glibc's qsort,
//     which for this size is a stable merge sort: equal probabilities keep
//     their index order;
//  4. top-k, then the nucleus: acc += p in sorted order until acc >= top_p;
//  5. cum = the sum of the first m probabilities, vectorized 8 wide over the
//     sorted list (lane j adds entries 8t + j, t < (m-1)/8, then the fold,
//     one 4-lane step when 5..8 remain, scalar adds);
//  6. r = frand * cum (frand: the top 24 bits of the next xorshift64 state
//     over 2^24), then the first sorted entry whose running sum reaches r.
// Here: one CTA takes 1-2 and writes sort keys; one CTA sorts (least
// significant digit first, 4 bits a pass: stable); one warp takes 4-6.
#include "hakm_exact.cuh"

namespace hakm {

constexpr int SMP_THREADS = 1024;

// rcpss: tab[m] = rcpss(1 + m/2048) for the top 11 mantissa bits, the
// exponent scaling the result (measured from the host instruction).
__device__ __forceinline__ float rcp_est(float v, const uint32_t* tab) {
  const uint32_t u = __float_as_uint(v);
  const int e = (int)(u >> 23) - 127;
  return __uint_as_float(__ldg(tab + ((u >> 12) & 2047)) - ((uint32_t)e << 23));
}

__device__ float block_max_1024(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float m = red[0];
  for (int i = 1; i < SMP_THREADS / 32; i++) m = fmaxf(m, red[i]);
  return m;
}

// Steps 1-2 on p[0..n) in place (n >= 9), then the sort keys: key =
// ~bits(p) (probabilities are >= +0, so ascending keys = descending p),
// val = index.
__global__ void __launch_bounds__(SMP_THREADS) smp_softmax_kernel(float* p, int n, float temp,
                                                                 const uint32_t* rcp_tab, uint32_t* key,
                                                                 uint32_t* val) {
  __shared__ float red[32];
  __shared__ float s_inv;
  const int t = threadIdx.x;
  const float inv = __fdiv_rn(1.0f, temp);
  const int q = (n - 1) >> 3, rem = (n - 1) & 7;
  float inv4 = 0.f;
  if (rem >= 4) {
    const float r0 = rcp_est(temp, rcp_tab);
    inv4 = __fsub_rn(__fadd_rn(r0, r0), __fmul_rn(__fmul_rn(temp, r0), r0));
  }
  float mx = -CUDART_INF_F;
  for (int i = t; i < n; i += SMP_THREADS) {
    float v = p[i];
    if (i == 0) v = __fdiv_rn(v, temp);
    else if (i <= 8 * q) v = __fmul_rn(v, inv);
    else if (rem >= 4 && i <= 8 * q + 4) v = __fmul_rn(v, inv4);
    else v = __fdiv_rn(v, temp);
    p[i] = v;
    mx = fmaxf(mx, v);
  }
  mx = block_max_1024(mx, red);
  for (int i = t; i < n; i += SMP_THREADS) p[i] = exp_softmax(__fsub_rn(p[i], mx), i, n);
  __syncthreads();
  if (t < 32) {
    const int lane = t, n8 = n & ~7, r2 = n - n8;
    float c = 0.f;
    if (lane < 8)
      for (int i = lane; i < n8; i += 8) c = __fadd_rn(c, p[i]);
    const float c4 = __fadd_rn(c, __shfl_xor_sync(0xffffffffu, c, 4));
    const float u2 = __fadd_rn(c4, __shfl_xor_sync(0xffffffffu, c4, 2));
    float sum = __fadd_rn(u2, __shfl_xor_sync(0xffffffffu, u2, 1));
    if (r2 >= 4) {
      const float uk = __fadd_rn(p[n8 + (lane & 3)], c4);
      const float a2 = __fadd_rn(uk, __shfl_xor_sync(0xffffffffu, uk, 2));
      sum = __fadd_rn(a2, __shfl_xor_sync(0xffffffffu, a2, 1));
    }
    if (lane == 0) {
      for (int i = r2 >= 4 ? n8 + 4 : n8; i < n; i++) sum = __fadd_rn(sum, p[i]);
      s_inv = __fdiv_rn(1.0f, sum);
    }
  }
  __syncthreads();
  const float pinv = s_inv;
  for (int i = t; i < n; i += SMP_THREADS) {
    const float v = __fmul_rn(p[i], pinv);
    p[i] = v;
    key[i] = ~__float_as_uint(v);
    val[i] = (uint32_t)i;
  }
}

// Stable ascending sort of (key, val) by key: 8 passes of 4-bit digits,
// least significant first, ping-pong between (k0, v0) and (k1, v1); the
// result ends in (k0, v0). Thread t owns the slice [t*S, (t+1)*S) of each
// pass; its digit counts sit in column t of cnt[16][1024], so an exclusive
// scan over (digit, thread) order gives every element its stable place.
__global__ void __launch_bounds__(SMP_THREADS) smp_sort_kernel(uint32_t* k0, uint32_t* v0, uint32_t* k1,
                                                              uint32_t* v1, int n) {
  extern __shared__ uint32_t cnt[];  // [16][SMP_THREADS]
  __shared__ uint32_t wsum[32];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int S = (n + SMP_THREADS - 1) / SMP_THREADS;
  const int lo = min(n, t * S), hi = min(n, lo + S);
  for (int pass = 0; pass < 8; pass++) {
    const int sh = 4 * pass;
    const uint32_t* ki = (pass & 1) ? k1 : k0;
    const uint32_t* vi = (pass & 1) ? v1 : v0;
    uint32_t* ko = (pass & 1) ? k0 : k1;
    uint32_t* vo = (pass & 1) ? v0 : v1;
#pragma unroll
    for (int d = 0; d < 16; d++) cnt[d * SMP_THREADS + t] = 0u;
    for (int i = lo; i < hi; i++) cnt[((ki[i] >> sh) & 15u) * SMP_THREADS + t]++;
    __syncthreads();
    // exclusive scan over the 16384 counters in linear order: thread t
    // scans entries 16t .. 16t+15, then the 1024 partial sums
    uint32_t loc[16], s = 0;
#pragma unroll
    for (int j = 0; j < 16; j++) { loc[j] = s; s += cnt[16 * t + j]; }
    uint32_t x = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
      uint32_t z = wsum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, z, o);
        if (lane >= o) z += y;
      }
      wsum[lane] = z;
    }
    __syncthreads();
    const uint32_t base = x - s + (w ? wsum[w - 1] : 0u);
#pragma unroll
    for (int j = 0; j < 16; j++) cnt[16 * t + j] = base + loc[j];
    __syncthreads();
    for (int i = lo; i < hi; i++) {
      const uint32_t kv = ki[i];
      const uint32_t dst = cnt[((kv >> sh) & 15u) * SMP_THREADS + t]++;
      ko[dst] = kv;
      vo[dst] = vi[i];
    }
    __syncthreads();
  }
}

// Steps 4-6 over the sorted probabilities (p = ~key) and indices; one warp.
// rng[0]: the generator state in, the advanced state out; out[0]: the pick.
__global__ void smp_draw_kernel(const uint32_t* key, const uint32_t* idx, int n, float top_p, int top_k,
                                unsigned long long* rng, int* out) {
  const int lane = threadIdx.x;
  auto P = [&](int i) { return __uint_as_float(~key[i]); };
  const int k = (top_k > 0 && top_k < n) ? top_k : n;
  int m = k;
  if (top_p > 0.0f && top_p < 1.0f) {
    // sequential: every lane runs the same scan (uniform result)
    float acc = 0.0f;
    m = 0;
    for (int i = 0; i < k; i++) {
      acc = __fadd_rn(acc, P(i));
      m++;
      if (acc >= top_p) break;
    }
  }
  // cum: 8 lanes over the first 8 * ((m-1)/8) entries, fold, then the tail
  float cum = 0.f;
  {
    const int q = m >= 1 ? (m - 1) >> 3 : 0;
    float c = 0.f;
    if (lane < 8)
      for (int t = 0; t < q; t++) c = __fadd_rn(c, P(8 * t + lane));
    const float c4 = __fadd_rn(c, __shfl_xor_sync(0xffffffffu, c, 4));
    const float u2 = __fadd_rn(c4, __shfl_xor_sync(0xffffffffu, c4, 2));
    cum = __fadd_rn(u2, __shfl_xor_sync(0xffffffffu, u2, 1));
    int i = 8 * q;
    if (m - 1 - 8 * q >= 4) {
      const float uk = __fadd_rn(P(8 * q + (lane & 3)), c4);
      const float a2 = __fadd_rn(uk, __shfl_xor_sync(0xffffffffu, uk, 2));
      cum = __fadd_rn(a2, __shfl_xor_sync(0xffffffffu, a2, 1));
      i += 4;
    }
    for (; i < m; i++) cum = __fadd_rn(cum, P(i));
  }
  if (lane != 0) return;
  unsigned long long x = *rng;
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  *rng = x;
  const float fr = __double2float_rn(__dmul_rn((double)(long long)(x >> 40), 0x1p-24));
  const float r = __fmul_rn(fr, cum);
  float run = 0.0f;
  int chosen = (int)idx[0];
  for (int i = 0; i < m; i++) {
    run = __fadd_rn(run, P(i));
    if (run >= r) { chosen = (int)idx[i]; break; }
  }
  *out = chosen;
}

size_t sample_scratch_words(int n) { return (size_t)4 * n; }

cudaError_t launch_sample(float* logits, int n, float temp, float top_p, int top_k, const uint32_t* rcp_tab,
                          uint32_t* scratch, unsigned long long* rng_dev, int* out_dev, cudaStream_t s) {
  if (n < 9 || !(temp > 0.0f)) return cudaErrorInvalidValue;
  static unsigned done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t sort_smem = (size_t)16 * SMP_THREADS * 4;
  if (dev < 32 && !(done & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(smp_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sort_smem);
    if (e != cudaSuccess) return e;
    done |= 1u << dev;
  }
  uint32_t *k0 = scratch, *v0 = scratch + n, *k1 = scratch + 2 * (size_t)n, *v1 = scratch + 3 * (size_t)n;
  smp_softmax_kernel<<<1, SMP_THREADS, 0, s>>>(logits, n, temp, rcp_tab, k0, v0);
  smp_sort_kernel<<<1, SMP_THREADS, sort_smem, s>>>(k0, v0, k1, v1, n);
  smp_draw_kernel<<<1, 32, 0, s>>>(k0, v0, n, top_p, top_k, rng_dev, out_dev);
  return cudaGetLastError();
}

}  // namespace hakm
