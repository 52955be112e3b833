// hakm_rows.cu — the row-batched kernels of prompt processing and batched
// decode (many activation rows through one weight read) with the reference
// build's roundings, so every row equals the reference's hakm_forward for
// that position bit for bit:
//   rx_norm_quant  rmsnorm of each row (src/nn.c:13-18 as built: 8-lane sum
//                  of squares and fold, IEEE divide, rsqrtss + Newton,
//                  (x*w)*scale) and its q8_32 codes (src/quant.c:127-144);
//   rx_q6k_gemm    Q6_K rows x fp32 activation rows (src/nn.c:84-95 as
//                  built): out[m][n] is the fold of 8 lane chains, chain l
//                  adding the rounded products w[n][8t+l] * x[m][8t+l] in
//                  increasing t;
//   rx_swiglu      silu(g) * u with glibc's scalar expf (src/model.c:154);
//   rx_attention   GQA attention of each row over its own positions
//                  (src/model.c:124-142): the scores, softmax and V chains of
//                  the decode attention (hakm_attn.cuh), one CTA per (row,
//                  query head) with the head's dimension slices run by
//                  separate warps.
#include <algorithm>
#include <atomic>

#include "hakm_attn.cuh"
#include "hakm_exact.cuh"

namespace hakm {

// ------------------------------------------------------------------ rmsnorm

// One CTA (256 threads) per row. xn: the normed row (may be null); xq / xs:
// its q8_32 codes and scales (may be null). D a multiple of 256.
__global__ void __launch_bounds__(256) rx_norm_quant_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                            int D, float eps, const uint32_t* __restrict__ rsq,
                                                            float* __restrict__ xn, int8_t* __restrict__ xq,
                                                            float* __restrict__ xs) {
  __shared__ float xr[8192];
  __shared__ float s_scale;
  const size_t r = blockIdx.x;
  const float* src = x + r * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) xr[i] = src[i];
  __syncthreads();
  if (threadIdx.x < 32) {
    const int l = threadIdx.x & 7;
    float acc = 0.f;
    if (threadIdx.x < 8)
      for (int i = l; i < D; i += 8) acc = __fadd_rn(acc, __fmul_rn(xr[i], xr[i]));
    const float ss = fold8_lanes(acc);
    if (threadIdx.x == 0) s_scale = rsqrt_nr(__fadd_rn(__fdiv_rn(ss, (float)D), eps), rsq);
  }
  __syncthreads();
  const float scale = s_scale;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int g = warp; g < D / 32; g += nw) {
    const int i = 32 * g + lane;
    const float y = __fmul_rn(__fmul_rn(xr[i], w[i]), scale);
    if (xn) xn[r * D + i] = y;
    if (xq) {
      const float amax = warp_max(fmaxf(0.0f, fabsf(y)));
      const float sc = __fmul_rn(amax, 1.0f / 127.0f);
      xq[r * D + i] = (int8_t)q8_round(__fmul_rn(y, q8_inv(amax, sc)));
      if (lane == 0) xs[r * (D / 32) + g] = sc;
    }
  }
}

cudaError_t launch_rx_norm_quant(const float* x, const float* w, int M, int D, float eps, const uint32_t* rsq,
                                 float* xn, int8_t* xq, float* xs, cudaStream_t s) {
  if (D % 256 || D > 8192 || !rsq) return cudaErrorInvalidValue;
  rx_norm_quant_kernel<<<M, 256, 0, s>>>(x, w, D, eps, rsq, xn, xq, xs);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ Q6_K x fp32 rows

// CTA tile: 32 weight rows x 32 activation rows, K by super-block (256 = 8
// classes x 32 positions). Thread (l, mi, ni) = (tid % 8, (tid / 8) / 4,
// (tid / 8) % 4) runs class l's chains of 4 x 8 outputs (activation rows
// 4mi.., weight rows 8ni..). Pipeline per super-block b: the raw bytes of
// block b + 1 (each row's 208-byte body and its chunk's 16 bytes of d) and
// the 32 activation rows' 256 values go to shared memory by cp.async while
// block b is worked; block b's bodies are dequantized from shared memory
// into a float tile by class, [l][t][row] (the class pitch padded by 4
// floats: the 8 classes' float4 reads fall in distinct banks), and the
// activations are read in place, [row][k].
constexpr int RQ_BN = 32, RQ_BM = 32, RQ_TP = 32, RQ_LP = 32 * RQ_TP + 4, RQ_RAW = 224;

struct RqTile {
  float w[8 * RQ_LP];             // dequantized block, by class
  float x[2][RQ_BM][QK];          // activation rows of blocks b, b + 1
  uint8_t raw[2][RQ_BN][RQ_RAW];  // bodies + d of blocks b, b + 1
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(256, 2) rx_q6k_gemm_kernel(float* __restrict__ out, const uint8_t* __restrict__ wt,
                                                            const float* __restrict__ x, const float* __restrict__ bias,
                                                            int n_out, int K, int M, int accumulate) {
  extern __shared__ __align__(16) uint8_t rq_smem[];
  RqTile& S = *reinterpret_cast<RqTile*>(rq_smem);
  const int tid = threadIdx.x, l = tid & 7, sub = tid >> 3, mi = sub >> 2, ni = sub & 3;
  const int n0 = blockIdx.x * RQ_BN, m0 = blockIdx.y * RQ_BM;
  const int nb = K / QK;
  const size_t rowB = dev_row_bytes(W_Q6K, nb);

  // block b's copies: raw bytes (14 x 16 B a row) and activations (64 x 16 B a row)
  auto issue = [&](int b, int buf) {
    const int c = b >> 3, j = b & 7, m = q6_chunk_blocks(nb, c);
    for (int i = tid; i < RQ_BN * 14; i += 256) {
      const int rr = i / 14, k = i % 14;
      const uint8_t* chunk = wt + (size_t)min(n0 + rr, n_out - 1) * rowB + (size_t)c * Q6K_CHUNK;
      const uint8_t* src = k < 13 ? chunk + j * Q6K_BODY + 16 * k : chunk + m * Q6K_BODY;
      cp_async16(&S.raw[buf][rr][16 * k], src);
    }
    for (int i = tid; i < RQ_BM * (QK / 4); i += 256) {
      const int rr = i / (QK / 4), k = i % (QK / 4);
      cp_async16(&S.x[buf][rr][4 * k], x + (size_t)min(m0 + rr, M - 1) * K + (size_t)b * QK + 4 * k);
    }
    cp_async_commit();
  };

  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

  issue(0, 0);
  for (int b = 0; b < nb; b++) {
    const int buf = b & 1;
    cp_async_wait_all();
    __syncthreads();  // block b landed; every thread is done with block b - 1's tiles
    if (b + 1 < nb) issue(b + 1, buf ^ 1);
    // dequantize weight row (tid / 8), class l: 32 exact values (q - 32) * (d * sc)
    {
      const int lr = tid >> 3, j = b & 7;
      const uint8_t* body = S.raw[buf][lr];
      const uint2* wp = reinterpret_cast<const uint2*>(body + 24 * l);
      const uint2 w0 = wp[0], w1 = wp[1], w2 = wp[2];
      const uint4 sc = *reinterpret_cast<const uint4*>(body + 192);
      const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(body + 208 + 2 * j));
      const uint32_t scw[4] = {sc.x, sc.y, sc.z, sc.w};
      float* dst = S.w + l * RQ_LP + lr;
#pragma unroll
      for (int n = 0; n < 2; n++) {
        const uint32_t W0 = n ? w1.y : w0.x, W1 = n ? w2.x : w0.y, WH = n ? w2.y : w1.x;
#pragma unroll
        for (int k = 0; k < 4; k++) {
          uint32_t q;
          if (k == 0) q = (W0 & 0x0F0F0F0Fu) | ((WH << 4) & 0x30303030u);
          else if (k == 1) q = (W1 & 0x0F0F0F0Fu) | ((WH << 2) & 0x30303030u);
          else if (k == 2) q = ((W0 >> 4) & 0x0F0F0F0Fu) | (WH & 0x30303030u);
          else q = ((W1 >> 4) & 0x0F0F0F0Fu) | ((WH >> 2) & 0x30303030u);
          const uint32_t sw = scw[2 * n + (k >> 1)];
          const float g0 = __fmul_rn((float)(int8_t)(sw >> (16 * (k & 1))), d);
          const float g1 = __fmul_rn((float)(int8_t)(sw >> (16 * (k & 1) + 8)), d);
#pragma unroll
          for (int bb = 0; bb < 4; bb++) {
            const float qv = (float)(int)((q >> (8 * bb)) & 63u) - 32.0f;
            dst[(16 * n + 4 * k + bb) * RQ_TP] = __fmul_rn(qv, bb < 2 ? g0 : g1);
          }
        }
      }
    }
    __syncthreads();
    const float* wl = S.w + l * RQ_LP + 8 * ni;
    const float* xl = &S.x[buf][4 * mi][l];
#pragma unroll 4
    for (int t = 0; t < 32; t++) {
      const float4 wa = *reinterpret_cast<const float4*>(wl + t * RQ_TP);
      const float4 wb = *reinterpret_cast<const float4*>(wl + t * RQ_TP + 4);
      const float2 wp[4] = {make_float2(wa.x, wa.y), make_float2(wa.z, wa.w), make_float2(wb.x, wb.y),
                            make_float2(wb.z, wb.w)};
      // packed products, scalar sums (a packed add after a packed multiply
      // may be contracted into a packed FMA)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float xv = xl[i * QK + 8 * t];
        const float2 xx = make_float2(xv, xv);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float2 p = mul2(xx, wp[j]);
          acc[i][2 * j] = __fadd_rn(acc[i][2 * j], p.x);
          acc[i][2 * j + 1] = __fadd_rn(acc[i][2 * j + 1], p.y);
        }
      }
    }
  }
  // fold the 8 classes (lanes 8s .. 8s+7 of a warp hold one subtile), then
  // lane l writes the subtile's outputs 4l .. 4l+3 (row i = l / 2)
  float res[4][8];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) res[i][j] = fold8_lanes(acc[i][j]);
  const int m = m0 + 4 * mi + (l >> 1);
  if (m < M) {
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int n = n0 + 8 * ni + 4 * (l & 1) + e;
      float v = 0.f;
#pragma unroll
      for (int i = 0; i < 4; i++)
        if ((l >> 1) == i) v = (l & 1) ? res[i][4 + e] : res[i][e];
      if (n >= n_out) continue;
      if (bias) v = __fadd_rn(v, bias[n]);
      float* o = out + (size_t)m * n_out + n;
      *o = accumulate ? __fadd_rn(*o, v) : v;
    }
  }
}

cudaError_t launch_rx_q6k_gemm(float* out, const uint8_t* w, const float* x, const float* bias, int n_out, int K,
                               int M, bool accumulate, cudaStream_t s) {
  if (K % QK || n_out <= 0 || M <= 0) return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> ready{0};  // devices with the shared-memory limit raised
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(ready.load() & bit)) {
    e = cudaFuncSetAttribute(rx_q6k_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(RqTile));
    if (e != cudaSuccess) return e;
    ready.fetch_or(bit);
  }
  const dim3 grid((unsigned)((n_out + RQ_BN - 1) / RQ_BN), (unsigned)((M + RQ_BM - 1) / RQ_BM));
  rx_q6k_gemm_kernel<<<grid, 256, sizeof(RqTile), s>>>(out, w, x, bias, n_out, K, M, accumulate ? 1 : 0);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ attention

// Row r at position pos = row_pos[r] (decode rows: row r's cache starts
// slot_stride floats after row r-1's) or pos0 + r (prompt rows: one cache,
// the chunk's own K/V rows already in it). q, out: [rows][H * HD]. Scores
// live in shared memory: n_max = the largest pos + 1 of the launch.
template <int HD>
__global__ void __launch_bounds__(256) rx_attention_kernel(float* __restrict__ out, const float* __restrict__ q,
                                                           const float* __restrict__ kc, const float* __restrict__ vc,
                                                           int pos0, const int* __restrict__ row_pos,
                                                           size_t slot_stride, int H, int KVH, float scale) {
  extern __shared__ __align__(16) float ra_smem[];
  constexpr int NSL = HD / 32;
  float* qs = ra_smem;      // [HD]
  float* red = qs + HD;     // [64]
  float* sc = red + 64;     // [n]
  const int h = blockIdx.x, r = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x, nw = nthr >> 5;
  const int pos = row_pos ? row_pos[r] : pos0 + r, n = pos + 1;
  const int kvh = h / (H / KVH), kv_dim = KVH * HD, D = H * HD;
  const size_t slot = row_pos ? (size_t)r * slot_stride : 0;
  const float* kb = kc + slot + kvh * HD;
  const float* vb = vc + slot + kvh * HD;
  auto sync = [] { __syncthreads(); };

  for (int i = tid; i < HD; i += nthr) qs[i] = q[(size_t)r * D + h * HD + i];
  sync();
  // scores: lane (p, l) = (lane / 8, lane % 8) runs chain l of position
  // 4 * (iteration) + p; the 8 chains of a position fold over its lanes
  {
    const int l = lane & 7;
    float qv[HD / 8];
#pragma unroll
    for (int j = 0; j < HD / 8; j++) qv[j] = qs[8 * j + l];
    for (int t0 = 4 * warp; t0 < n; t0 += 4 * nw) {
      const int t = t0 + (lane >> 3);
      float acc = 0.f;
      if (t < n) {
        const float* kr = kb + (size_t)t * kv_dim + l;
        float kv[HD / 8];
#pragma unroll
        for (int j = 0; j < HD / 8; j++) kv[j] = kr[8 * j];
#pragma unroll
        for (int j = 0; j < HD / 8; j++) acc = __fadd_rn(acc, __fmul_rn(qv[j], kv[j]));
      }
      const float dot = fold8_lanes(acc);
      if (t < n && l == 0) sc[t] = __fmul_rn(dot, scale);
    }
  }
  sync();
  softmax_exact(sc, n, red, tid, nthr, sync);
  // weighted V: warp w < NSL runs out[32w + lane] = fma(p_t, v_t, out) over
  // t in order, the loads of 8 positions issued ahead of their FMAs
  if (warp < NSL) {
    const float* vp = vb + 32 * warp + lane;
    float acc = 0.f;
    int t = 0;
    for (; t + 8 <= n; t += 8) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = vp[(size_t)(t + i) * kv_dim];
#pragma unroll
      for (int i = 0; i < 8; i++) acc = __fmaf_rn(sc[t + i], v[i], acc);
    }
    for (; t < n; t++) acc = __fmaf_rn(sc[t], vp[(size_t)t * kv_dim], acc);
    out[(size_t)r * D + h * HD + 32 * warp + lane] = acc;
  }
}

size_t rx_attention_smem_bytes(int hd, int n_max) { return (size_t)(hd + 64 + n_max) * 4; }

// The same rows, one CTA per (row, kv head) for all G = H / KVH query heads
// of the group, so each K and V row is read once per row instead of G
// times: thread (position group of 4, class l) loads K[t][8j + l] once and
// runs the G heads' class-l chains on it; in the V pass thread (head group,
// dimension d) loads V[t][d] once and runs the fma chains of the heads of
// its group. Per-head arithmetic as rx_attention_kernel. Scores for all G
// heads live in shared memory (G * n_stride floats).
constexpr int RA_GMAX = 8, RA_THREADS = 512;

__host__ __device__ inline size_t rx_attention_gqa_smem_bytes(int hd, int g, int n_stride) {
  return ((size_t)g * 8 * (hd / 8 + 4) + 64 + (size_t)g * n_stride) * 4;
}

template <int HD>
__global__ void __launch_bounds__(RA_THREADS, 1)
    rx_attention_gqa_kernel(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ kc,
                            const float* __restrict__ vc, int pos0, const int* __restrict__ row_pos,
                            size_t slot_stride, int H, int KVH, float scale, int n_stride) {
  extern __shared__ __align__(16) float rg_smem[];
  constexpr int QP = HD / 8 + 4;  // a class's 16 (or 8) q values, padded: conflict-free float4 reads
  const int G = H / KVH;
  float* qt = rg_smem;                // [G][8][QP]
  float* red = qt + G * 8 * QP;       // [64]
  float* sc = red + 64;               // [G][n_stride]
  const int kvh = blockIdx.x, r = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x, nw = nthr >> 5;
  const int pos = row_pos ? row_pos[r] : pos0 + r, n = pos + 1;
  const int kv_dim = KVH * HD, D = H * HD;
  const size_t slot = row_pos ? (size_t)r * slot_stride : 0;
  const float* kb = kc + slot + kvh * HD;
  const float* vb = vc + slot + kvh * HD;
  const float* qg = q + (size_t)r * D + (size_t)kvh * G * HD;
  auto sync = [] { __syncthreads(); };

  for (int i = tid; i < G * HD; i += nthr) {
    const int g = i / HD, e = i % HD;
    qt[(g * 8 + (e & 7)) * QP + (e >> 3)] = qg[i];
  }
  sync();
  // scores: lane (p, l) = (lane / 8, lane % 8) runs chain l of position
  // 4 * (iteration) + p for every head of the group; the K values of the
  // next two iterations load while this one's are used
  {
    const int l = lane & 7, step = 4 * nw;
    float kn[2][HD / 8];
    auto load_k = [&](int t0, float (&dst)[HD / 8]) {
      const int t = t0 + (lane >> 3);
      const float* kr = kb + (size_t)(t < n ? t : 0) * kv_dim + l;
#pragma unroll
      for (int j = 0; j < HD / 8; j++) dst[j] = kr[8 * j];
    };
    auto score = [&](int t0, const float (&kv)[HD / 8]) {
      const int t = t0 + (lane >> 3);
      for (int g = 0; g < G; g++) {
        const float4* q4 = reinterpret_cast<const float4*>(qt + (g * 8 + l) * QP);
        float acc = 0.f;
#pragma unroll
        for (int j4 = 0; j4 < HD / 32; j4++) {
          const float4 qv = q4[j4];
          acc = __fadd_rn(acc, __fmul_rn(qv.x, kv[4 * j4]));
          acc = __fadd_rn(acc, __fmul_rn(qv.y, kv[4 * j4 + 1]));
          acc = __fadd_rn(acc, __fmul_rn(qv.z, kv[4 * j4 + 2]));
          acc = __fadd_rn(acc, __fmul_rn(qv.w, kv[4 * j4 + 3]));
        }
        const float dot = fold8_lanes(acc);
        if (t < n && l == 0) sc[(size_t)g * n_stride + t] = __fmul_rn(dot, scale);
      }
    };
    const int t_first = 4 * warp;
    if (t_first < n) load_k(t_first, kn[0]);
    if (t_first + step < n) load_k(t_first + step, kn[1]);
    for (int t0 = t_first; t0 < n; t0 += 2 * step) {
      {
        float kv[HD / 8];
#pragma unroll
        for (int j = 0; j < HD / 8; j++) kv[j] = kn[0][j];
        if (t0 + 2 * step < n) load_k(t0 + 2 * step, kn[0]);
        score(t0, kv);
      }
      if (t0 + step < n) {
        float kv[HD / 8];
#pragma unroll
        for (int j = 0; j < HD / 8; j++) kv[j] = kn[1][j];
        if (t0 + 3 * step < n) load_k(t0 + 3 * step, kn[1]);
        score(t0 + step, kv);
      }
    }
  }
  sync();
  for (int g = 0; g < G; g++) softmax_exact(sc + (size_t)g * n_stride, n, red, tid, nthr, sync);
  // weighted V: thread (head group hg, dimension d) runs the chains of heads
  // hg, hg + NHG, ... on each V[t][d] it loads
  {
    constexpr int NHG = RA_THREADS / HD;  // head groups
    constexpr int GPT = (RA_GMAX + NHG - 1) / NHG;  // heads per thread at most
    const int d = tid % HD, hg = tid / HD;
    const float* vp = vb + d;
    float acc[GPT];
#pragma unroll
    for (int i = 0; i < GPT; i++) acc[i] = 0.f;
    auto chains = [&](int t, const float (&v)[8]) {
#pragma unroll
      for (int i = 0; i < GPT; i++) {
        const int g = hg + NHG * i;
        if (g < G) {
          const float4* p4 = reinterpret_cast<const float4*>(sc + (size_t)g * n_stride + t);
          const float4 pa = p4[0], pb = p4[1];
          const float pv[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
          for (int k = 0; k < 8; k++) acc[i] = __fmaf_rn(pv[k], v[k], acc[i]);
        }
      }
    };
    // groups of 8 positions; the loads run 4 groups (32 positions) ahead
    const int n8 = n & ~7;
    float vr[4][8];
#pragma unroll
    for (int bi = 0; bi < 4; bi++)
      if (8 * bi < n8) {
#pragma unroll
        for (int k = 0; k < 8; k++) vr[bi][k] = vp[(size_t)(8 * bi + k) * kv_dim];
      }
    int t = 0;
    for (; t < n8; t += 32) {
#pragma unroll
      for (int bi = 0; bi < 4; bi++) {
        const int tb = t + 8 * bi;
        if (tb < n8) {
          float v[8];
#pragma unroll
          for (int k = 0; k < 8; k++) v[k] = vr[bi][k];
          if (tb + 32 < n8) {
#pragma unroll
            for (int k = 0; k < 8; k++) vr[bi][k] = vp[(size_t)(tb + 32 + k) * kv_dim];
          }
          chains(tb, v);
        }
      }
    }
    for (t = n8; t < n; t++) {
      const float v = vp[(size_t)t * kv_dim];
#pragma unroll
      for (int i = 0; i < GPT; i++) {
        const int g = hg + NHG * i;
        if (g < G) acc[i] = __fmaf_rn(sc[(size_t)g * n_stride + t], v, acc[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < GPT; i++) {
      const int g = hg + NHG * i;
      if (g < G) out[(size_t)r * D + (size_t)(kvh * G + g) * HD + d] = acc[i];
    }
  }
}



template <int HD>
static cudaError_t launch_rx_attention_hd(float* out, const float* q, const float* kc, const float* vc, int rows,
                                          int pos0, const int* row_pos, int n_max, size_t slot_stride, int H, int KVH,
                                          float scale, cudaStream_t s) {
  static std::atomic<unsigned long long> ready{0};  // devices with the shared-memory limit raised
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(ready.load() & bit)) {
    e = cudaFuncSetAttribute(rx_attention_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)RX_ATTN_SMEM_MAX);
    if (e != cudaSuccess) return e;
    ready.fetch_or(bit);
  }
  const size_t smem = rx_attention_smem_bytes(HD, n_max);
  rx_attention_kernel<HD><<<dim3((unsigned)H, (unsigned)rows), 256, smem, s>>>(out, q, kc, vc, pos0, row_pos,
                                                                             slot_stride, H, KVH, scale);
  return cudaGetLastError();
}

template <int HD>
static cudaError_t launch_rx_attention_gqa_hd(float* out, const float* q, const float* kc, const float* vc, int rows,
                                              int pos0, const int* row_pos, int n_stride, size_t slot_stride, int H,
                                              int KVH, float scale, cudaStream_t s) {
  static std::atomic<unsigned long long> ready{0};  // devices with the shared-memory limit raised
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(ready.load() & bit)) {
    e = cudaFuncSetAttribute(rx_attention_gqa_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)RX_ATTN_SMEM_MAX);
    if (e != cudaSuccess) return e;
    ready.fetch_or(bit);
  }
  const size_t smem = rx_attention_gqa_smem_bytes(HD, H / KVH, n_stride);
  rx_attention_gqa_kernel<HD><<<dim3((unsigned)KVH, (unsigned)rows), RA_THREADS, smem, s>>>(
      out, q, kc, vc, pos0, row_pos, slot_stride, H, KVH, scale, n_stride);
  return cudaGetLastError();
}

cudaError_t launch_rx_attention(float* out, const float* q, const float* kc, const float* vc, int rows, int pos0,
                                const int* row_pos, int n_max, size_t slot_stride, int H, int KVH, int hd,
                                float scale, cudaStream_t s) {
  if (rows <= 0 || n_max <= 0 || KVH <= 0 || H % KVH || rx_attention_smem_bytes(hd, n_max) > RX_ATTN_SMEM_MAX)
    return cudaErrorInvalidValue;
  // the kv head's query heads in one CTA when their score rows fit (n_max
  // rounded to 4 floats keeps the float4 reads of the V pass aligned)
  const int G = H / KVH, n_stride = (n_max + 3) & ~3;
  if (G <= RA_GMAX && rx_attention_gqa_smem_bytes(hd, G, n_stride) <= RX_ATTN_SMEM_MAX) {
    if (hd == 128)
      return launch_rx_attention_gqa_hd<128>(out, q, kc, vc, rows, pos0, row_pos, n_stride, slot_stride, H, KVH,
                                             scale, s);
    if (hd == 64)
      return launch_rx_attention_gqa_hd<64>(out, q, kc, vc, rows, pos0, row_pos, n_stride, slot_stride, H, KVH,
                                            scale, s);
  }
  if (hd == 128)
    return launch_rx_attention_hd<128>(out, q, kc, vc, rows, pos0, row_pos, n_max, slot_stride, H, KVH, scale, s);
  if (hd == 64)
    return launch_rx_attention_hd<64>(out, q, kc, vc, rows, pos0, row_pos, n_max, slot_stride, H, KVH, scale, s);
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------ SwiGLU

// gu: [M][2F], gate and up rows interleaved; h[m][i] = silu(gate) * up.
__global__ void rx_swiglu_kernel(float* __restrict__ h, const float* __restrict__ gu, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)blockDim.x * gridDim.x) {
    const float2 a = reinterpret_cast<const float2*>(gu)[i];
    h[i] = swiglu_exact(a.x, a.y);
  }
}

cudaError_t launch_rx_swiglu(float* h, const float* gu, int M, int F, cudaStream_t s) {
  const size_t n = (size_t)M * F;
  rx_swiglu_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 148 * 16), 256, 0, s>>>(h, gu, n);
  return cudaGetLastError();
}

}  // namespace hakm
