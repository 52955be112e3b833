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

// CTA tile: 32 weight rows x 32 activation rows, K in steps of one
// super-block (256 = 8 classes x 32 positions). Thread (l, mi, ni) =
// (tid % 8, (tid / 8) / 4, (tid / 8) % 4) runs class l's chains of the 4 x 8
// outputs (rows 4mi.., weight rows 8ni..). Both tiles sit in shared memory
// by class: [l][t][row], the t pitch padded to 36 and the class pitch to
// 36*32 + 4 floats, so the 8 classes' accesses fall in distinct banks.
constexpr int RQ_BN = 32, RQ_BM = 32, RQ_TP = 36, RQ_LP = 32 * RQ_TP + 4;

struct RqTile {
  float w[8 * RQ_LP];
  float x[8 * RQ_LP];
};

__global__ void __launch_bounds__(256, 2) rx_q6k_gemm_kernel(float* __restrict__ out, const uint8_t* __restrict__ wt,
                                                            const float* __restrict__ x, const float* __restrict__ bias,
                                                            int n_out, int K, int M, int accumulate) {
  extern __shared__ __align__(16) float rq_smem[];
  RqTile& S = *reinterpret_cast<RqTile*>(rq_smem);
  const int tid = threadIdx.x, l = tid & 7, sub = tid >> 3, mi = sub >> 2, ni = sub & 3;
  const int n0 = blockIdx.x * RQ_BN, m0 = blockIdx.y * RQ_BM;
  const int nb = K / QK;
  const size_t rowB = dev_row_bytes(W_Q6K, nb);
  // loaders: weight row n0 + (tid / 8), activation row m0 + (tid / 8), class l
  const int lr = tid >> 3;
  const uint8_t* wrow = wt + (size_t)min(n0 + lr, n_out - 1) * rowB;
  const float* xrow = x + (size_t)min(m0 + lr, M - 1) * K;
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

  for (int b = 0; b < nb; b++) {
    // weight row lr, class l of block b: 32 exact values (q - 32) * (d * sc)
    {
      const int c = b >> 3, j = b & 7, m = q6_chunk_blocks(nb, c);
      const uint8_t* chunk = wrow + (size_t)c * Q6K_CHUNK;
      const uint8_t* body = chunk + j * Q6K_BODY;
      const uint2* wp = reinterpret_cast<const uint2*>(body + 24 * l);
      const uint2 w0 = wp[0], w1 = wp[1], w2 = wp[2];
      const uint4 sc = *reinterpret_cast<const uint4*>(body + 192);
      const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(chunk + m * Q6K_BODY + 2 * j));
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
    // activation row lr, class l of block b
    {
      const float* xs = xrow + (size_t)b * QK + l;
      float* dst = S.x + l * RQ_LP + lr;
#pragma unroll 8
      for (int t = 0; t < 32; t++) dst[t * RQ_TP] = __ldg(xs + 8 * t);
    }
    __syncthreads();
    const float* wl = S.w + l * RQ_LP + 8 * ni;
    const float* xl = S.x + l * RQ_LP + 4 * mi;
#pragma unroll 4
    for (int t = 0; t < 32; t++) {
      const float4 xv = *reinterpret_cast<const float4*>(xl + t * RQ_TP);
      const float4 wa = *reinterpret_cast<const float4*>(wl + t * RQ_TP);
      const float4 wb = *reinterpret_cast<const float4*>(wl + t * RQ_TP + 4);
      const float xs4[4] = {xv.x, xv.y, xv.z, xv.w};
      const float2 wp[4] = {make_float2(wa.x, wa.y), make_float2(wa.z, wa.w), make_float2(wb.x, wb.y),
                            make_float2(wb.z, wb.w)};
      // packed products, scalar sums (a packed add after a packed multiply
      // may be contracted into a packed FMA)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float2 xx = make_float2(xs4[i], xs4[i]);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float2 p = mul2(xx, wp[j]);
          acc[i][2 * j] = __fadd_rn(acc[i][2 * j], p.x);
          acc[i][2 * j + 1] = __fadd_rn(acc[i][2 * j + 1], p.y);
        }
      }
    }
    __syncthreads();
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

cudaError_t launch_rx_attention(float* out, const float* q, const float* kc, const float* vc, int rows, int pos0,
                                const int* row_pos, int n_max, size_t slot_stride, int H, int KVH, int hd,
                                float scale, cudaStream_t s) {
  if (rows <= 0 || n_max <= 0 || KVH <= 0 || H % KVH || rx_attention_smem_bytes(hd, n_max) > RX_ATTN_SMEM_MAX)
    return cudaErrorInvalidValue;
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
