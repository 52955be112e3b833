// hakm_prefill.cu — prompt processing with the rows of a prompt chunk
// batched through every layer. The reference feeds a prompt one position at
// a time (cli/main.c:56-60, src/hakm_api.c:105-111: hakm_forward per id);
// here M positions go through each matmul together, so every weight byte
// read serves M rows:
//   Q4_K matmuls  on the tensor cores (hakm_mma.cu) over the q8_32 codes of
//                 the rows (quantize_row_q8_32 per row, src/quant.c:127-144);
//   Q6_K matmuls  as fp32 register-tiled products of dequantized weight tiles
//                 with the fp32 rows (the generic path, src/nn.c:84-95);
//   attention     causal GQA over the KV cache (src/model.c:118-142 per row):
//                 row r at position pos0 + r reads cache positions
//                 0..pos0 + r, so the rows' own K/V are written first.
// Each row's arithmetic is the reference's per-position arithmetic; only
// summation orders differ (fp32 rounding, as between any two fp32 orders).
#include "hakm_device.cuh"

namespace hakm {

namespace {

__device__ float pf_block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}

}  // namespace

// x[r][:] = row tokens[r] of the packed Q6_K embedding (deq_row,
// src/nn.c:55-59), bit-exact as q6k_dequant_packed forms the products in the
// reference's order.
__global__ void pf_embed_kernel(float* __restrict__ x, const uint8_t* __restrict__ w, const int* __restrict__ tokens,
                                int D) {
  const int r = blockIdx.y, nb = D / QK;
  const uint8_t* row = w + (size_t)tokens[r] * dev_row_bytes(W_Q6K, nb);
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < D; e += blockDim.x * gridDim.x)
    x[(size_t)r * D + e] = q6k_dequant_packed(row, nb, e);
}

cudaError_t launch_pf_embed(float* x, const uint8_t* w, const int* tokens, int M, int D, cudaStream_t s) {
  pf_embed_kernel<<<dim3((D + 255) / 256, M), 256, 0, s>>>(x, w, tokens, D);
  return cudaGetLastError();
}

// One CTA per row: y = x * (1 / sqrtf(sum(x^2) / n + eps)) * w (rmsnorm,
// src/nn.c:13-18) into xn (may be null), and the q8_32 codes of y
// (quantize_row_q8_32, src/quant.c:127-144) into xq / xs (may be null).
__global__ void __launch_bounds__(256) pf_norm_quant_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                            int D, float eps, float* __restrict__ xn,
                                                            int8_t* __restrict__ xq, float* __restrict__ xs) {
  __shared__ float red[32];
  const size_t r = blockIdx.x;
  const float* xr = x + r * D;
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) ss += xr[i] * xr[i];
  const float tot = pf_block_sum(ss, red);
  const float scale = 1.0f / sqrtf(tot / (float)D + eps);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int g = warp; g < D / 32; g += nw) {
    const int i = 32 * g + lane;
    const float y = xr[i] * scale * w[i];
    if (xn) xn[r * D + i] = y;
    if (xq) {
      const float amax = warp_max(fmaxf(0.0f, fabsf(y)));
      const float sc = amax * (1.0f / 127.0f);
      xq[r * D + i] = (int8_t)q8_round(y * q8_inv(amax, sc));
      if (lane == 0) xs[r * (D / 32) + g] = sc;
    }
  }
}

cudaError_t launch_pf_norm_quant(const float* x, const float* w, int M, int D, float eps, float* xn, int8_t* xq,
                                 float* xs, cudaStream_t s) {
  pf_norm_quant_kernel<<<M, 256, 0, s>>>(x, w, D, eps, xn, xq, xs);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- Q6_K x fp32
//
// out[m][n] = sum_k x[m][k] * w[n][k] (+ bias[n]) (+ out[m][n] when
// accumulating: the residual add of src/model.c:146,156) for packed Q6_K rows
// and fp32 rows x: the dequant-and-dot matmul (src/nn.c:84-95) for M rows at
// once. The dequantized weights (d * sc) * (q - 32) are exact in fp32 (an
// 11-bit d times an 8-bit scale times a 6-bit code), so only the order of
// the k sum differs from the reference's: here one fma chain per output in
// k order. CTA tile 128 weight rows x 64 activation rows, k tiles of 32 (two
// 16-element scale groups); thread tile 8 weight rows x 4 activation rows.
constexpr int G6_BN = 128, G6_BM = 64, G6_BK = 32;

__global__ void __launch_bounds__(256) pf_q6k_gemm_kernel(float* __restrict__ out, const uint8_t* __restrict__ w,
                                                          const float* __restrict__ x, const float* __restrict__ bias,
                                                          int n_out, int K, int M, int accumulate) {
  __shared__ __align__(16) float Ws[G6_BK][G6_BN];
  __shared__ __align__(16) float Xs[G6_BK][G6_BM + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int n0 = blockIdx.x * G6_BN, m0 = blockIdx.y * G6_BM;
  const int nb = K / QK;
  const size_t rowB = dev_row_bytes(W_Q6K, nb);
  // dequantization: weight row lr, 16 values at k0 + 16 * hf (one scale group)
  const int lr = tid >> 1, hf = tid & 1;
  const uint8_t* wrow = w + (size_t)min(n0 + lr, n_out - 1) * rowB;
  // activations: row xm, 8 values at k0 + xk
  const int xm = tid >> 2, xk = (tid & 3) * 8;
  const float* xrow = x + (size_t)min(m0 + xm, M - 1) * K;
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < K; k0 += G6_BK) {
    {
      const int kk = k0 + 16 * hf;
      const int b = kk / QK, i0 = kk % QK;
      const int c = b >> 3, j = b & 7, m = q6_chunk_blocks(nb, c);
      const uint8_t* chunk = wrow + (size_t)c * Q6K_CHUNK;
      const uint8_t* body = chunk + j * Q6K_BODY;
      const float d = half_bits_to_float((uint32_t)chunk[m * Q6K_BODY + 2 * j] |
                                         ((uint32_t)chunk[m * Q6K_BODY + 2 * j + 1] << 8));
      const float ds = __fmul_rn(d, (float)(int8_t)body[192 + (i0 >> 4)]);
      const int nh = i0 >> 7, qd = (i0 >> 5) & 3, l0 = i0 & 31;
      const uint4 lo = *reinterpret_cast<const uint4*>(body + 64 * nh + 32 * (qd & 1) + l0);
      const uint4 hi = *reinterpret_cast<const uint4*>(body + 128 + 32 * nh + l0);
      const uint32_t lw[4] = {lo.x, lo.y, lo.z, lo.w}, hw[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
      for (int e = 0; e < 16; e++) {
        const uint32_t lb = (lw[e >> 2] >> (8 * (e & 3))) & 0xFFu, hb = (hw[e >> 2] >> (8 * (e & 3))) & 0xFFu;
        const int nib = qd < 2 ? (int)(lb & 15u) : (int)(lb >> 4);
        const int q = (nib | (int)(((hb >> (2 * qd)) & 3u) << 4)) - 32;
        Ws[16 * hf + e][lr] = __fmul_rn(ds, (float)q);
      }
    }
    {
      const float4 a = *reinterpret_cast<const float4*>(xrow + k0 + xk);
      const float4 b = *reinterpret_cast<const float4*>(xrow + k0 + xk + 4);
      Xs[xk + 0][xm] = a.x; Xs[xk + 1][xm] = a.y; Xs[xk + 2][xm] = a.z; Xs[xk + 3][xm] = a.w;
      Xs[xk + 4][xm] = b.x; Xs[xk + 5][xm] = b.y; Xs[xk + 6][xm] = b.z; Xs[xk + 7][xm] = b.w;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < G6_BK; kk++) {
      const float4 w0 = *reinterpret_cast<const float4*>(&Ws[kk][tx * 8]);
      const float4 w1 = *reinterpret_cast<const float4*>(&Ws[kk][tx * 8 + 4]);
      const float4 xv = *reinterpret_cast<const float4*>(&Xs[kk][ty * 4]);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = __fmaf_rn(xa[i], wv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int n = n0 + tx * 8 + j;
      if (n >= n_out) continue;
      float v = acc[i][j];
      if (bias) v += bias[n];
      float* o = out + (size_t)m * n_out + n;
      *o = accumulate ? *o + v : v;
    }
  }
}

cudaError_t launch_pf_q6k_gemm(float* out, const uint8_t* w, const float* x, const float* bias, int n_out, int K,
                               int M, bool accumulate, cudaStream_t s) {
  if (K % QK || n_out <= 0 || M <= 0) return cudaErrorInvalidValue;
  const dim3 grid((n_out + G6_BN - 1) / G6_BN, (M + G6_BM - 1) / G6_BM);
  pf_q6k_gemm_kernel<<<grid, 256, 0, s>>>(out, w, x, bias, n_out, K, M, accumulate ? 1 : 0);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- RoPE + KV
//
// qk: [M][D + KV] q and k rows in the device order of the fused q/k matrix
// (within a head, rows 2i and 2i + 1 are the pair (i, i + hd/2) that NeoX
// RoPE rotates, src/nn.c:32-42), bias already added; v: [M][KV]. Writes q
// (rotated, natural order) to q[M][D] and k, v to the cache rows
// pos0 + r (src/model.c:118-121).
__global__ void pf_rope_kv_kernel(const float* __restrict__ qk, const float* __restrict__ v, float* __restrict__ q,
                                  float* __restrict__ kc, float* __restrict__ vc, const float* __restrict__ rope_cs,
                                  int pos0, int D, int KV, int hd) {
  const int r = blockIdx.y, pos = pos0 + r, half = hd >> 1;
  const int n_pairs = (D + KV) >> 1;
  const float* row = qk + (size_t)r * (D + KV);
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < n_pairs + KV; p += blockDim.x * gridDim.x) {
    if (p < n_pairs) {
      const int dr = 2 * p;
      const bool is_k = dr >= D;
      const int lr = is_k ? dr - D : dr;
      const int head = lr / hd, pi = (lr % hd) >> 1;
      const float2 cs = reinterpret_cast<const float2*>(rope_cs)[(size_t)pos * half + pi];
      const float2 rr = rope_rotate(row[dr], row[dr + 1], cs.x, cs.y);
      const int o0 = head * hd + pi, o1 = o0 + half;
      if (is_k) {
        kc[(size_t)pos * KV + o0] = rr.x;
        kc[(size_t)pos * KV + o1] = rr.y;
      } else {
        q[(size_t)r * D + o0] = rr.x;
        q[(size_t)r * D + o1] = rr.y;
      }
    } else {
      const int e = p - n_pairs;
      vc[(size_t)pos * KV + e] = v[(size_t)r * KV + e];
    }
  }
}

cudaError_t launch_pf_rope_kv(const float* qk, const float* v, float* q, float* kc, float* vc, const float* rope_cs,
                              int M, int pos0, int D, int KV, int hd, cudaStream_t s) {
  const int n = (D + KV) / 2 + KV;
  pf_rope_kv_kernel<<<dim3((n + 255) / 256, M), 256, 0, s>>>(qk, v, q, kc, vc, rope_cs, pos0, D, KV, hd);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- attention
//
// Causal GQA attention of M consecutive rows of one sequence (the per-row
// arithmetic of src/model.c:122-142: score = (q . k) * (1 / sqrtf(hd)),
// softmax over positions 0..pos, out = sum p * v), with the softmax taken
// online over tiles of 32 positions. One CTA per (kv head, block of rows):
// the block's query vectors (rows x the kv head's query heads, <= 32) share
// every K/V tile it stages in shared memory. Warp w owns vectors 4w..4w+3;
// in the score pass lane j takes position j of the tile, in the weighted
// sum lane l takes dimensions l, l + 32, ...
constexpr int PA_TILE = 32, PA_VECS = 32;

template <int HD>
__global__ void __launch_bounds__(256) pf_attn_kernel(float* __restrict__ out, const float* __restrict__ q,
                                                      const float* __restrict__ kc, const float* __restrict__ vc,
                                                      int M, int pos0, int H, int KVH, float scale) {
  constexpr int DL = HD / 32;  // dimensions per lane in the weighted sum
  extern __shared__ __align__(16) float pa_smem[];
  float(*Qt)[PA_VECS] = reinterpret_cast<float(*)[PA_VECS]>(pa_smem);                        // [HD][PA_VECS]
  float(*Ks)[HD + 1] = reinterpret_cast<float(*)[HD + 1]>(pa_smem + HD * PA_VECS);            // [PA_TILE][HD + 1]
  float(*Vs)[HD] = reinterpret_cast<float(*)[HD]>(pa_smem + HD * PA_VECS + PA_TILE * (HD + 1));  // [PA_TILE][HD]
  const int G = H / KVH, rows = PA_VECS / G;  // rows per block
  const int n_blocks = (M + rows - 1) / rows;
  const int blk = n_blocks - 1 - (int)blockIdx.x;  // longest blocks first
  const int g = blockIdx.y, r0 = blk * rows, r1 = min(M, r0 + rows);
  const int nv = (r1 - r0) * G;
  const int KV = KVH * HD, D = H * HD;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < PA_VECS * HD; i += blockDim.x) {
    const int v = i / HD, d = i % HD;
    float val = 0.f;
    if (v < nv) val = q[(size_t)(r0 + v / G) * D + (size_t)(g * G + v % G) * HD + d];
    Qt[d][v] = val;
  }
  int vpos[4];
  bool live[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int v = 4 * warp + i;
    live[i] = v < nv;
    vpos[i] = live[i] ? pos0 + r0 + v / G : -1;
  }
  float mx[4], sum[4], acc[4][DL];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    mx[i] = -CUDART_INF_F;
    sum[i] = 0.f;
#pragma unroll
    for (int e = 0; e < DL; e++) acc[i][e] = 0.f;
  }
  const int last = pos0 + r1 - 1;  // the block's last position
  for (int t0 = 0; t0 <= last; t0 += PA_TILE) {
    __syncthreads();  // previous tile consumed (and Qt written, first time)
    for (int i = tid; i < PA_TILE * HD / 4; i += blockDim.x) {
      const int j = i / (HD / 4), d4 = (i % (HD / 4)) * 4;
      const int p = t0 + j;
      float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
      if (p <= last) {
        kv4 = *reinterpret_cast<const float4*>(kc + (size_t)p * KV + g * HD + d4);
        vv4 = *reinterpret_cast<const float4*>(vc + (size_t)p * KV + g * HD + d4);
      }
      Ks[j][d4] = kv4.x; Ks[j][d4 + 1] = kv4.y; Ks[j][d4 + 2] = kv4.z; Ks[j][d4 + 3] = kv4.w;
      *reinterpret_cast<float4*>(&Vs[j][d4]) = vv4;
    }
    __syncthreads();
    if (4 * warp >= nv) continue;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int d = 0; d < HD; d++) {
      const float kd = Ks[lane][d];
      const float4 q4 = *reinterpret_cast<const float4*>(&Qt[d][4 * warp]);
      s[0] = __fmaf_rn(q4.x, kd, s[0]);
      s[1] = __fmaf_rn(q4.y, kd, s[1]);
      s[2] = __fmaf_rn(q4.z, kd, s[2]);
      s[3] = __fmaf_rn(q4.w, kd, s[3]);
    }
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const bool ok = live[i] && t0 + lane <= vpos[i];
      const float sc = ok ? s[i] * scale : -CUDART_INF_F;
      const float tmax = warp_max(sc);
      const float mnew = fmaxf(mx[i], tmax);
      // every live vector sees position 0 in the first tile: mnew is finite
      const float alpha = live[i] ? expf(mx[i] - mnew) : 0.f;
      p[i] = ok ? expf(sc - mnew) : 0.f;
      sum[i] = sum[i] * alpha + warp_sum(p[i]);
      mx[i] = live[i] ? mnew : mx[i];
#pragma unroll
      for (int e = 0; e < DL; e++) acc[i][e] *= alpha;
    }
#pragma unroll 4
    for (int j = 0; j < PA_TILE; j++) {
      float vj[DL];
#pragma unroll
      for (int e = 0; e < DL; e++) vj[e] = Vs[j][lane + 32 * e];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float pj = __shfl_sync(0xffffffffu, p[i], j);
#pragma unroll
        for (int e = 0; e < DL; e++) acc[i][e] = __fmaf_rn(pj, vj[e], acc[i][e]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int v = 4 * warp + i;
    if (v >= nv) continue;
    float* o = out + (size_t)(r0 + v / G) * D + (size_t)(g * G + v % G) * HD;
    const float inv = 1.0f / sum[i];
#pragma unroll
    for (int e = 0; e < DL; e++) o[lane + 32 * e] = acc[i][e] * inv;
  }
}

template <int HD>
static cudaError_t launch_pf_attn_hd(dim3 grid, float* out, const float* q, const float* kc, const float* vc, int M,
                                     int pos0, int H, int KVH, float scale, cudaStream_t s) {
  constexpr size_t smem = (size_t)(HD * PA_VECS + PA_TILE * (HD + 1) + PA_TILE * HD) * 4;
  static unsigned done = 0;  // attribute set, per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 32 && !(done & (1u << dev))) {
    e = cudaFuncSetAttribute(pf_attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    done |= 1u << dev;
  }
  pf_attn_kernel<HD><<<grid, 256, smem, s>>>(out, q, kc, vc, M, pos0, H, KVH, scale);
  return cudaGetLastError();
}

cudaError_t launch_pf_attention(float* out, const float* q, const float* kc, const float* vc, int M, int pos0, int H,
                                int KVH, int hd, float scale, cudaStream_t s) {
  const int G = H / KVH;
  if (H % KVH || G > PA_VECS || M <= 0) return cudaErrorInvalidValue;
  const int rows = PA_VECS / G;
  const dim3 grid((M + rows - 1) / rows, KVH);
  if (hd == 64) return launch_pf_attn_hd<64>(grid, out, q, kc, vc, M, pos0, H, KVH, scale, s);
  if (hd == 128) return launch_pf_attn_hd<128>(grid, out, q, kc, vc, M, pos0, H, KVH, scale, s);
  return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------- FFN, residual
//
// gu: [M][2F], gate and up rows interleaved (device row 2i = gate row i,
// 2i + 1 = up row i); h[m][i] = silu(gate) * up (src/model.c:154 with silu_f,
// src/nn.c:29).
__global__ void pf_swiglu_kernel(float* __restrict__ h, const float* __restrict__ gu, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)blockDim.x * gridDim.x) {
    const float2 a = reinterpret_cast<const float2*>(gu)[i];
    h[i] = a.x / (1.0f + expf(-a.x)) * a.y;
  }
}

cudaError_t launch_pf_swiglu(float* h, const float* gu, int M, int F, cudaStream_t s) {
  const size_t n = (size_t)M * F;
  pf_swiglu_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 148 * 16), 256, 0, s>>>(h, gu, n);
  return cudaGetLastError();
}

// x += o (the residual adds, src/model.c:146,156)
__global__ void pf_add_kernel(float* __restrict__ x, const float* __restrict__ o, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)blockDim.x * gridDim.x)
    x[i] = x[i] + o[i];
}

cudaError_t launch_pf_add(float* x, const float* o, size_t n, cudaStream_t s) {
  pf_add_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 148 * 16), 256, 0, s>>>(x, o, n);
  return cudaGetLastError();
}

}  // namespace hakm
