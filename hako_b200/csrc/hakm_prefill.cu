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

#include <algorithm>

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
// k order.
// CTA tile 128 weight rows x BM activation rows (128, 64, or 16 for short
// batches), k tiles of 32 (two 16-element scale groups); thread tile 8 weight
// rows x BM/16 activation rows, read as float4 pairs 64 apart (conflict-free
// shared loads). Double-buffered: the next k tile's raw weight bytes are
// loaded into registers and its activations copied asynchronously into a
// staging tile while the current one is multiplied, then both go
// (dequantized, transposed) into the other buffer; one barrier per tile.
constexpr int G6_BN = 128, G6_BK = 32;

template <int BM>
struct G6Tile {
  float w[2][G6_BK][G6_BN];
  float x[2][G6_BK][BM + 4];
  float xs[BM][G6_BK + 4];  // the next activation tile as copied, [row][k]
};

// Asynchronous global -> shared copy of BYTES (8 or 16) bytes.
template <int BYTES>
__device__ __forceinline__ void g6_cp_async(void* dst, const void* src) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  if constexpr (BYTES == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(d), "l"(src), "n"(BYTES) : "memory");
}

template <int BM>
__global__ void __launch_bounds__(256, BM == 128 ? 2 : BM == 64 ? 3 : 4) pf_q6k_gemm_kernel(float* __restrict__ out, const uint8_t* __restrict__ w,
                                                          const float* __restrict__ x, const float* __restrict__ bias,
                                                          int n_out, int K, int M, int accumulate, int kt_per) {
  constexpr int TM = BM / 16;                // activation rows per thread (1, 4 or 8)
  constexpr int XE = BM * G6_BK / 256;       // activation values per thread and tile (16, 8 or 2)
  constexpr int XPR = G6_BK / XE;            // threads per activation row
  constexpr int CB = XE >= 4 ? 16 : 4 * XE;  // bytes per asynchronous copy
  constexpr int NCP = 4 * XE / CB;           // copies per thread and tile
  extern __shared__ __align__(16) float g6_smem[];
  G6Tile<BM>& S = *reinterpret_cast<G6Tile<BM>*>(g6_smem);
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int n0 = blockIdx.x * G6_BN, m0 = blockIdx.y * BM;
  const int nb = K / QK;
  // this CTA's k tiles: [kt0, kt0 + nk) (split over grid z)
  const int kt0 = blockIdx.z * kt_per, nk = min(K / G6_BK - kt0, kt_per);
  const size_t rowB = dev_row_bytes(W_Q6K, nb);
  // dequantization: weight row lr, 16 values at k0 + 16 * hf (one scale group)
  const int lr = tid >> 1, hf = tid & 1;
  const uint8_t* wrow = w + (size_t)min(n0 + lr, n_out - 1) * rowB;
  // activations: row xm, XE values at k0 + xk, copied by cp.async into xs
  // (no registers held across the multiply), then transposed by the same
  // thread (its own copies: no barrier) into x[buf]
  const int xm = tid / XPR, xk = (tid % XPR) * XE;
  const float* xrow = x + (size_t)min(m0 + xm, M - 1) * K;

  uint4 rlo, rhi;
  float rds;
  auto load = [&](int k0) {
    const int kk = k0 + 16 * hf;
    const int b = kk / QK, i0 = kk % QK;
    const int c = b >> 3, j = b & 7, m = q6_chunk_blocks(nb, c);
    const uint8_t* chunk = wrow + (size_t)c * Q6K_CHUNK;
    const uint8_t* body = chunk + j * Q6K_BODY;
    const float d = half_bits_to_float((uint32_t)chunk[m * Q6K_BODY + 2 * j] |
                                       ((uint32_t)chunk[m * Q6K_BODY + 2 * j + 1] << 8));
    rds = __fmul_rn(d, (float)(int8_t)body[192 + (i0 >> 4)]);
    // the group's 16 elements i0 + e are classes e % 8 at positions 2g, 2g+1
    // of their class (device body layout, hakm_internal.h): byte e of rlo /
    // rhi gets element e's ql / qh byte
    const int g = i0 >> 4, nh = g >> 3, qd = (g & 7) >> 1, b0 = 2 * (g & 1);
    uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
#pragma unroll
    for (int l = 0; l < 8; l++) {
      const uint8_t* cb = body + 24 * l + 12 * nh;
      const uint32_t wl = *reinterpret_cast<const uint16_t*>(cb + 4 * (qd & 1) + b0);
      const uint32_t wh = *reinterpret_cast<const uint16_t*>(cb + 8 + b0);
      // element l (byte l) and element l + 8 (byte l + 8)
      lo[l >> 2] |= (wl & 255u) << (8 * (l & 3));
      lo[2 + (l >> 2)] |= (wl >> 8) << (8 * (l & 3));
      hi[l >> 2] |= (wh & 255u) << (8 * (l & 3));
      hi[2 + (l >> 2)] |= (wh >> 8) << (8 * (l & 3));
    }
    rlo = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    rhi = make_uint4(hi[0], hi[1], hi[2], hi[3]);
#pragma unroll
    for (int c = 0; c < NCP; c++) g6_cp_async<CB>(&S.xs[xm][xk + c * CB / 4], xrow + k0 + xk + c * CB / 4);
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  auto store = [&](int buf, int k0) {
    const int qd = (((k0 + 16 * hf) % QK) >> 5) & 3;
    const uint32_t lw[4] = {rlo.x, rlo.y, rlo.z, rlo.w}, hw[4] = {rhi.x, rhi.y, rhi.z, rhi.w};
#pragma unroll
    for (int e = 0; e < 16; e++) {
      const uint32_t lb = (lw[e >> 2] >> (8 * (e & 3))) & 0xFFu, hb = (hw[e >> 2] >> (8 * (e & 3))) & 0xFFu;
      const int nib = qd < 2 ? (int)(lb & 15u) : (int)(lb >> 4);
      const int q = (nib | (int)(((hb >> (2 * qd)) & 3u) << 4)) - 32;
      S.w[buf][16 * hf + e][lr] = __fmul_rn(rds, (float)q);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
    for (int e = 0; e < XE; e++) S.x[buf][xk + e][xm] = S.xs[xm][xk + e];
  };

  float acc[TM][8];
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.f;
  load(kt0 * G6_BK);
  store(0, kt0 * G6_BK);
  __syncthreads();
  for (int t = 0; t < nk; t++) {
    const int buf = t & 1;
    if (t + 1 < nk) load((kt0 + t + 1) * G6_BK);
#pragma unroll 4
    for (int kk = 0; kk < G6_BK; kk++) {
      const float4 w0 = *reinterpret_cast<const float4*>(&S.w[buf][kk][tx * 4]);
      const float4 w1 = *reinterpret_cast<const float4*>(&S.w[buf][kk][64 + tx * 4]);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      float xa[TM];
      if constexpr (TM == 1) xa[0] = S.x[buf][kk][ty];
#pragma unroll
      for (int h = 0; h < TM / 4; h++) {
        const float4 xv = *reinterpret_cast<const float4*>(&S.x[buf][kk][64 * h + ty * 4]);
        xa[4 * h] = xv.x; xa[4 * h + 1] = xv.y; xa[4 * h + 2] = xv.z; xa[4 * h + 3] = xv.w;
      }
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = __fmaf_rn(xa[i], wv[j], acc[i][j]);
    }
    if (t + 1 < nk) store(buf ^ 1, (kt0 + t + 1) * G6_BK);
    __syncthreads();
  }
  // a K split writes its partial sums to out[split][m][n] (added in order by
  // the chunk-sum kernel)
  const bool split = gridDim.z > 1;
  if (split) out += (size_t)blockIdx.z * M * n_out;
#pragma unroll
  for (int i = 0; i < TM; i++) {
    const int m = TM == 1 ? m0 + ty : m0 + 64 * (i >> 2) + ty * 4 + (i & 3);
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int n = n0 + 64 * (j >> 2) + tx * 4 + (j & 3);
      if (n >= n_out) continue;
      float v = acc[i][j];
      float* o = out + (size_t)m * n_out + n;
      if (split) {
        *o = v;
        continue;
      }
      if (bias) v += bias[n];
      *o = accumulate ? *o + v : v;
    }
  }
}

template <int BM>
static cudaError_t launch_g6(dim3 grid, float* out, const uint8_t* w, const float* x, const float* bias, int n_out,
                             int K, int M, bool accumulate, int kt_per, cudaStream_t s) {
  static unsigned done = 0;  // attribute set, per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 32 && !(done & (1u << dev))) {
    e = cudaFuncSetAttribute(pf_q6k_gemm_kernel<BM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(G6Tile<BM>));
    if (e != cudaSuccess) return e;
    done |= 1u << dev;
  }
  pf_q6k_gemm_kernel<BM><<<grid, 256, sizeof(G6Tile<BM>), s>>>(out, w, x, bias, n_out, K, M, accumulate ? 1 : 0,
                                                               kt_per);
  return cudaGetLastError();
}

namespace {

struct G6Plan {
  int bm, tn, tm, split, kt_per;
};

// Tile height and K split: the height that wastes least of the last wave (2
// CTAs of 128, 3 of 64 or 4 of 16 per SM; a 64-row tile does ~15% less work
// per instruction), then the k tiles split over CTAs (at least 8 per CTA)
// until the last wave is nearly full.
G6Plan g6_plan(int n_out, int K, int M, int sms) {
  G6Plan p;
  p.tn = (n_out + G6_BN - 1) / G6_BN;
  const long t128 = (long)p.tn * ((M + 127) / 128), t64 = (long)p.tn * ((M + 63) / 64);
  const double c128 = (double)((t128 + 2L * sms - 1) / (2L * sms)) * 128.0;
  const double c64 = (double)((t64 + 3L * sms - 1) / (3L * sms)) * 64.0 * 1.15;
  p.bm = M <= 16 ? 16 : (M > 64 && c128 <= c64) ? 128 : 64;
  p.tm = (M + p.bm - 1) / p.bm;
  const long tiles = (long)p.tn * p.tm, slots = (p.bm == 128 ? 2L : p.bm == 64 ? 3L : 4L) * sms;
  const int nk = K / G6_BK;
  // the smallest split (at least 8 k tiles per CTA) whose CTAs fill their
  // last wave to 90%; else the best-filling one (a last wave of 224 tiles
  // on 296 slots left a quarter of the SMs idle: measured)
  const int max_split = std::max(1, std::min(nk / 8, 32));
  int split = 1;
  double best = 0.0;
  for (int sp = 1; sp <= max_split; sp++) {
    const long ctas = tiles * sp, waves = (ctas + slots - 1) / slots;
    const double fill = (double)ctas / (double)(waves * slots);
    if (fill > best + 1e-9) { best = fill; split = sp; }
    if (fill >= 0.9) break;
  }
  p.kt_per = (nk + split - 1) / split;
  p.split = (nk + p.kt_per - 1) / p.kt_per;
  return p;
}

int g6_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace

size_t pf_q6k_part_floats(int n_out, int K, int M) {
  const G6Plan p = g6_plan(n_out, K, M, g6_sms());
  return p.split > 1 ? (size_t)p.split * M * n_out : 0;
}

cudaError_t launch_pf_q6k_gemm(float* out, const uint8_t* w, const float* x, const float* bias, int n_out, int K,
                               int M, bool accumulate, float* part, size_t part_floats, float* tmp, cudaStream_t s) {
  if (K % QK || n_out <= 0 || M <= 0) return cudaErrorInvalidValue;
  const int sms = g6_sms();
  G6Plan p = g6_plan(n_out, K, M, sms);
  if (p.split > 1 && (!part || part_floats < (size_t)p.split * M * n_out || (accumulate && !tmp))) {
    p.split = 1;  // no room for the partials: one CTA per tile takes all of K
    p.kt_per = K / G6_BK;
  }
  const dim3 grid((unsigned)p.tn, (unsigned)p.tm, (unsigned)p.split);
  float* dst = p.split > 1 ? part : out;
  cudaError_t e = p.bm == 128  ? launch_g6<128>(grid, dst, w, x, bias, n_out, K, M, accumulate, p.kt_per, s)
                  : p.bm == 64 ? launch_g6<64>(grid, dst, w, x, bias, n_out, K, M, accumulate, p.kt_per, s)
                               : launch_g6<16>(grid, dst, w, x, bias, n_out, K, M, accumulate, p.kt_per, s);
  if (e != cudaSuccess || p.split == 1) return e;
  e = launch_chunk_sum(accumulate ? tmp : out, part, bias, n_out, M, p.split, sms, s);
  if (e != cudaSuccess || !accumulate) return e;
  return launch_pf_add(out, tmp, (size_t)M * n_out, s);
}

// ---------------------------------------------------------------- RoPE + KV
//
// qk: [M][D + KV] q and k rows in the device order of the fused q/k matrix
// (within a head, rows 2i and 2i + 1 are the pair (i, i + hd/2) that NeoX
// RoPE rotates, src/nn.c:32-42), bias already added; v: [M][KV]. Writes q
// (rotated, natural order) to q[M][D] and k, v to the cache rows
// pos0 + r (src/model.c:118-121). With row_pos (batched decode: row r is
// sequence r) the position is row_pos[r] and the cache rows those of slot r,
// slot_stride floats apart.
__global__ void pf_rope_kv_kernel(const float* __restrict__ qk, const float* __restrict__ v, float* __restrict__ q,
                                  float* __restrict__ kc, float* __restrict__ vc, const float* __restrict__ rope_cs,
                                  int pos0, const int* __restrict__ row_pos, size_t slot_stride, int D, int KV,
                                  int hd) {
  const int r = blockIdx.y, half = hd >> 1;
  const int pos = row_pos ? row_pos[r] : pos0 + r;
  if (row_pos) {
    kc += (size_t)r * slot_stride;
    vc += (size_t)r * slot_stride;
  }
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
                              int M, int pos0, const int* row_pos, size_t slot_stride, int D, int KV, int hd,
                              cudaStream_t s) {
  const int n = (D + KV) / 2 + KV;
  pf_rope_kv_kernel<<<dim3((n + 255) / 256, M), 256, 0, s>>>(qk, v, q, kc, vc, rope_cs, pos0, row_pos, slot_stride, D,
                                                             KV, hd);
  return cudaGetLastError();
}

// out[r] = index of the largest of logits[r][0..V) (greedy sample_token,
// src/sample.c:28-32: the first maximum wins). One CTA per row.
__global__ void __launch_bounds__(256) pf_argmax_kernel(int* __restrict__ out, const float* __restrict__ logits, int V) {
  __shared__ unsigned long long best[8];
  const float* row = logits + (size_t)blockIdx.x * V;
  unsigned long long k = 0ull;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const unsigned long long kk = argmax_key(row[i], i);
    k = kk > k ? kk : k;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
    k = other > k ? other : k;
  }
  if ((threadIdx.x & 31) == 0) best[threadIdx.x >> 5] = k;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) k = best[w] > k ? best[w] : k;
    out[blockIdx.x] = argmax_key_index(k);
  }
}

cudaError_t launch_pf_argmax(int* out, const float* logits, int M, int V, cudaStream_t s) {
  pf_argmax_kernel<<<M, 256, 0, s>>>(out, logits, V);
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

// ---------------------------------------------------------------- decode rows
//
// Attention of batched decode rows (one query position per row): row r is
// sequence r at position row_pos[r], its cache slot_stride floats after row
// r - 1's (src/model.c:122-142 per row). Flash-decoding: CTA = (position
// split, kv head, row); the kv head's G <= 8 query heads share every K/V
// tile of 32 positions, which cp.async brings into a double buffer while
// the previous tile is used. All 8 warps work on every tile: for the scores
// warp w sums dimensions [w * HD/8, (w + 1) * HD/8) of every (head,
// position) pair (lane = position), the partial sums meet in shared memory,
// warp v finishes head v's scores and its online softmax, and for the
// weighted sum thread (v, lane) owns head v's dimensions 4 lane..4 lane + 3
// (HD 128; HD 64: two halves of the tile). Each CTA leaves (max, sum,
// unnormalised output) per head; da_merge_kernel combines the splits in
// order.
constexpr int DA_TILE = 32, DA_MAXG = 8;

template <int HD>
struct DaSmem {
  float k[2][DA_TILE][HD + 4];
  float v[2][DA_TILE][HD];
  float q[DA_MAXG][HD];
  float part[8][DA_MAXG][DA_TILE];  // [warp][head][position] partial dots
  float p[DA_MAXG][DA_TILE];        // probabilities of the tile
  float alpha[DA_MAXG];             // rescale of the running output
};

struct DaArgs {
  float* part;  // [rows][H][splits][HD + 2]
  const float* q;
  const float* kc;
  const float* vc;
  const int* row_pos;
  size_t slot_stride;
  int H, KVH, tiles_per_split;
  float scale;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  const int n = valid ? 16 : 0;  // 0: zero-fill, nothing read
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}

template <int HD>
__global__ void __launch_bounds__(256) da_rows_kernel(const DaArgs a) {
  constexpr int DW = HD / 8;   // dimensions per warp in the score pass
  constexpr int NV = HD / 4;   // float4 per K or V row
  constexpr int VW = HD / 32;  // dimensions per lane in the weighted sum
  extern __shared__ __align__(16) float da_raw[];
  DaSmem<HD>& S = *reinterpret_cast<DaSmem<HD>*>(da_raw);
  const int G = a.H / a.KVH, g = blockIdx.y, r = blockIdx.z;
  const int KV = a.KVH * HD;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pos = a.row_pos[r];
  const float* kc = a.kc + (size_t)r * a.slot_stride + g * HD;
  const float* vc = a.vc + (size_t)r * a.slot_stride + g * HD;
  const int t_begin = blockIdx.x * a.tiles_per_split * DA_TILE;
  const int t_end = min(pos + 1, t_begin + a.tiles_per_split * DA_TILE);
  const int n_tiles = t_end > t_begin ? (t_end - t_begin + DA_TILE - 1) / DA_TILE : 0;
  for (int i = tid; i < G * HD; i += 256)
    S.q[i / HD][i % HD] = a.q[(size_t)r * a.H * HD + (size_t)(g * G) * HD + i];
  auto issue = [&](int tile, int buf) {
    const int t0 = t_begin + tile * DA_TILE;
    for (int i = tid; i < DA_TILE * NV; i += 256) {
      const int j = i / NV, c4 = (i % NV) * 4, p = t0 + j;
      const bool ok = p < t_end;
      const size_t off = (size_t)(ok ? p : t_begin) * KV + c4;
      cp_async16(&S.k[buf][j][c4], kc + off, ok);
      cp_async16(&S.v[buf][j][c4], vc + off, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float acc[VW];  // head `warp`, dimensions VW * lane ..
#pragma unroll
  for (int e = 0; e < VW; e++) acc[e] = 0.f;
  float m = -CUDART_INF_F, l = 0.f;  // head `warp`'s running max and sum (warps < G)
  if (n_tiles > 0) issue(0, 0);
  for (int it = 0; it < n_tiles; it++) {
    const int buf = it & 1, t0 = t_begin + it * DA_TILE;
    if (it + 1 < n_tiles) {
      issue(it + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();  // tile `it` in shared memory for every thread (and q, the first time)
    {
      float sacc[DA_MAXG];
#pragma unroll
      for (int v = 0; v < DA_MAXG; v++) sacc[v] = 0.f;
#pragma unroll
      for (int d4 = 0; d4 < DW; d4 += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(&S.k[buf][lane][warp * DW + d4]);
#pragma unroll
        for (int v = 0; v < DA_MAXG; v++) {
          if (v < G) {
            const float4 q4 = *reinterpret_cast<const float4*>(&S.q[v][warp * DW + d4]);
            sacc[v] = __fmaf_rn(q4.x, k4.x, sacc[v]);
            sacc[v] = __fmaf_rn(q4.y, k4.y, sacc[v]);
            sacc[v] = __fmaf_rn(q4.z, k4.z, sacc[v]);
            sacc[v] = __fmaf_rn(q4.w, k4.w, sacc[v]);
          }
        }
      }
#pragma unroll
      for (int v = 0; v < DA_MAXG; v++)
        if (v < G) S.part[warp][v][lane] = sacc[v];
    }
    __syncthreads();
    if (warp < G) {
      float sc = 0.f;
#pragma unroll
      for (int w = 0; w < 8; w++) sc += S.part[w][warp][lane];
      const bool ok = t0 + lane < t_end;
      sc = ok ? sc * a.scale : -CUDART_INF_F;
      const float mnew = fmaxf(m, warp_max(sc));  // the tile holds >= 1 position: finite
      const float al = expf(m - mnew);
      const float p = ok ? expf(sc - mnew) : 0.f;
      l = l * al + warp_sum(p);
      m = mnew;
      S.p[warp][lane] = p;
#pragma unroll
      for (int e = 0; e < VW; e++) acc[e] *= al;
    }
    __syncthreads();
    if (warp < G) {
#pragma unroll 8
      for (int j = 0; j < DA_TILE; j++) {
        const float pj = S.p[warp][j];
        if constexpr (VW == 4) {
          const float4 v4 = *reinterpret_cast<const float4*>(&S.v[buf][j][4 * lane]);
          acc[0] = __fmaf_rn(pj, v4.x, acc[0]); acc[1] = __fmaf_rn(pj, v4.y, acc[1]);
          acc[2] = __fmaf_rn(pj, v4.z, acc[2]); acc[3] = __fmaf_rn(pj, v4.w, acc[3]);
        } else {
          const float2 v2 = *reinterpret_cast<const float2*>(&S.v[buf][j][2 * lane]);
          acc[0] = __fmaf_rn(pj, v2.x, acc[0]); acc[1] = __fmaf_rn(pj, v2.y, acc[1]);
        }
      }
    }
    __syncthreads();  // buffer `buf` is refilled by the next issue
  }
  // partials: [row][head][split][max, sum, out]
  if (warp < G) {
    float* pp = a.part + (((size_t)r * a.H + g * G + warp) * gridDim.x + blockIdx.x) * (HD + 2);
    if (lane == 0) { pp[0] = m; pp[1] = l; }
#pragma unroll
    for (int e = 0; e < VW; e++) pp[2 + VW * lane + e] = acc[e];
  }
}

// out[row][head] from the splits' partials, in split order: one warp per
// (row, head).
template <int HD>
__global__ void __launch_bounds__(256) da_merge_kernel(float* __restrict__ out, const float* __restrict__ part,
                                                       int rows, int H, int n_split) {
  constexpr int VW = HD / 32;
  const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (w >= rows * H) return;
  const float* pp = part + (size_t)w * n_split * (HD + 2);
  float m = -CUDART_INF_F;
  for (int sp = 0; sp < n_split; sp++) m = fmaxf(m, pp[(size_t)sp * (HD + 2)]);
  float l = 0.f, acc[VW];
#pragma unroll
  for (int e = 0; e < VW; e++) acc[e] = 0.f;
  for (int sp = 0; sp < n_split; sp++) {
    const float* ps = pp + (size_t)sp * (HD + 2);
    if (ps[1] == 0.f) continue;  // a split with no position of this row
    const float f = expf(ps[0] - m);
    l = __fmaf_rn(ps[1], f, l);
#pragma unroll
    for (int e = 0; e < VW; e++) acc[e] = __fmaf_rn(ps[2 + VW * lane + e], f, acc[e]);
  }
  float* o = out + (size_t)w * HD;  // rows' outputs are [row][H][HD]
  const float inv = 1.0f / l;
#pragma unroll
  for (int e = 0; e < VW; e++) o[VW * lane + e] = acc[e] * inv;
}

namespace {
// Position splits: about two waves of 2 CTAs per SM.
int da_splits(int rows, int KVH, int max_pos, int sms, int* tiles_per) {
  const int n_tiles = max_pos / DA_TILE + 1;
  int split = (4 * sms + rows * KVH - 1) / (rows * KVH);
  split = std::max(1, std::min(split, n_tiles));
  *tiles_per = (n_tiles + split - 1) / split;
  return (n_tiles + *tiles_per - 1) / *tiles_per;
}

template <int HD>
cudaError_t launch_da_hd(dim3 grid, const DaArgs& a, float* out, int rows, cudaStream_t s) {
  static unsigned done = 0;  // attribute set, per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 32 && !(done & (1u << dev))) {
    e = cudaFuncSetAttribute(da_rows_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(DaSmem<HD>));
    if (e != cudaSuccess) return e;
    done |= 1u << dev;
  }
  da_rows_kernel<HD><<<grid, 256, sizeof(DaSmem<HD>), s>>>(a);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  da_merge_kernel<HD><<<(rows * a.H + 7) / 8, 256, 0, s>>>(out, a.part, rows, a.H, (int)grid.x);
  return cudaGetLastError();
}
}  // namespace

int pf_decode_attention_plan(int rows, int KVH, int max_pos, int sms, int* tiles_per) {
  return da_splits(rows, KVH, max_pos, sms, tiles_per);
}

size_t pf_decode_attention_part_floats(int rows, int H, int KVH, int hd, int max_pos, int sms) {
  int per = 0;
  return (size_t)rows * H * da_splits(rows, KVH, max_pos, sms, &per) * (hd + 2);
}

cudaError_t launch_pf_decode_attention(float* out, const float* q, const float* kc, const float* vc, int rows,
                                       const int* row_pos, int max_pos, size_t slot_stride, int H, int KVH, int hd,
                                       float scale, float* part, size_t part_floats, int sms, cudaStream_t s) {
  if (H % KVH || H / KVH > DA_MAXG || rows <= 0 || !row_pos || !part) return cudaErrorInvalidValue;
  int per = 0;
  const int split = da_splits(rows, KVH, max_pos, sms, &per);
  if (part_floats < (size_t)rows * H * split * (hd + 2)) return cudaErrorInvalidValue;
  const DaArgs a = {part, q, kc, vc, row_pos, slot_stride, H, KVH, per, scale};
  const dim3 grid(split, KVH, rows);
  if (hd == 128) return launch_da_hd<128>(grid, a, out, rows, s);
  if (hd == 64) return launch_da_hd<64>(grid, a, out, rows, s);
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

// Seeded N(0, 1) fp32 values (a measurement workload's synthetic KV cache):
// element i of block y gets a Box-Muller value from two uniforms taken from a
// splitmix64 hash of (seed, y, i). dst + y * ystride, n per block.
__device__ __forceinline__ uint64_t pf_mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void pf_fill_normal_kernel(float* dst, size_t ystride, size_t n, uint64_t seed) {
  float* d = dst + blockIdx.y * ystride;
  const uint64_t base = pf_mix64(seed ^ ((uint64_t)blockIdx.y << 40));
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)blockDim.x * gridDim.x) {
    const uint64_t h = pf_mix64(base + i);
    const float u1 = ((float)(uint32_t)(h >> 40) + 1.0f) * (1.0f / 16777217.0f);  // (0, 1]
    const float u2 = (float)(uint32_t)(h & 0xFFFFFFu) * (1.0f / 16777216.0f);      // [0, 1)
    d[i] = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
  }
}

cudaError_t launch_pf_fill_normal(float* dst, size_t ystride, size_t n, int blocks_y, uint64_t seed, cudaStream_t s) {
  const unsigned gx = (unsigned)std::min<size_t>((n + 255) / 256, 4096);
  pf_fill_normal_kernel<<<dim3(gx, blocks_y), 256, 0, s>>>(dst, ystride, n, seed);
  return cudaGetLastError();
}

}  // namespace hakm
