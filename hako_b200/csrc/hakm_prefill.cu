// hakm_prefill.cu — the small row-wise kernels of the row-batched passes
// (prompt chunks, batched decode; the matmuls, norms, attention and SwiGLU
// are in hakm_mma.cu and hakm_rows.cu): the embedding rows, RoPE with the
// KV cache writes, the greedy pick per row, the residual add, and a seeded
// fill for measurement caches. Each keeps the reference's per-position
// arithmetic: the embedding and the cache writes are exact copies, the
// rotation has the reference's roundings, the add is one IEEE add.
#include "hakm_device.cuh"

#include <algorithm>

namespace hakm {

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
