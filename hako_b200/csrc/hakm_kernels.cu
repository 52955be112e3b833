// hakm_kernels.cu — the small kernels of libhakm_cuda: the stand-alone
// activation quantizer, exact Q4_K integer sub-block sums, Q6_K re-layout,
// dequantization, rmsnorm, embedding lookup, NeoX RoPE and GQA decode
// attention. The streaming GEMV phases live in hakm_stream.cu.
#include "hakm_device.cuh"

#include <mutex>

namespace hakm {

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

// Verbatim 210-byte blocks -> the chunked device layout (hakm_internal.h):
// per 8-block chunk the 208-byte bodies, then the 8 fp16 d values. One warp
// per block; the destination is zeroed first so chunk padding is defined.
__global__ void q6k_pack_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, int n_rows, int nb) {
  const long blk = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (blk >= (long)n_rows * nb) return;
  const int r = (int)(blk / nb), b = (int)(blk % nb);
  const int c = b / CHUNK_BLOCKS, j = b % CHUNK_BLOCKS, m = q6_chunk_blocks(nb, c);
  const uint8_t* s = src + blk * Q6K_BYTES;
  uint8_t* chunk = dst + (size_t)r * dev_row_bytes(W_Q6K, nb) + (size_t)c * Q6K_CHUNK;
  for (int i = lane; i < Q6K_BODY; i += 32) chunk[j * Q6K_BODY + i] = s[i];
  if (lane < 2) chunk[m * Q6K_BODY + 2 * j + lane] = s[Q6K_BODY + lane];
}

cudaError_t launch_q6k_pack(uint8_t* dst, const uint8_t* src, int n_rows, int n_in, cudaStream_t s) {
  const int nb = n_in / QK;
  cudaError_t e = cudaMemsetAsync(dst, 0, (size_t)n_rows * dev_row_bytes(W_Q6K, nb), s);
  if (e != cudaSuccess) return e;
  const long nbk = (long)n_rows * nb;
  q6k_pack_kernel<<<(unsigned)((nbk + 7) / 8), 256, 0, s>>>(dst, src, n_rows, nb);
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
__global__ void embed_q6k_kernel(float* __restrict__ xb, const uint8_t* __restrict__ w, const int* token,
                                 int n_in) {
  pdl_launch_dependents();
  pdl_wait();
  const int nb = n_in / QK;
  const uint8_t* row = w + (size_t)(*token) * dev_row_bytes(W_Q6K, nb);
  for (int e = threadIdx.x + blockIdx.x * blockDim.x; e < n_in; e += blockDim.x * gridDim.x)
    xb[e] = q6k_dequant_packed(row, nb, e);
}

cudaError_t launch_embed_q6k(float* xb, const uint8_t* w, const int* token, int n_in, cudaStream_t s,
                             bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((n_in + 255) / 256);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, embed_q6k_kernel, xb, w, token, n_in);
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
// share the kv head. The chunk's K and V rows are staged in shared memory
// with every load in flight at once (rows padded by 4 floats so float4 reads
// down a column of positions are bank-conflict free); scores, softmax and the
// weighted V sum then run out of shared memory. Chunks combine flash-decode
// style (max / sum rescale); the last CTA of a kv head (atomic ticket) merges
// them, so one launch suffices at any context length.
template <int HD>
__global__ void __launch_bounds__(256) attention_kernel(const AttnParams a) {
  extern __shared__ __align__(16) float sm[];
  constexpr int MAXG = 8, KP = HD + 4;
  const int G = a.n_heads / a.n_kv;
  const int kvh = blockIdx.x, split = blockIdx.y;
  const int kv_dim = a.n_kv * HD;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  float* qs = sm;                     // [G][HD]
  float* ks = qs + MAXG * HD;         // [ATTN_CHUNK][KP]
  float* vs = ks + ATTN_CHUNK * KP;   // [ATTN_CHUNK][HD]
  float* sc = vs + ATTN_CHUNK * HD;   // [G][ATTN_CHUNK]
  __shared__ float stat_m[MAXG], stat_l[MAXG];
  __shared__ bool last;

  pdl_launch_dependents();
  pdl_wait();
  const int pos = *a.pos_dev;
  const int s0 = split * ATTN_CHUNK;
  const int ns = min(ATTN_CHUNK, pos + 1 - s0);  // may be <= 0 for chunks past pos

  // stage q, K and V (all loads issued before any use)
  constexpr int R4 = HD / 4;
  const float4* q4 = reinterpret_cast<const float4*>(a.q + (size_t)kvh * G * HD);
  for (int i = tid; i < G * R4; i += blockDim.x) reinterpret_cast<float4*>(qs)[i] = q4[i];
  if (ns > 0) {
    const float* kb = a.k_cache + (size_t)s0 * kv_dim + kvh * HD;
    const float* vb = a.v_cache + (size_t)s0 * kv_dim + kvh * HD;
    for (int i = tid; i < ns * R4; i += blockDim.x) {
      const int r = i / R4, c4 = i % R4;
      const float4 kv = *reinterpret_cast<const float4*>(kb + (size_t)r * kv_dim + 4 * c4);
      const float4 vv = *reinterpret_cast<const float4*>(vb + (size_t)r * kv_dim + 4 * c4);
      *reinterpret_cast<float4*>(ks + r * KP + 4 * c4) = kv;
      *reinterpret_cast<float4*>(vs + r * HD + 4 * c4) = vv;
    }
  }
  __syncthreads();

  // scores: one (head, position) pair per thread iteration, positions fastest
  for (int i = tid; i < G * ATTN_CHUNK; i += blockDim.x) {
    const int g = i / ATTN_CHUNK, r = i % ATTN_CHUNK;
    if (r < ns) {
      const float4* kr = reinterpret_cast<const float4*>(ks + r * KP);
      const float4* qr = reinterpret_cast<const float4*>(qs + g * HD);
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int c4 = 0; c4 < R4; c4 += 2) {
        const float4 k0 = kr[c4], k1 = kr[c4 + 1], x0 = qr[c4], x1 = qr[c4 + 1];
        d0 = fmaf(x0.x, k0.x, d0); d0 = fmaf(x0.y, k0.y, d0); d0 = fmaf(x0.z, k0.z, d0); d0 = fmaf(x0.w, k0.w, d0);
        d1 = fmaf(x1.x, k1.x, d1); d1 = fmaf(x1.y, k1.y, d1); d1 = fmaf(x1.z, k1.z, d1); d1 = fmaf(x1.w, k1.w, d1);
      }
      sc[g * ATTN_CHUNK + r] = (d0 + d1) * a.scale;
    }
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

  // weighted V: one (head, 4 dims) pair per thread iteration
  const bool single = (a.n_split == 1);
  for (int i = tid; i < G * R4; i += blockDim.x) {
    const int g = i / R4, c4 = i % R4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < ns; r++) {
      const float e = sc[g * ATTN_CHUNK + r];
      const float4 v = *reinterpret_cast<const float4*>(vs + r * HD + 4 * c4);
      acc.x = fmaf(e, v.x, acc.x); acc.y = fmaf(e, v.y, acc.y);
      acc.z = fmaf(e, v.z, acc.z); acc.w = fmaf(e, v.w, acc.w);
    }
    if (single) {
      const float inv = 1.0f / stat_l[g];
      float4 o;
      o.x = acc.x * inv; o.y = acc.y * inv; o.z = acc.z * inv; o.w = acc.w * inv;
      *reinterpret_cast<float4*>(a.out + (size_t)(kvh * G + g) * HD + 4 * c4) = o;
    } else {
      float* pp = a.part + ((size_t)(kvh * a.n_split + split) * G + g) * (HD + 2);
      pp[2 + 4 * c4] = acc.x; pp[3 + 4 * c4] = acc.y; pp[4 + 4 * c4] = acc.z; pp[5 + 4 * c4] = acc.w;
      if (c4 == 0) { pp[0] = ns > 0 ? stat_m[g] : -CUDART_INF_F; pp[1] = ns > 0 ? stat_l[g] : 0.f; }
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
        float l = 0.f, acc = 0.f;
        for (int sp = 0; sp < a.n_split; sp++) {
          const volatile float* pp = a.part + ((size_t)(kvh * a.n_split + sp) * G + g) * (HD + 2);
          if (pp[1] > 0.f) {
            const float f = expf(pp[0] - m);
            l += pp[1] * f;
            acc += pp[2 + d] * f;
          }
        }
        a.out[(kvh * G + g) * HD + d] = acc / l;
      }
      if (tid == 0) a.counters[kvh] = 0u;
    }
  }
}

size_t attention_scratch_floats(int n_kv, int n_split, int group, int head_dim) {
  return (size_t)n_kv * n_split * group * (head_dim + 2);
}

template <int HD>
static cudaError_t launch_attn(const AttnParams& a, cudaStream_t s, bool pdl) {
  constexpr int MAXG = 8;
  const size_t smem = (size_t)(MAXG * HD + ATTN_CHUNK * (HD + 4) + ATTN_CHUNK * HD + MAXG * ATTN_CHUNK) * 4;
  static unsigned done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 32 && !(done & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    done |= 1u << dev;
  }
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
  return cudaLaunchKernelEx(&cfg, attention_kernel<HD>, a);
}

cudaError_t launch_attention(const AttnParams& a, cudaStream_t s, bool pdl) {
  if (a.n_heads % a.n_kv || a.n_heads / a.n_kv > 8) return cudaErrorInvalidValue;
  if (a.head_dim == 128) return launch_attn<128>(a, s, pdl);
  if (a.head_dim == 64) return launch_attn<64>(a, s, pdl);
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------ allocation-free attention

// Scratch of hakmc_attention_noalloc: split partials, per-kv-head tickets and
// the position word, in one file-scope device array. Every GPU that loads the
// library holds it (about 1 MiB) until the process exits.
constexpr size_t NOALLOC_PART_FLOATS = 256 * 1024;  // 1 MiB of split partials
constexpr int NOALLOC_TICKETS = 64;
struct NoAllocScratch {
  float part[NOALLOC_PART_FLOATS];
  unsigned tickets[NOALLOC_TICKETS];
  int pos;
};
static __device__ __align__(256) NoAllocScratch g_noalloc;

// Host code cannot use &g_noalloc (a host-side stand-in, not a device
// address): the device address comes from cudaGetSymbolAddress, once per
// device, with that device current.
static std::mutex g_noalloc_mu;
static NoAllocScratch* g_noalloc_dev[64];

__global__ void noalloc_prepare_kernel(NoAllocScratch* s, int pos) {
  if (threadIdx.x < NOALLOC_TICKETS) s->tickets[threadIdx.x] = 0u;  // must start at zero
  if (threadIdx.x == 0) s->pos = pos;
}

size_t noalloc_part_floats() { return NOALLOC_PART_FLOATS; }

cudaError_t attention_noalloc(float* out, const float* q, const float* kc, const float* vc, int pos, int n_heads,
                              int n_kv, int head_dim, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  NoAllocScratch* s = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_dev[dev]) {
      void* ptr = nullptr;
      e = cudaGetSymbolAddress(&ptr, g_noalloc);
      if (e != cudaSuccess) return e;
      g_noalloc_dev[dev] = static_cast<NoAllocScratch*>(ptr);
    }
    s = g_noalloc_dev[dev];
  }
  noalloc_prepare_kernel<<<1, NOALLOC_TICKETS, 0, stream>>>(s, pos);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  AttnParams a = {};
  a.q = q; a.k_cache = kc; a.v_cache = vc; a.out = out; a.pos_dev = &s->pos;
  a.n_heads = n_heads; a.n_kv = n_kv; a.head_dim = head_dim; a.scale = 1.0f / sqrtf((float)head_dim);
  a.n_split = pos / ATTN_CHUNK + 1;
  a.part = s->part;
  a.counters = s->tickets;
  return launch_attention(a, stream, false);
}

}  // namespace hakm
