// hakm_kernels.cu — the small kernels of libhakm_cuda: the stand-alone
// activation quantizer, exact Q4_K integer sub-block sums, Q6_K re-layout,
// dequantization, rmsnorm, embedding lookup, NeoX RoPE and GQA decode
// attention. The streaming GEMV phases live in hakm_stream.cu.
#include "hakm_attn.cuh"
#include "hakm_device.cuh"
#include "hakm_exact.cuh"

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
  // NaN elements do not raise amax (src/quant.c:131-133 keeps the larger of
  // amax and |x| with a comparison that a NaN never wins)
  const float amax = warp_max(fmaxf(0.0f, fabsf(v)));
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
// per 8-block chunk the 208-byte bodies (bytes reordered by lane class,
// q6k_body_pos), then the 8 fp16 d values. One warp
// per block; the destination is zeroed first so chunk padding is defined.
__global__ void q6k_pack_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, int n_rows, int nb) {
  const long blk = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (blk >= (long)n_rows * nb) return;
  const int r = (int)(blk / nb), b = (int)(blk % nb);
  const int c = b / CHUNK_BLOCKS, j = b % CHUNK_BLOCKS, m = q6_chunk_blocks(nb, c);
  const uint8_t* s = src + blk * Q6K_BYTES;
  uint8_t* chunk = dst + (size_t)r * dev_row_bytes(W_Q6K, nb) + (size_t)c * Q6K_CHUNK;
  for (int i = lane; i < Q6K_BODY; i += 32) chunk[j * Q6K_BODY + q6k_body_pos(i)] = s[i];
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

// rmsnorm (src/nn.c:13-18) as the reference's build computes it: one warp
// takes sum(x*x) in the 8-lane vectorized order (lane l adds the rounded
// squares of x[8t + l] in order, then the lanes fold), ss/n + eps, the
// rsqrtss Newton step, then y = (x * w) * scale. n is a multiple of 8.
__global__ void rmsnorm_kernel(float* y, const float* x, const float* w, int n, float eps, const uint32_t* rsq) {
  __shared__ float s_scale;
  if (threadIdx.x < 32) {
    const int l = threadIdx.x & 7;
    float acc = 0.f;
    if (threadIdx.x < 8)
      for (int i = l; i < n; i += 8) acc = __fadd_rn(acc, __fmul_rn(x[i], x[i]));
    const float ss = fold8_lanes(acc);
    if (threadIdx.x == 0) s_scale = rsqrt_nr(__fadd_rn(__fdiv_rn(ss, (float)n), eps), rsq);
  }
  __syncthreads();
  const float scale = s_scale;
  for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fmul_rn(__fmul_rn(x[i], w[i]), scale);
}

cudaError_t launch_rmsnorm(float* y, const float* x, const float* w, int n, float eps, const uint32_t* rsq,
                           cudaStream_t s) {
  if (n % 8 || !rsq) return cudaErrorInvalidValue;
  rmsnorm_kernel<<<1, 1024, 0, s>>>(y, x, w, n, eps, rsq);
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
  const float2 r = rope_rotate(a, b, cs.x, cs.y);
  x[h * hd + i] = r.x;
  x[h * hd + i + half] = r.y;
}

cudaError_t launch_rope(float* x, const float* rope_cs, const int* pos_dev, int n_heads, int head_dim,
                        cudaStream_t s) {
  const int n = n_heads * head_dim / 2;
  rope_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, rope_cs, pos_dev, n_heads, head_dim);
  return cudaGetLastError();
}

// ------------------------------------------------------------ attention

// Standalone attention launch: one CTA per (query head, dimension slice).
struct BlockSync {
  __device__ void operator()() const { __syncthreads(); }
};

template <int HD>
__global__ void __launch_bounds__(256) attention_kernel(const AttnParams a) {
  extern __shared__ __align__(16) float sm[];
  pdl_launch_dependents();
  pdl_wait();
  attn_item<HD, false>(a, blockIdx.x, *a.pos_dev, sm, threadIdx.x, blockDim.x, BlockSync());
}

size_t attention_scratch_floats(int n_heads, int head_dim, int n_pos) {
  return (size_t)attn_units(n_heads, head_dim) * (size_t)n_pos;
}

template <int HD>
static cudaError_t launch_attn(const AttnParams& a, cudaStream_t s, bool pdl) {
  const size_t smem = attn_smem_bytes(HD);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(attn_units(a.n_heads, HD));
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
  if (a.n_kv <= 0 || a.n_heads % a.n_kv || !a.part || a.score_stride < 1) return cudaErrorInvalidValue;
  if (a.head_dim == 128) return launch_attn<128>(a, s, pdl);
  if (a.head_dim == 64) return launch_attn<64>(a, s, pdl);
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------ exp test hook

__global__ void exp_probe_kernel(float* out, const float* in, int n, int variant) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = in[i];
  out[i] = variant == 1 ? exp_v8(x) : variant == 2 ? exp_v4(x) : exp_scalar(x);
}

cudaError_t launch_exp_probe(float* out, const float* in, int n, int variant, cudaStream_t s) {
  exp_probe_kernel<<<(n + 255) / 256, 256, 0, s>>>(out, in, n, variant);
  return cudaGetLastError();
}

// ------------------------------------------------------------ rsqrtss table

extern "C" void hakm_host_rsqrt_table(uint32_t* out);
extern "C" int hakm_host_rsqrt_table_ok(const uint32_t* tab);
extern "C" float hakm_host_rsqrt_nr(float v);

float host_rsqrt_nr(float v) { return hakm_host_rsqrt_nr(v); }

// One copy per device, made on first use and kept until the process exits.
static std::mutex g_rsq_mu;
static uint32_t* g_rsq_dev[64];

const uint32_t* rsqrt_table_device(int dev) {
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_rsq_mu);
  if (g_rsq_dev[dev]) return g_rsq_dev[dev];
  static uint32_t host[2048];
  static int host_ok = -1;
  if (host_ok < 0) {
    hakm_host_rsqrt_table(host);
    host_ok = hakm_host_rsqrt_table_ok(host);
  }
  if (!host_ok) return nullptr;
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return nullptr;
  if (cur != dev && cudaSetDevice(dev) != cudaSuccess) return nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, sizeof host);
  if (e == cudaSuccess) e = cudaMemcpy(p, host, sizeof host, cudaMemcpyHostToDevice);
  if (cur != dev) cudaSetDevice(cur);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return nullptr;
  }
  g_rsq_dev[dev] = static_cast<uint32_t*>(p);
  return g_rsq_dev[dev];
}

extern "C" void hakm_host_rcp_table(uint32_t* out);
extern "C" int hakm_host_rcp_table_ok(const uint32_t* tab);
static uint32_t* g_rcp_dev[64];

const uint32_t* rcp_table_device(int dev) {
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_rsq_mu);
  if (g_rcp_dev[dev]) return g_rcp_dev[dev];
  static uint32_t host[2048];
  static int host_ok = -1;
  if (host_ok < 0) {
    hakm_host_rcp_table(host);
    host_ok = hakm_host_rcp_table_ok(host);
  }
  if (!host_ok) return nullptr;
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return nullptr;
  if (cur != dev && cudaSetDevice(dev) != cudaSuccess) return nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, sizeof host);
  if (e == cudaSuccess) e = cudaMemcpy(p, host, sizeof host, cudaMemcpyHostToDevice);
  if (cur != dev) cudaSetDevice(cur);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return nullptr;
  }
  g_rcp_dev[dev] = static_cast<uint32_t*>(p);
  return g_rcp_dev[dev];
}

// ------------------------------------------------------------ allocation-free attention

// Scratch of hakmc_attention_noalloc: the score rows of the attention units
// and the position word, in one file-scope device array. Every GPU that
// loads the library holds it (about 1 MiB) until the process exits.
constexpr size_t NOALLOC_PART_FLOATS = 256 * 1024;  // 1 MiB of score rows
struct NoAllocScratch {
  float part[NOALLOC_PART_FLOATS];
  int pos;
};
static __device__ __align__(256) NoAllocScratch g_noalloc;

// Host code cannot use &g_noalloc (a host-side stand-in, not a device
// address): the device address comes from cudaGetSymbolAddress, once per
// device, with that device current.
static std::mutex g_noalloc_mu;
static NoAllocScratch* g_noalloc_dev[64];

__global__ void noalloc_prepare_kernel(NoAllocScratch* s, int pos) {
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
  noalloc_prepare_kernel<<<1, 32, 0, stream>>>(s, pos);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  AttnParams a = {};
  a.q = q; a.k_cache = kc; a.v_cache = vc; a.out = out; a.pos_dev = &s->pos;
  a.n_heads = n_heads; a.n_kv = n_kv; a.head_dim = head_dim; a.scale = host_rsqrt_nr((float)head_dim);
  a.part = s->part;
  a.score_stride = pos + 1;
  return launch_attention(a, stream, false);
}

}  // namespace hakm
