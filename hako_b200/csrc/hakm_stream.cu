// hakm_stream.cu — the streaming GEMV "phase" kernel of the decode step.
//
// One launch computes out = W . act for one or more row segments that share
// the activation (e.g. q/k rows + v rows), with a fused prologue and epilogue.
// Each CTA (one per SM) owns a balanced slice of every segment's rows.
//
//   warp 0      producer: streams the CTA's weight rows through a ring of
//               shared-memory stages with cp.async.bulk (the TMA engine, no
//               tensor map: rows are contiguous), one 16-row x 8-block tile
//               per stage, completion on an mbarrier per stage. Weights do
//               not depend on the previous kernel, so the producer starts
//               before griddepcontrol.wait: under programmatic dependent
//               launch the next phase's weights are already in flight while
//               the previous phase drains.
//   warps 1..8  consumers: wait for the previous kernel (griddepcontrol.wait),
//               rebuild the activation in shared memory (rmsnorm and per-32
//               int8 quantization, src/nn.c:13-18 and src/quant.c:127-144),
//               then each takes 4-row units of a stage: Q4_K rows with dp4a
//               integer sub-block sums (src/quant.c:150-232), Q6_K rows as an
//               fp32 dot on the fly (src/nn.c:84-95, src/quant.c:94-123).
//               Per-(row, chunk) partial sums land in shared memory and are
//               summed in a fixed order, so results are deterministic.
//   epilogue    bias / residual / NeoX RoPE + K append / V append / SwiGLU /
//               logits + greedy argmax, and for the lm_head phase the step
//               finalisation (next token, token log, position + 1).
//
// Every wait on an mbarrier is bounded (clock64); a timeout sets
// PhaseParams::err_flag and the CTA drains its own copies and returns.
#include "hakm_device.cuh"

namespace hakm {

constexpr int CONSUMER_WARPS = 12;
constexpr int THREADS = 32 * (CONSUMER_WARPS + 1);
constexpr int TILE_ROWS = 16;
constexpr int UNITS = TILE_ROWS / 4;  // 4-row units per stage
constexpr int GROUPS = CONSUMER_WARPS / UNITS;  // consumer groups, one stage each
constexpr int MAX_STAGES = 12;
constexpr int SMEM_HEADER = 256;  // full[MAX_STAGES] and empty[MAX_STAGES] mbarriers
constexpr long long WAIT_LIMIT = 4000000000LL;  // ~2 s of SM clock
constexpr int BAR_CONSUMERS = 1;
constexpr int RMS_SLOTS = 2;  // 8-element slots per consumer thread in the rmsnorm prologue
constexpr int PHASE_BUDGET = 220 * 1024;

// ------------------------------------------------------------------ PTX

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > WAIT_LIMIT) return false;
  return true;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// trace slots per CTA: 0 start, 1 prologue done, 2 first stage ready,
// 3 last unit done, 4 epilogue done, 5 producer done issuing
constexpr int TRACE_SLOTS = 8;
#define TRACE(i)                                                               \
  do {                                                                         \
    if (p.trace) p.trace[(size_t)blockIdx.x * TRACE_SLOTS + (i)] = gtime();   \
  } while (0)

__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(BAR_CONSUMERS), "n"(CONSUMER_WARPS * 32) : "memory");
}

// ------------------------------------------------------------------ schedule

struct SegRange {
  int row0, row1, nch, part_base;
};

// This CTA's rows of segment s: the segment's 4-row groups split evenly over
// the grid, each segment's split rotated by the groups before it so the
// remainders of consecutive segments land on different CTAs.
__device__ __forceinline__ void cta_ranges(const PhaseParams& p, SegRange* sr) {
  const int grid = gridDim.x, cta = blockIdx.x, nb = p.n_in / QK;
  int goff = 0, pbase = 0;
  for (int s = 0; s < p.n_seg; s++) {
    const int n = p.seg[s].n_rows, G = (n + 3) / 4;
    const int idx = (cta - goff % grid + grid) % grid;
    const int g0 = (int)((long long)idx * G / grid), g1 = (int)((long long)(idx + 1) * G / grid);
    sr[s].row0 = 4 * g0;
    sr[s].row1 = min(4 * g1, n);
    sr[s].nch = n_chunks(nb);
    sr[s].part_base = pbase;
    pbase += (sr[s].row1 - sr[s].row0) * sr[s].nch;
    goff += G;
  }
}

// ------------------------------------------------------------------ prologue

__device__ float consumers_sum(float v, float* red) {
  const int cl = threadIdx.x - 32, lane = cl & 31, w = cl >> 5;
  v = warp_sum(v);
  consumers_sync();
  if (lane == 0) red[w] = v;
  consumers_sync();
  float t = lane < CONSUMER_WARPS ? red[lane] : 0.f;
  return warp_sum(t);
}

// 8-element slot s of the activation: fp32 values to xf, and for Q4_K rows the
// per-32 int8 codes. The 4 slots of a 32-block are 4 adjacent lanes, so the
// block max and code sum take two shuffles (quantize_row_q8_32 as built:
// xs = amax * fl(1/127), q = rint(x * (127/amax)), src/quant.c:127-144).
__device__ __forceinline__ void store_slot(const PhaseParams& p, int s, bool live, const float v[8], float* xf,
                                           int8_t* xq, float* xs, int* xsum) {
  if (live) {
    reinterpret_cast<float4*>(xf)[2 * s] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(xf)[2 * s + 1] = make_float4(v[4], v[5], v[6], v[7]);
  }
  if (!p.need_q8) return;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const float sc = amax * (1.0f / 127.0f);
  const float inv = q8_inv(amax, sc);
  int q[8], sum = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) { q[i] = q8_round(v[i] * inv); sum += q[i]; }
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  if (live) {
    uint2 pk;
    pk.x = (uint32_t)(q[0] & 255) | ((uint32_t)(q[1] & 255) << 8) | ((uint32_t)(q[2] & 255) << 16) |
           ((uint32_t)(q[3] & 255) << 24);
    pk.y = (uint32_t)(q[4] & 255) | ((uint32_t)(q[5] & 255) << 8) | ((uint32_t)(q[6] & 255) << 16) |
           ((uint32_t)(q[7] & 255) << 24);
    reinterpret_cast<uint2*>(xq)[s] = pk;
    if ((s & 3) == 0) { xs[s >> 2] = sc; xsum[s >> 2] = sum; }
  }
}

// Activation in shared memory: fp32 x (rmsnorm'ed for ACT_RMS) and, for Q4_K
// segments, its per-32 int8 quantization with the per-block sums of xq.
// ACT_RMS (K <= 8 * consumer threads): one slot per thread, the norm weights
// already in registers (loaded before the dependency wait), one reduction.
__device__ void build_activation(const PhaseParams& p, const float wpre[RMS_SLOTS][8], float* xf, int8_t* xq, float* xs,
                                 int* xsum, float* red) {
  const int K = p.n_in, nsb = K >> 5, nslot = K >> 3;
  const int t = threadIdx.x - 32, nt = CONSUMER_WARPS * 32;
  const int lane = t & 31, w = t >> 5;
  if (p.act == ACT_Q8) {
    const int4* src = reinterpret_cast<const int4*>(p.xq);
    int4* dst = reinterpret_cast<int4*>(xq);
    for (int i = t; i < K / 16; i += nt) dst[i] = src[i];
    for (int i = t; i < nsb; i += nt) xs[i] = p.xs[i];
    consumers_sync();
    for (int b = w; b < nsb; b += CONSUMER_WARPS) {
      const int s = warp_isum((int)xq[32 * b + lane]);
      if (lane == 0) xsum[b] = s;
    }
    consumers_sync();
    return;
  }
  const float4* x4 = reinterpret_cast<const float4*>(p.x);
  if (p.act == ACT_RMS) {
    float v[RMS_SLOTS][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < RMS_SLOTS; j++) {
      const int s = t + j * nt;
      if (s < nslot) {
        const float4 a = x4[2 * s], b = x4[2 * s + 1];
        v[j][0] = a.x; v[j][1] = a.y; v[j][2] = a.z; v[j][3] = a.w;
        v[j][4] = b.x; v[j][5] = b.y; v[j][6] = b.z; v[j][7] = b.w;
#pragma unroll
        for (int i = 0; i < 8; i++) ss += v[j][i] * v[j][i];
      } else {
#pragma unroll
        for (int i = 0; i < 8; i++) v[j][i] = 0.f;
      }
    }
    const float tot = consumers_sum(ss, red);
    // src/nn.c:16-17: scale = 1/sqrtf(ss/n + eps); y = x * scale * w
    const float scale = 1.0f / sqrtf(tot / (float)K + p.eps);
#pragma unroll
    for (int j = 0; j < RMS_SLOTS; j++) {
      const int s = t + j * nt;
      if (j * nt >= nslot) break;  // uniform: no live slot for any thread
#pragma unroll
      for (int i = 0; i < 8; i++) v[j][i] = v[j][i] * scale * wpre[j][i];
      store_slot(p, s, s < nslot, v[j], xf, xq, xs, xsum);
    }
  } else {
    for (int s0 = 0; s0 < nslot; s0 += nt) {
      const int s = s0 + t;
      const bool live = s < nslot;
      float v[8];
      if (live) {
        const float4 a = x4[2 * s], b = x4[2 * s + 1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = 0.f;
      }
      store_slot(p, s, live, v, xf, xq, xs, xsum);
    }
  }
  consumers_sync();
}

// ------------------------------------------------------------------ units

// Exact int -> float for |v| < 2^22 without a conversion instruction: v is
// added to the integer image of 1.5 * 2^23 and the bias removed in float.
__device__ __forceinline__ float i22_to_float(int v) {
  return __int_as_float(0x4B400000 + v) - 12582912.0f;
}

// Q4_K: lane (bl = lane/4, g = lane%4) owns qs bytes [32g, 32g+32) of block bl
// of the chunk: low nibbles are sub-block 2g, high nibbles sub-block 2g+1
// (src/quant.c:239-259). Per sub-block: xs * (d*s*sum(q*xq) - dmin*m*sum(xq)).
// The lane's activation slice of one chunk (64 int8 codes, two scales, two
// code sums) fits in registers; short rows keep it for the whole kernel.
struct Q4X {
  int a[8], b[8];
  float xsa, xsb;
  int sma, smb;
};

__device__ __forceinline__ Q4X q4x_load(const int8_t* xq, const float* xs, const int* xsum, int c, int nb) {
  const int lane = threadIdx.x & 31, bl = lane >> 2, g = lane & 3;
  Q4X X;
  const int b = min(CHUNK_BLOCKS * c + bl, nb - 1);  // lanes past the row end load a valid block, unused
  const int4* xa = reinterpret_cast<const int4*>(xq + 256 * b + 64 * g);
  const int4 xa0 = xa[0], xa1 = xa[1], xb0 = xa[2], xb1 = xa[3];
  X.a[0] = xa0.x; X.a[1] = xa0.y; X.a[2] = xa0.z; X.a[3] = xa0.w;
  X.a[4] = xa1.x; X.a[5] = xa1.y; X.a[6] = xa1.z; X.a[7] = xa1.w;
  X.b[0] = xb0.x; X.b[1] = xb0.y; X.b[2] = xb0.z; X.b[3] = xb0.w;
  X.b[4] = xb1.x; X.b[5] = xb1.y; X.b[6] = xb1.z; X.b[7] = xb1.w;
  X.xsa = xs[8 * b + 2 * g]; X.xsb = xs[8 * b + 2 * g + 1];
  X.sma = xsum[8 * b + 2 * g]; X.smb = xsum[8 * b + 2 * g + 1];
  return X;
}

__device__ __forceinline__ void q4k_unit(const uint8_t* st, int nrows, int m, const Q4X& X, float acc[4]) {
  const int lane = threadIdx.x & 31, bl = lane >> 2, g = lane & 3;
#pragma unroll
  for (int r = 0; r < 4; r++) acc[r] = 0.f;
  if (bl >= m) return;
  const int shf = 8 * (g & 1);  // byte of j&3 inside the scale words, (2g)&3 = 2(g&1)
#pragma unroll
  for (int r = 0; r < 4; r++) {
    if (r < nrows) {
      const uint8_t* blk = st + r * Q4K_CHUNK + bl * Q4K_BYTES;
      const uint4 hd = *reinterpret_cast<const uint4*>(blk);
      const uint4 q0 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * g);
      const uint4 q1 = *reinterpret_cast<const uint4*>(blk + 32 + 32 * g);
      const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
      int ia = 0, ib = 0;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        ia = __dp4a((int)(qw[i] & 0x0F0F0F0Fu), X.a[i], ia);
        ib = __dp4a((int)((qw[i] >> 4) & 0x0F0F0F0Fu), X.b[i], ib);
      }
      const float d = half_bits_to_float(hd.x), dmin = half_bits_to_float(hd.x >> 16);
      // get_scale_min_k4 (src/quant.c:57-66) for j = 2g and 2g+1: scales[0..3]
      // in hd.y, [4..7] in hd.z, [8..11] in hd.w; j < 4 iff g < 2
      int sa, ma, sb, mb;
      {
        const uint32_t Y = hd.y >> (2 * shf), Z = hd.z >> (2 * shf), W = hd.w >> (2 * shf);
        const uint32_t Y1 = Y >> 8, Z1 = Z >> 8, W1 = W >> 8;
        if (g < 2) {
          sa = Y & 63; ma = Z & 63; sb = Y1 & 63; mb = Z1 & 63;
        } else {
          sa = (W & 15) | ((Y >> 2) & 0x30); ma = ((W >> 4) & 15) | ((Z >> 2) & 0x30);
          sb = (W1 & 15) | ((Y1 >> 2) & 0x30); mb = ((W1 >> 4) & 15) | ((Z1 >> 2) & 0x30);
        }
      }
      // xs * (d*(s*iqx) - dmin*(m*ix)): the integer products are exact
      // (|s*iqx| <= 63*32*15*127 < 2^22) and become floats by exponent bias
      acc[r] += X.xsa * (d * i22_to_float(sa * ia) - dmin * i22_to_float(ma * X.sma));
      acc[r] += X.xsb * (d * i22_to_float(sb * ib) - dmin * i22_to_float(mb * X.smb));
    }
  }
}

// Q6_K: two passes of 4 blocks. Lane (bq = lane/8, n = half, k = quarter) of
// block bl = 4*pass + bq owns ql[64n + 16k .. +16]: low nibbles are elements
// 128n + 16k + i (scale group 8n + k), high nibbles 128n + 64 + 16k + i (group
// 8n + 4 + k); their two high bits sit in qh[32n + 16(k&1) + i] at bits 0/2
// and 4/6 — the element map of dequant_q6_K (src/quant.c:94-123).
struct Q6X {
  float lo[2][16], hi[2][16];
};

__device__ __forceinline__ void q6x_load(const float* xf, int c, int nb, Q6X& X) {
  const int lane = threadIdx.x & 31, bq = lane >> 3, n = (lane >> 2) & 1, k = lane & 3;
#pragma unroll
  for (int pass = 0; pass < 2; pass++) {
    const int b = min(CHUNK_BLOCKS * c + 4 * pass + bq, nb - 1);
    const float4* xl4 = reinterpret_cast<const float4*>(xf + 256 * b + 128 * n + 16 * k);
    const float4* xh4 = reinterpret_cast<const float4*>(xf + 256 * b + 128 * n + 64 + 16 * k);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float4 a = xl4[i], e = xh4[i];
      X.lo[pass][4 * i] = a.x; X.lo[pass][4 * i + 1] = a.y; X.lo[pass][4 * i + 2] = a.z; X.lo[pass][4 * i + 3] = a.w;
      X.hi[pass][4 * i] = e.x; X.hi[pass][4 * i + 1] = e.y; X.hi[pass][4 * i + 2] = e.z; X.hi[pass][4 * i + 3] = e.w;
    }
  }
}

__device__ __forceinline__ void q6k_unit(const uint8_t* st, int nrows, int m, const Q6X& X, float acc[4]) {
  const int lane = threadIdx.x & 31, bq = lane >> 3, n = (lane >> 2) & 1, k = lane & 3;
  const int sh_lo = (k < 2) ? 0 : 2, sh_hi = (k < 2) ? 4 : 6;
#pragma unroll
  for (int r = 0; r < 4; r++) acc[r] = 0.f;
#pragma unroll
  for (int pass = 0; pass < 2; pass++) {
    const int bl = 4 * pass + bq;
    if (bl >= m) continue;
#pragma unroll
    for (int r = 0; r < 4; r++) {
      if (r < nrows) {
        const uint8_t* chunk = st + r * Q6K_CHUNK;
        const uint8_t* body = chunk + bl * Q6K_BODY;
        const uint4 ql = *reinterpret_cast<const uint4*>(body + 64 * n + 16 * k);
        const uint4 qh = *reinterpret_cast<const uint4*>(body + 128 + 32 * n + 16 * (k & 1));
        const uint2 sc = *reinterpret_cast<const uint2*>(body + 192 + 8 * n);
        const float d = __half2float(*reinterpret_cast<const __half*>(chunk + m * Q6K_BODY + 2 * bl));
        const uint32_t lw[4] = {ql.x, ql.y, ql.z, ql.w};
        const uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
        float slo = 0.f, shi = 0.f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint32_t lo = (lw[i] & 0x0F0F0F0Fu) | (((hw[i] >> sh_lo) & 0x03030303u) << 4);
          const uint32_t hi = ((lw[i] >> 4) & 0x0F0F0F0Fu) | (((hw[i] >> sh_hi) & 0x03030303u) << 4);
#pragma unroll
          for (int t = 0; t < 4; t++) {
            slo = fmaf(q6_val(lo, t), X.lo[pass][4 * i + t], slo);
            shi = fmaf(q6_val(hi, t), X.hi[pass][4 * i + t], shi);
          }
        }
        // scales: sc[8n + k] is byte k of word 0 of this half, sc[8n + 4 + k] byte k of word 1
        const float sl = (float)(int8_t)(sc.x >> (8 * k)), sh = (float)(int8_t)(sc.y >> (8 * k));
        acc[r] += d * sl * slo + d * sh * shi;
      }
    }
  }
}

// Sum each of 4 per-lane partials over the warp with 6 shuffles: afterwards
// lane 8r (r < 4) holds the total of partial r.
__device__ __forceinline__ float reduce4(const float acc[4]) {
  const int lane = threadIdx.x & 31;
  const bool hi16 = lane & 16, hi8 = lane & 8;
  const float k0 = hi16 ? acc[2] : acc[0], k1 = hi16 ? acc[3] : acc[1];
  const float s0 = hi16 ? acc[0] : acc[2], s1 = hi16 ? acc[1] : acc[3];
  const float a0 = k0 + __shfl_xor_sync(0xffffffffu, s0, 16);
  const float a1 = k1 + __shfl_xor_sync(0xffffffffu, s1, 16);
  float b = (hi8 ? a1 : a0) + __shfl_xor_sync(0xffffffffu, hi8 ? a0 : a1, 8);
  b += __shfl_xor_sync(0xffffffffu, b, 4);
  b += __shfl_xor_sync(0xffffffffu, b, 2);
  b += __shfl_xor_sync(0xffffffffu, b, 1);
  return b;
}

// ------------------------------------------------------------------ epilogue

__device__ __forceinline__ float row_total(const float* part, const SegRange& r, int row) {
  const float* pp = part + r.part_base + (row - r.row0) * r.nch;
  float v = pp[0];
  for (int c = 1; c < r.nch; c++) v += pp[c];
  return v;
}

__device__ void epilogue(const PhaseParams& p, const SegRange* sr, const float* part, float* red) {
  const int t = threadIdx.x - 32, nt = CONSUMER_WARPS * 32;
  const int pos = p.pos_dev ? *p.pos_dev : 0;
  unsigned long long best = 0ull;
  for (int s = 0; s < p.n_seg; s++) {
    const Seg& S = p.seg[s];
    const SegRange& r = sr[s];
    if (S.epi == EPI_ROPE_QK || S.epi == EPI_SWIGLU) {
      for (int q = t; 2 * q + 1 < r.row1 - r.row0; q += nt) {
        const int dr = r.row0 + 2 * q;
        const float a0 = row_total(part, r, dr), a1 = row_total(part, r, dr + 1);
        if (S.epi == EPI_SWIGLU) {
          // src/model.c:154 with silu_f (src/nn.c:29)
          S.out[dr >> 1] = a0 / (1.0f + expf(-a0)) * a1;
        } else {
          const float x0 = S.bias ? a0 + S.bias[dr] : a0;
          const float x1 = S.bias ? a1 + S.bias[dr + 1] : a1;
          const bool is_k = dr >= S.split;
          const int lr = is_k ? dr - S.split : dr;
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
    } else {
      for (int row = r.row0 + t; row < r.row1; row += nt) {
        const float v = row_total(part, r, row);
        switch (S.epi) {
          case EPI_STORE: S.out[row] = S.bias ? v + S.bias[row] : v; break;
          case EPI_RESID: S.out[row] += v; break;
          case EPI_V_CACHE: {
            const float o = S.bias ? v + S.bias[row] : v;
            S.out[row] = o;
            S.cache[(size_t)pos * p.kv_dim + row] = o;
            break;
          }
          case EPI_ARGMAX: {
            if (S.out) S.out[row] = v;
            const unsigned long long kk = argmax_key(v, row);
            best = kk > best ? kk : best;
            break;
          }
        }
      }
    }
  }
  if (p.argmax_key) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if ((t & 31) == 0 && best) atomicMax(p.argmax_key, best);
  }
}

// ------------------------------------------------------------------ kernel

// KINDS: bit 0 = Q4_K segments, bit 1 = Q6_K segments. CACHE: the lane's
// activation slices stay in registers for the whole kernel (rows of at most
// two chunks for Q4_K, one chunk for Q6_K); otherwise they are re-read from
// shared memory per 4-row unit.
template <int KINDS, bool CACHE>
__global__ void __launch_bounds__(THREADS, 1) stream_kernel(const __grid_constant__ PhaseParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + MAX_STAGES;
  const int S_ = p.n_stages, SB = p.stage_bytes;
  uint8_t* ring = smem + SMEM_HEADER;
  const int K = p.n_in, nb = K / QK, nsb = K / 32;
  float* xf = reinterpret_cast<float*>(ring + (size_t)S_ * SB);
  int8_t* xq = reinterpret_cast<int8_t*>(xf + K);
  float* xs = reinterpret_cast<float*>(xq + K);
  int* xsum = reinterpret_cast<int*>(xs + nsb);
  float* part = reinterpret_cast<float*>(xsum + nsb);
  float* red = part + p.part_floats;

  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) TRACE(0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S_; i++) {
      mbar_init(smem_addr(&full[i]), 1);
      mbar_init(smem_addr(&empty[i]), UNITS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();

  SegRange sr[MAX_SEGS];
  cta_ranges(p, sr);
  bool failed = false;

  if (warp == 0) {
    // ---------------- producer ----------------
    int i = 0;
    for (int s = 0; s < p.n_seg && !failed; s++) {
      const Seg& S = p.seg[s];
      const int type = (KINDS == 1) ? W_Q4K : (KINDS == 2) ? W_Q6K : S.type;
      const size_t rowB = dev_row_bytes(type, nb);
      const int stride = type == W_Q4K ? Q4K_CHUNK : Q6K_CHUNK;
      for (int rt = sr[s].row0; rt < sr[s].row1 && !failed; rt += TILE_ROWS) {
        const int nr = min(TILE_ROWS, sr[s].row1 - rt);
        for (int c = 0; c < sr[s].nch; c++, i++) {
          const int slot = i % S_;
          if (i >= S_) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait(smem_addr(&empty[slot]), ((i / S_) - 1) & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) { failed = true; break; }
          }
          const int cb = chunk_bytes(type, nb, c);
          if (lane == 0) mbar_expect_tx(smem_addr(&full[slot]), (uint32_t)(nr * cb));
          __syncwarp();
          if (lane < nr)
            bulk_g2s(smem_addr(ring + (size_t)slot * SB + lane * stride),
                     S.w + (size_t)(rt + lane) * rowB + (size_t)c * stride, (uint32_t)cb,
                     smem_addr(&full[slot]));
        }
      }
    }
    if (lane == 0) TRACE(5);
    // drain: every copy this CTA issued must land before the CTA exits
    if (lane == 0) {
      for (int j = (i > S_ ? i - S_ : 0); j < i; j++)
        if (!mbar_wait(smem_addr(&full[j % S_]), (j / S_) & 1)) failed = true;
    }
  } else {
    // ---------------- consumers ----------------
    // norm weights do not depend on the previous kernel: fetch them first
    float wpre[RMS_SLOTS][8];
#pragma unroll
    for (int j = 0; j < RMS_SLOTS; j++) {
      const int s = threadIdx.x - 32 + j * CONSUMER_WARPS * 32;
      if (p.act == ACT_RMS && s < p.n_in / 8) {
        const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
        const float4 a = w4[2 * s], b = w4[2 * s + 1];
        wpre[j][0] = a.x; wpre[j][1] = a.y; wpre[j][2] = a.z; wpre[j][3] = a.w;
        wpre[j][4] = b.x; wpre[j][5] = b.y; wpre[j][6] = b.z; wpre[j][7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; i++) wpre[j][i] = 0.f;
      }
    }
    pdl_wait();
    build_activation(p, wpre, xf, xq, xs, xsum, red);
    if (threadIdx.x == 32) TRACE(1);
    const int cw = warp - 1, mine = cw >> 2, unit = cw & 3;
    bool first = true;
    // short rows: the lane's activation slice stays in registers for the kernel
    const int nch_all = n_chunks(nb);
    constexpr bool c4 = CACHE && (KINDS & 1);
    constexpr bool c6 = CACHE && KINDS == 2;
    Q4X x4c0, x4c1;
    Q6X x6c;
    if constexpr (c4) {
      x4c0 = q4x_load(xq, xs, xsum, 0, nb);
      x4c1 = nch_all > 1 ? q4x_load(xq, xs, xsum, 1, nb) : x4c0;
    }
    if constexpr (c6) q6x_load(xf, 0, nb, x6c);
    int i = 0;
    for (int s = 0; s < p.n_seg && !failed; s++) {
      const int type = (KINDS == 1) ? W_Q4K : (KINDS == 2) ? W_Q6K : p.seg[s].type;
      for (int rt = sr[s].row0; rt < sr[s].row1 && !failed; rt += TILE_ROWS) {
        const int nr = min(TILE_ROWS, sr[s].row1 - rt);
        for (int c = 0; c < sr[s].nch; c++, i++) {
          if (i % GROUPS != mine) continue;
          const int slot = i % S_;
          if (!mbar_wait(smem_addr(&full[slot]), (i / S_) & 1)) { failed = true; break; }
          if (first && threadIdx.x == 32) TRACE(2);
          first = false;
          const int t0 = 4 * unit, nru = min(4, nr - t0);
          if (nru > 0) {
            const uint8_t* st = ring + (size_t)slot * SB;
            const int m = q6_chunk_blocks(nb, c);
            float acc[4];
#pragma unroll
            for (int r = 0; r < 4; r++) acc[r] = 0.f;
            if (type == W_Q4K) {
              if constexpr (KINDS & 1) {
                if constexpr (c4) q4k_unit(st + t0 * Q4K_CHUNK, nru, m, c == 0 ? x4c0 : x4c1, acc);
                else q4k_unit(st + t0 * Q4K_CHUNK, nru, m, q4x_load(xq, xs, xsum, c, nb), acc);
              }
            } else {
              if constexpr (KINDS & 2) {
                if constexpr (c6) {
                  q6k_unit(st + t0 * Q6K_CHUNK, nru, m, x6c, acc);
                } else {
                  Q6X X;
                  q6x_load(xf, c, nb, X);
                  q6k_unit(st + t0 * Q6K_CHUNK, nru, m, X, acc);
                }
              }
            }
            const float tot = reduce4(acc);
            if ((lane & 7) == 0 && (lane >> 3) < nru)
              part[sr[s].part_base + (rt - sr[s].row0 + t0 + (lane >> 3)) * sr[s].nch + c] = tot;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_addr(&empty[slot]));
        }
      }
    }
    consumers_sync();
    if (threadIdx.x == 32) TRACE(3);
    if (!failed) epilogue(p, sr, part, red);
    if (threadIdx.x == 32) TRACE(4);
  }

  if (failed && p.err_flag) atomicExch(p.err_flag, 1);
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

// ------------------------------------------------------------------ host

static int phase_kinds(const PhaseParams& p) {
  int k = 0;
  for (int i = 0; i < p.n_seg; i++) k |= (p.seg[i].type == W_Q4K) ? 1 : 2;
  return k;
}

static int phase_grid_size(const PhaseParams& p, int num_sms) {
  int groups = 0;
  for (int s = 0; s < p.n_seg; s++) groups += (p.seg[s].n_rows + 3) / 4;
  return groups < num_sms ? (groups < 1 ? 1 : groups) : num_sms;
}

// Fills n_stages / stage_bytes / part_floats; returns the dynamic smem size.
static size_t plan(PhaseParams& q, int grid) {
  const int K = q.n_in, nb = K / QK;
  int stride = 0, part = 0;
  for (int s = 0; s < q.n_seg; s++) {
    const int st = q.seg[s].type == W_Q4K ? Q4K_CHUNK : Q6K_CHUNK;
    stride = st > stride ? st : stride;
    const int G = (q.seg[s].n_rows + 3) / 4;
    part += ((G + grid - 1) / grid) * 4 * n_chunks(nb);
  }
  q.stage_bytes = TILE_ROWS * stride;
  q.part_floats = (part + 3) & ~3;
  const size_t fixed = SMEM_HEADER + (size_t)K * 4 + K + (size_t)(K / 32) * 8 + (size_t)q.part_floats * 4 + 64 * 4;
  // Stage i lives in slot i % S and is consumed by group i % GROUPS. S must
  // be a multiple of GROUPS: then every slot belongs to one group, which waits
  // on that slot's phases strictly in order — a parity wait can never see a
  // phase two behind and alias.
  const long avail = (long)PHASE_BUDGET - (long)fixed;
  const int k = avail >= 3L * GROUPS * q.stage_bytes ? 3 : (avail >= 2L * GROUPS * q.stage_bytes ? 2 : 1);
  q.n_stages = k * GROUPS;
  return fixed + (size_t)q.n_stages * q.stage_bytes;
}

size_t phase_smem_bytes(const PhaseParams& p, int grid) {
  PhaseParams q = p;
  return plan(q, grid);
}

template <int KINDS, bool CACHE>
static cudaError_t launch_k(const PhaseParams& p, int grid, size_t smem, cudaStream_t s, bool pdl) {
  static unsigned done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 32 && !(done & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(stream_kernel<KINDS, CACHE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         PHASE_SMEM_MAX);
    if (e != cudaSuccess) return e;
    done |= 1u << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, stream_kernel<KINDS, CACHE>, p);
}

cudaError_t launch_phase(const PhaseParams& p0, int num_sms, cudaStream_t s, bool pdl) {
  PhaseParams p = p0;
  if (p.act == ACT_RMS && p.n_in > 8 * RMS_SLOTS * CONSUMER_WARPS * 32) return cudaErrorInvalidValue;
  const int grid = phase_grid_size(p, num_sms);
  const size_t smem = plan(p, grid);
  if (smem > (size_t)PHASE_SMEM_MAX || p.n_stages > MAX_STAGES) return cudaErrorInvalidValue;
  const int kinds = phase_kinds(p), nch = n_chunks(p.n_in / QK);
  if (kinds == 1) return nch <= 2 ? launch_k<1, true>(p, grid, smem, s, pdl) : launch_k<1, false>(p, grid, smem, s, pdl);
  if (kinds == 2) return nch == 1 ? launch_k<2, true>(p, grid, smem, s, pdl) : launch_k<2, false>(p, grid, smem, s, pdl);
  return nch <= 2 ? launch_k<3, true>(p, grid, smem, s, pdl) : launch_k<3, false>(p, grid, smem, s, pdl);
}

}  // namespace hakm
