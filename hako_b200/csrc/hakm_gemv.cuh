// hakm_gemv.cuh — device building blocks of the streaming GEMV phases, shared
// by the per-phase kernel (hakm_stream.cu) and the persistent decode-step
// kernel (hakm_step.cu): bulk-copy / mbarrier helpers, per-CTA row schedule,
// the activation prologue (rmsnorm, int8 q8_32 codes, fixed-point limbs), the
// Q4_K and Q6_K 4-row units and the fused epilogues.
//
// Activations produced by other SMs earlier in the same kernel are read with
// L2-coherent loads (__ldcg): L1 is not coherent across SMs.
#pragma once
#include "hakm_device.cuh"

namespace hakm {


constexpr int CONSUMER_WARPS = 11;  // 12 warps in all: 168 registers a thread, no spills
constexpr int THREADS = 32 * (CONSUMER_WARPS + 1);
constexpr int TILE_ROWS = 16;         // most rows a stage holds
constexpr int STAGE_TARGET = 40 * 1024;  // bytes a stage aims for
constexpr int PHASE_BUDGET = 220 * 1024;  // dynamic shared memory a phase CTA may use
// Consumer groups of the per-phase kernel: stage i is consumed by group
// i % groups (one group of all consumer warps).
constexpr int MAX_STAGES = 12;
constexpr int SMEM_HEADER = 256;  // full[MAX_STAGES] and empty[MAX_STAGES] mbarriers
constexpr long long WAIT_LIMIT = 4000000000LL;  // ~2 s of SM clock
constexpr int BAR_CONSUMERS = 1;
constexpr int RMS_SLOTS = 2;  // 8-element slots per consumer thread in the rmsnorm prologue

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
// As mbar_try_wait, but the thread may be suspended (up to the hint, 1 ms)
// until the phase completes instead of returning at once: a waiting warp
// issues nothing while it sleeps.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "n"(1000000)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_sleep(bar, parity))
    if (clock64() - t0 > WAIT_LIMIT) return false;
  return true;
}
// Weight rows are read once per token: the copy carries an L2 evict-first
// policy so the stream does not push the small hot data (exchanged vectors,
// K/V rows, norm weights, descriptors) out of L2.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
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

// Limb planes of the Q6_K activation: 64 bytes of padding after every 128
// elements (see struct Act).
__host__ __device__ inline size_t limb_plane_bytes(int K) { return (size_t)K + (size_t)K / 2; }
__device__ __forceinline__ int limb_pos(int e) { return e + 64 * (e >> 7); }

// Shared-memory bytes of the activation for an n_in of K.
__host__ __device__ inline size_t act_bytes(int K, bool q8, bool q6) {
  size_t b = 0;
  if (q8) b += (size_t)K + (size_t)(K / 32) * 8;
  if (q6) b += 3 * limb_plane_bytes(K) + (size_t)(K / 16) * 8;
  return b;
}

// Rows per stage for a segment: whole rows, as many (power of two, <= 16) as
// fit STAGE_TARGET. A segment's rows are contiguous, so a stage is ONE bulk
// copy: per-copy cost in the copy engine made 16 row-sized copies per stage
// the bottleneck.
__host__ __device__ inline int phase_groups(int) { return 1; }
__host__ __device__ inline int stage_rows(int type, int nb) {
  const size_t rb = dev_row_bytes(type, nb);
  // long rows: up to twice the target, but two stages must fit beside the
  // activation (fp32 + int8 copies, scales) in the shared-memory budget
  const size_t act = act_bytes(nb * QK, true, true) + 8192;
  size_t target = STAGE_TARGET;
  if (phase_groups(nb) == 1) {
    const size_t two = ((size_t)PHASE_BUDGET - act) / 2;
    target = two < 2 * (size_t)STAGE_TARGET ? two : 2 * (size_t)STAGE_TARGET;
  }
  int r = TILE_ROWS;
  while (r > 1 && (size_t)r * rb > target) r >>= 1;
  return r;
}

// Rows per stage in the persistent step kernel, whose ring has one slot size
// for every phase: as many whole rows as fit the slot, a multiple of 4 when
// that still leaves at least 8 (full 4-row units).
__host__ __device__ inline int stage_rows_for(int type, int nb, int slot_bytes) {
  const int r = (int)((unsigned)slot_bytes / (unsigned)dev_row_bytes(type, nb));
  return r >= 8 ? (r & ~3) : r;
}


// This CTA's rows of segment s: the segment's 4-row groups split evenly over
// the grid, each segment's split rotated by the groups before it so the
// remainders of consecutive segments land on different CTAs.
// 32-bit arithmetic throughout (groups * grid < 2^31): this runs in every
// CTA at the start of every phase, on the critical path.
__device__ __forceinline__ void cta_ranges(const PhaseParams& p, SegRange* sr) {
  const unsigned grid = gridDim.x, cta = blockIdx.x;
  const int nb = p.n_in / QK;
  unsigned goff = 0;
  int pbase = 0;
  for (int s = 0; s < p.n_seg; s++) {
    const int n = p.seg[s].n_rows;
    const unsigned G = (unsigned)(n + 3) / 4;
    const unsigned idx = (cta + grid - goff % grid) % grid;
    const int g0 = (int)(idx * G / grid), g1 = (int)((idx + 1) * G / grid);
    sr[s].row0 = 4 * g0;
    sr[s].row1 = min(4 * g1, n);
    sr[s].nch = n_chunks(nb);
    sr[s].part_base = pbase;
    pbase += (sr[s].row1 - sr[s].row0) * sr[s].nch;
    goff += G;
  }
}

// ------------------------------------------------------------------ prologue

static __device__ float consumers_sum(float v, float* red) {
  const int cl = threadIdx.x - 32, lane = cl & 31, w = cl >> 5;
  v = warp_sum(v);
  consumers_sync();
  if (lane == 0) red[w] = v;
  consumers_sync();
  float t = lane < CONSUMER_WARPS ? red[lane] : 0.f;
  return warp_sum(t);
}

// The activation in shared memory, in the two forms the row types consume:
//  q8    (Q4_K rows): per-32 int8 codes xq, scales xs and code sums xsum —
//        quantize_row_q8_32 as the reference builds it (src/quant.c:127-144).
//  limbs (Q6_K rows): each 16-element group as exact 23-bit fixed point
//        relative to its largest element, X = rint(x * 2^(22-E)), split into
//        bytes X = X2*2^16 + X1*2^8 + X0 (X0, X1 unsigned, X2 signed) so the
//        fp32-activation dot of the generic path (src/nn.c:84-95) becomes
//        three int8 dot products; lp[g] = (32 * sum(X), 2^(E-22)). Planes
//        put 64 bytes of padding after every 128 elements, which makes the
//        lanes' 16-byte reads bank-conflict free.
struct Act {
  int8_t* xq;
  float* xs;
  int* xsum;
  uint8_t* l0;
  uint8_t* l1;
  uint8_t* l2;
  float2* lp;
};


__device__ __forceinline__ Act carve_act(uint8_t* base, int K, bool q8, bool q6) {
  Act a = {};
  uint8_t* p = base;
  if (q6) {
    a.lp = reinterpret_cast<float2*>(p);
    p += (size_t)(K / 16) * 8;
    a.l0 = p; p += limb_plane_bytes(K);
    a.l1 = p; p += limb_plane_bytes(K);
    a.l2 = p; p += limb_plane_bytes(K);
  }
  if (q8) {
    a.xs = reinterpret_cast<float*>(p);
    p += (size_t)(K / 32) * 4;
    a.xsum = reinterpret_cast<int*>(p);
    p += (size_t)(K / 32) * 4;
    a.xq = reinterpret_cast<int8_t*>(p);
  }
  return a;
}

// 8-element slot s (elements [8s, 8s+8)). For q8 the 4 slots of a 32-block
// are 4 adjacent lanes, for limbs the 2 slots of a 16-group 2 adjacent lanes,
// so block and group reductions are one or two shuffles.
__device__ __forceinline__ void store_slot(const PhaseParams& p, int s, bool live, const float v[8], const Act& A) {
  float amax8 = 0.f;
#pragma unroll
  for (int i = 0; i < 8; i++) amax8 = fmaxf(amax8, fabsf(v[i]));
  if (p.need_q6) {
    const float amax = fmaxf(amax8, __shfl_xor_sync(0xffffffffu, amax8, 1));
    const uint32_t e = (__float_as_uint(amax) >> 23) & 0xFF;
    const bool ok = e >= 22 && e < 255;  // groups below 2^-105 contribute nothing
    const float f = ok ? __uint_as_float((275u - e) << 23) : 0.f;       // 2^(22-E)
    const float invf = ok ? __uint_as_float((e - 21u) << 23) : 0.f;     // 2^(E-22)
    uint32_t w0[2] = {0, 0}, w1[2] = {0, 0}, w2[2] = {0, 0};
    int xsum16 = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int X = __float2int_rn(v[i] * f);  // exact scaling, |X| <= 2^22
      xsum16 += X;
      w0[i >> 2] |= (uint32_t)(X & 255) << (8 * (i & 3));
      w1[i >> 2] |= (uint32_t)((X >> 8) & 255) << (8 * (i & 3));
      w2[i >> 2] |= (uint32_t)((X >> 16) & 255) << (8 * (i & 3));
    }
    xsum16 += __shfl_xor_sync(0xffffffffu, xsum16, 1);
    if (live) {
      const int pos = limb_pos(8 * s);
      *reinterpret_cast<uint2*>(A.l0 + pos) = make_uint2(w0[0], w0[1]);
      *reinterpret_cast<uint2*>(A.l1 + pos) = make_uint2(w1[0], w1[1]);
      *reinterpret_cast<uint2*>(A.l2 + pos) = make_uint2(w2[0], w2[1]);
      if ((s & 1) == 0) A.lp[s >> 1] = make_float2(32.0f * (float)xsum16, invf);
    }
  }
  if (p.need_q8) {
    float amax = fmaxf(amax8, __shfl_xor_sync(0xffffffffu, amax8, 1));
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
      reinterpret_cast<uint2*>(A.xq)[s] = pk;
      if ((s & 3) == 0) { A.xs[s >> 2] = sc; A.xsum[s >> 2] = sum; }
    }
  }
}

// Activation build. ACT_RMS (K <= 8 * RMS_SLOTS * consumer threads): the
// norm weights are already in registers (loaded before the dependency wait)
// and one block reduction gives the rms scale.
static __device__ void build_activation(const PhaseParams& p, const float wpre[RMS_SLOTS][8], const Act& A, float* red) {
  const int K = p.n_in, nsb = K >> 5, nslot = K >> 3;
  const int t = threadIdx.x - 32, nt = CONSUMER_WARPS * 32;
  const int lane = t & 31, w = t >> 5;
  if (p.act == ACT_Q8) {
    const int4* src = reinterpret_cast<const int4*>(p.xq);
    int4* dst = reinterpret_cast<int4*>(A.xq);
    for (int i = t; i < K / 16; i += nt) dst[i] = src[i];
    for (int i = t; i < nsb; i += nt) A.xs[i] = p.xs[i];
    consumers_sync();
    for (int b = w; b < nsb; b += CONSUMER_WARPS) {
      const int s = warp_isum((int)A.xq[32 * b + lane]);
      if (lane == 0) A.xsum[b] = s;
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
        const float4 a = __ldcg(x4 + 2 * s), b = __ldcg(x4 + 2 * s + 1);
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
      store_slot(p, s, s < nslot, v[j], A);
    }
  } else {
    // up to F32_BATCH slots per thread loaded before any is used: one L2
    // round trip per batch instead of one per slot
    constexpr int F32_BATCH = 4;
    for (int s0 = 0; s0 < nslot; s0 += F32_BATCH * nt) {
      float v[F32_BATCH][8];
#pragma unroll
      for (int j = 0; j < F32_BATCH; j++) {
        const int s = s0 + j * nt + t;
        if (s < nslot) {
          const float4 a = __ldcg(x4 + 2 * s), b = __ldcg(x4 + 2 * s + 1);
          v[j][0] = a.x; v[j][1] = a.y; v[j][2] = a.z; v[j][3] = a.w;
          v[j][4] = b.x; v[j][5] = b.y; v[j][6] = b.z; v[j][7] = b.w;
        } else {
#pragma unroll
          for (int i = 0; i < 8; i++) v[j][i] = 0.f;
        }
      }
#pragma unroll
      for (int j = 0; j < F32_BATCH; j++) {
        if (s0 + j * nt >= nslot) break;  // uniform: no live slot for any thread
        const int s = s0 + j * nt + t;
        store_slot(p, s, s < nslot, v[j], A);
      }
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

// NR rows (4, or 2 for phases with few rows per CTA: half the latency of a
// unit); acc[NR..3] stay 0.
template <int NR = 4>
__device__ __forceinline__ void q4k_unit(const uint8_t* st, int rstride, int nrows, int m, const Q4X& X,
                                         float acc[4]) {
  const int lane = threadIdx.x & 31, bl = lane >> 2, g = lane & 3;
#pragma unroll
  for (int r = 0; r < 4; r++) acc[r] = 0.f;
  if (bl >= m) return;
  // all four rows' loads first (rows past nrows re-read row 0, result unused)
  uint4 hd[NR], q0[NR], q1[NR];
#pragma unroll
  for (int r = 0; r < NR; r++) {
    const uint8_t* blk = st + (r < nrows ? r : 0) * rstride + bl * Q4K_BYTES;
    hd[r] = *reinterpret_cast<const uint4*>(blk);
    q0[r] = *reinterpret_cast<const uint4*>(blk + 16 + 32 * g);
    q1[r] = *reinterpret_cast<const uint4*>(blk + 32 + 32 * g);
  }
  const int shf = 16 * (g & 1);  // scale bytes of j = 2g, 2g+1 within their words
  const bool low = g < 2;        // j < 4: plain 6-bit fields (src/quant.c:59-61)
#pragma unroll
  for (int r = 0; r < NR; r++) {
    const uint32_t qw[8] = {q0[r].x, q0[r].y, q0[r].z, q0[r].w, q1[r].x, q1[r].y, q1[r].z, q1[r].w};
    int ia = 0, ib = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      ia = __dp4a((int)(qw[i] & 0x0F0F0F0Fu), X.a[i], ia);
      ib = __dp4a((int)((qw[i] >> 4) & 0x0F0F0F0Fu), X.b[i], ib);
    }
    const float d = half_bits_to_float(hd[r].x), dmin = half_bits_to_float(hd[r].x >> 16);
    // get_scale_min_k4 (src/quant.c:57-66) for j = 2g, 2g+1, branch-free:
    // scales[0..3] in hd.y, [4..7] in hd.z, [8..11] in hd.w
    const uint32_t Y = hd[r].y >> shf, Z = hd[r].z >> shf, W = hd[r].w >> shf;
    const uint32_t Y1 = Y >> 8, Z1 = Z >> 8, W1 = W >> 8;
    const int sa = low ? (Y & 63) : ((W & 15) | ((Y >> 2) & 0x30));
    const int ma = low ? (Z & 63) : (((W >> 4) & 15) | ((Z >> 2) & 0x30));
    const int sb = low ? (Y1 & 63) : ((W1 & 15) | ((Y1 >> 2) & 0x30));
    const int mb = low ? (Z1 & 63) : (((W1 >> 4) & 15) | ((Z1 >> 2) & 0x30));
    // xs * (d*(s*iqx) - dmin*(m*ix)): the integer products are exact
    // (|s*iqx| <= 63*32*15*127 < 2^22) and become floats by exponent bias
    float a = X.xsa * (d * i22_to_float(sa * ia) - dmin * i22_to_float(ma * X.sma));
    a += X.xsb * (d * i22_to_float(sb * ib) - dmin * i22_to_float(mb * X.smb));
    acc[r] = r < nrows ? a : 0.f;
  }
}

// Q6_K: two passes of 4 blocks. Lane (bq = lane/8, n = half, k = quarter) of
// block bl = 4*pass + bq owns ql[64n + 16k .. +16]: low nibbles are elements
// 128n + 16k + i (scale group 8n + k), high nibbles 128n + 64 + 16k + i (group
// 8n + 4 + k); their two high bits sit in qh[32n + 16(k&1) + i] at bits 0/2
// and 4/6 — the element map of dequant_q6_K (src/quant.c:94-123).
struct Q6L {
  uint4 l0[2][2], l1[2][2], l2[2][2];  // [pass][lo/hi group]
  float2 lp[2][2];
};

__device__ __forceinline__ void q6l_load(const Act& A, int c, int nb, Q6L& X) {
  const int lane = threadIdx.x & 31, bq = lane >> 3, n = (lane >> 2) & 1, k = lane & 3;
#pragma unroll
  for (int pass = 0; pass < 2; pass++) {
    const int b = min(CHUNK_BLOCKS * c + 4 * pass + bq, nb - 1);
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int e = 256 * b + 128 * n + 64 * h + 16 * k;  // first element of the lane's group
      const int pos = limb_pos(e);
      X.l0[pass][h] = *reinterpret_cast<const uint4*>(A.l0 + pos);
      X.l1[pass][h] = *reinterpret_cast<const uint4*>(A.l1 + pos);
      X.l2[pass][h] = *reinterpret_cast<const uint4*>(A.l2 + pos);
      X.lp[pass][h] = A.lp[e >> 4];
    }
  }
}

// sum over 16 codes of q * X for one limb plane: 4 dp4a
__device__ __forceinline__ int dot16u(const uint32_t q[4], const uint4& l) {
  unsigned r = __dp4a(q[0], l.x, 0u);
  r = __dp4a(q[1], l.y, r);
  r = __dp4a(q[2], l.z, r);
  r = __dp4a(q[3], l.w, r);
  return (int)r;
}
__device__ __forceinline__ int dot16s(const uint32_t q[4], const uint4& l) {
  int r = __dp4a((int)q[0], (int)l.x, 0);
  r = __dp4a((int)q[1], (int)l.y, r);
  r = __dp4a((int)q[2], (int)l.z, r);
  r = __dp4a((int)q[3], (int)l.w, r);
  return r;
}

// sum((q - 32) * X) of one 16-group from its three limb dot products; the
// partial sums are exact integers below 2^22, the combine is fp32
__device__ __forceinline__ float group_dot(const uint32_t q[4], const uint4& l0, const uint4& l1, const uint4& l2,
                                           float xs32) {
  const float s0 = i22_to_float(dot16u(q, l0));
  const float s1 = i22_to_float(dot16u(q, l1));
  const float s2 = i22_to_float(dot16s(q, l2));
  return fmaf(s2, 65536.0f, fmaf(s1, 256.0f, s0)) - xs32;
}

template <int NR = 4>
__device__ __forceinline__ void q6k_unit(const uint8_t* st, int rstride, int nrows, int m, const Q6L& X,
                                         float acc[4]) {
  const int lane = threadIdx.x & 31, bq = lane >> 3, n = (lane >> 2) & 1, k = lane & 3;
  const int sh_lo = (k < 2) ? 0 : 2, sh_hi = (k < 2) ? 4 : 6;
#pragma unroll
  for (int r = 0; r < 4; r++) acc[r] = 0.f;
#pragma unroll
  for (int pass = 0; pass < 2; pass++) {
    const int bl = 4 * pass + bq;
    if (bl >= m) continue;
    uint4 ql[NR], qh[NR];
    uint2 sc[NR];
    float d[NR];
#pragma unroll
    for (int r = 0; r < NR; r++) {  // rows past nrows re-read row 0, result unused
      const uint8_t* chunk = st + (r < nrows ? r : 0) * rstride;
      const uint8_t* body = chunk + bl * Q6K_BODY;
      ql[r] = *reinterpret_cast<const uint4*>(body + 64 * n + 16 * k);
      qh[r] = *reinterpret_cast<const uint4*>(body + 128 + 32 * n + 16 * (k & 1));
      sc[r] = *reinterpret_cast<const uint2*>(body + 192 + 8 * n);
      d[r] = __half2float(*reinterpret_cast<const __half*>(chunk + m * Q6K_BODY + 2 * bl));
    }
#pragma unroll
    for (int r = 0; r < NR; r++) {
      const uint32_t lw[4] = {ql[r].x, ql[r].y, ql[r].z, ql[r].w};
      const uint32_t hw[4] = {qh[r].x, qh[r].y, qh[r].z, qh[r].w};
      uint32_t qlo[4], qhi[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        qlo[i] = (lw[i] & 0x0F0F0F0Fu) | (((hw[i] >> sh_lo) << 4) & 0x30303030u);
        qhi[i] = ((lw[i] >> 4) & 0x0F0F0F0Fu) | (((hw[i] >> sh_hi) << 4) & 0x30303030u);
      }
      const float tlo = group_dot(qlo, X.l0[pass][0], X.l1[pass][0], X.l2[pass][0], X.lp[pass][0].x);
      const float thi = group_dot(qhi, X.l0[pass][1], X.l1[pass][1], X.l2[pass][1], X.lp[pass][1].x);
      // scales: sc[8n + k] is byte k of word 0 of this half, sc[8n + 4 + k] byte k of word 1
      const float sl = (float)(int8_t)(sc[r].x >> (8 * k)), sh = (float)(int8_t)(sc[r].y >> (8 * k));
      const float v = d[r] * (sl * X.lp[pass][0].y * tlo + sh * X.lp[pass][1].y * thi);
      acc[r] += r < nrows ? v : 0.f;
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

// key: where the argmax epilogue folds its pick (null: p.argmax_key).
static __device__ void epilogue(const PhaseParams& p, const SegRange* sr, const float* part, float* red, int pos,
                         unsigned long long* key = nullptr) {
  if (!key) key = p.argmax_key;
  const int t = threadIdx.x - 32, nt = CONSUMER_WARPS * 32;
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
          const float2 rr = rope_rotate(x0, x1, cs.x, cs.y);
          const float r0 = rr.x, r1 = rr.y;
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
          case EPI_RESID: S.out[row] = __ldcg(S.out + row) + v; break;
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
  if (key) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if ((t & 31) == 0 && best) atomicMax(key, best);
  }
}

}  // namespace hakm
