// hakm_gemv.cuh — device building blocks of the streaming GEMV phases, shared
// by the per-phase kernel (hakm_stream.cu) and the persistent decode-step
// kernel (hakm_step.cu): bulk-copy / mbarrier helpers, per-CTA row schedule,
// the activation prologue (rmsnorm, int8 q8_32 codes, the fp32 activation by
// lane class), the Q4_K and Q6_K units and the fused epilogues, all with the
// reference's own roundings (hakm_exact.cuh).
//
// Activations produced by other SMs earlier in the same kernel are read with
// L2-coherent loads (__ldcg): L1 is not coherent across SMs.
#pragma once
#include "hakm_device.cuh"
#include "hakm_exact.cuh"

namespace hakm {


constexpr int CONSUMER_WARPS = 11;  // 12 warps in all: at most 168 registers a thread, no spills
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
// Per-warp shared scratch of the units (Q4_K: 4 x 36 floats of pair values
// being handed to the row chains; Q6_K: 4 rows x 16 (d*sc, d*sc) pairs).
constexpr int WARP_SCRATCH_FLOATS = 160;
constexpr int WARP_SCRATCH_BYTES = CONSUMER_WARPS * WARP_SCRATCH_FLOATS * 4;

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
// 2-D tiled tensor copy (no multicast) of the box at (x, y) into shared memory.
__device__ __forceinline__ void tma_2d(uint32_t dst, const void* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// Weight rows are read once per token: these copies carry an L2
// evict-first policy, so that the stream does not push what is reused out
// of L2 (the kernel's own code, exchanged vectors, K/V rows, norm weights,
// activations that other CTAs read). tma_2d_stream is tma_2d with it.
__device__ __forceinline__ void tma_2d_stream(uint32_t dst, const void* map, int x, int y, uint32_t bar) {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(pol)
      : "memory");
}

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

// The fp32 activation "by lane class": class l holds x[8t + l], t = 0 ..
// K/8 - 1, the element order in which the reference's vectorized Q6_K dot
// feeds lane l of its accumulator (src/nn.c:92). Within each aligned group
// of four positions the middle two are swapped (t0, t2, t1, t3), so one
// 16-byte read gives the packed-fp32 operand pairs (t0, t2) and (t1, t3).
// The pitch is padded by 4 floats so the 8 classes' 16-byte reads of a warp
// fall in distinct banks.
__host__ __device__ inline int cls_pitch(int K) { return K / 8 + 4; }
__host__ __device__ inline int cls_slot(int t) { return (t & ~3) | ((t & 1) << 1) | ((t >> 1) & 1); }

// Shared-memory bytes of the activation for an n_in of K: the int8 codes,
// scales and code sums of q8_32 (Q4_K rows), and the fp32 activation by lane
// class (Q6_K rows; an rmsnorm prologue also keeps its squares there).
__host__ __device__ inline size_t act_bytes(int K, bool q8, bool f32) {
  size_t b = 0;
  if (f32) b += (size_t)8 * cls_pitch(K) * 4;
  if (q8) b += (size_t)K + (size_t)(K / 32) * 8;
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
  const size_t act = act_bytes(nb * QK, true, true) + 8192 + WARP_SCRATCH_BYTES;
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
// remainders of consecutive segments land on different CTAs. One result per
// row: a unit runs whole rows, every chunk, in order.
// 32-bit arithmetic throughout (groups * grid < 2^31): this runs in every
// CTA at the start of every phase, on the critical path.
__device__ __forceinline__ void cta_ranges(const PhaseParams& p, SegRange* sr) {
  const unsigned grid = gridDim.x, cta = blockIdx.x;
  unsigned goff = 0;
  int pbase = 0;
  for (int s = 0; s < p.n_seg; s++) {
    const int n = p.seg[s].n_rows;
    const unsigned G = (unsigned)(n + 3) / 4;
    const unsigned idx = (cta + grid - goff % grid) % grid;
    const int g0 = (int)(idx * G / grid), g1 = (int)((idx + 1) * G / grid);
    sr[s].row0 = 4 * g0;
    sr[s].row1 = min(4 * g1, n);
    sr[s].wdelta = 0;
    sr[s].part_base = pbase;
    pbase += sr[s].row1 - sr[s].row0;
    goff += G;
  }
}

// ------------------------------------------------------------------ prologue

// The activation in shared memory, in the two forms the row types consume:
//  q8 (Q4_K rows): per-32 int8 codes xq, scales xs and code sums xsum —
//     quantize_row_q8_32 as the reference builds it (src/quant.c:127-144).
//  xc (Q6_K rows): the fp32 activation by lane class (cls_pitch).
struct Act {
  int8_t* xq;
  float* xs;
  int* xsum;
  float* xc;
  int cp;  // class pitch (floats)
};

__device__ __forceinline__ Act carve_act(uint8_t* base, int K, bool q8, bool f32) {
  Act a = {};
  uint8_t* p = base;
  a.cp = cls_pitch(K);
  if (f32) {
    a.xc = reinterpret_cast<float*>(p);
    p += (size_t)8 * a.cp * 4;
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

// 8-element slot s (elements [8s, 8s+8)): element 8s + i is position s of
// class i. For q8 the 4 slots of a 32-block are 4 adjacent lanes, so the
// block reductions are two shuffles.
__device__ __forceinline__ void store_slot(const PhaseParams& p, int s, bool live, const float v[8], const Act& A) {
  if (p.need_q6 && live) {
    const int ts = cls_slot(s);
#pragma unroll
    for (int i = 0; i < 8; i++) A.xc[i * A.cp + ts] = v[i];
  }
  if (p.need_q8) {
    float amax8 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax8 = fmaxf(amax8, fabsf(v[i]));
    float amax = fmaxf(amax8, __shfl_xor_sync(0xffffffffu, amax8, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float sc = __fmul_rn(amax, 1.0f / 127.0f);
    const float inv = q8_inv(amax, sc);
    int q[8], sum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) { q[i] = q8_round(__fmul_rn(v[i], inv)); sum += q[i]; }
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

// rmsnorm's scale (src/nn.c:14-16 as built) of the squares sq (by lane class,
// pitch cp, K elements): lane chains l = 0..7 of sum(x*x) over t, folded,
// then ss/K + eps and the rsqrtss Newton step. Run by one full warp; every
// lane returns the scale.
__device__ __forceinline__ float rms_scale(const float* sq, int cp, int K, float eps, const uint32_t* rsq) {
  const int lane = threadIdx.x & 31, l = lane & 7, nt = K / 8;
  float acc = 0.f;
  if (lane < 8) {
    // float4 w holds positions (4t, 4t+2, 4t+1, 4t+3). The chain is 4 adds a
    // float4; groups of RG float4 are loaded one group ahead, so the shared
    // loads' latency hides behind the previous group's adds
    constexpr int RG = 4;
    const float4* row = reinterpret_cast<const float4*>(sq + l * cp);
    const int n4 = nt / 4, ng = n4 / RG;
    auto add4 = [&](const float4& w) {
      acc = __fadd_rn(acc, w.x); acc = __fadd_rn(acc, w.z);
      acc = __fadd_rn(acc, w.y); acc = __fadd_rn(acc, w.w);
    };
    if (ng > 0) {
      float4 cur[RG];
#pragma unroll
      for (int i = 0; i < RG; i++) cur[i] = row[i];
      for (int g = 1; g < ng; g++) {
        float4 nxt[RG];
#pragma unroll
        for (int i = 0; i < RG; i++) nxt[i] = row[RG * g + i];
#pragma unroll
        for (int i = 0; i < RG; i++) add4(cur[i]);
#pragma unroll
        for (int i = 0; i < RG; i++) cur[i] = nxt[i];
      }
#pragma unroll
      for (int i = 0; i < RG; i++) add4(cur[i]);
    }
    for (int t = RG * ng; t < n4; t++) add4(row[t]);
  }
  const float ss = fold8_lanes(acc);
  return rsqrt_nr(__fadd_rn(__fdiv_rn(ss, (float)K), eps), rsq);
}

// Activation build. ACT_RMS (K <= 8 * RMS_SLOTS * consumer threads): the
// norm weights are already in registers (loaded before the dependency wait);
// the squares go to the class region, one warp takes the scale, then
// y = (x * w) * scale (src/nn.c:17 as built).
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
#pragma unroll
    for (int j = 0; j < RMS_SLOTS; j++) {
      const int s = t + j * nt;
      if (s < nslot) {
        const float4 a = __ldcg(x4 + 2 * s), b = __ldcg(x4 + 2 * s + 1);
        v[j][0] = a.x; v[j][1] = a.y; v[j][2] = a.z; v[j][3] = a.w;
        v[j][4] = b.x; v[j][5] = b.y; v[j][6] = b.z; v[j][7] = b.w;
        const int ts = cls_slot(s);
#pragma unroll
        for (int i = 0; i < 8; i++) A.xc[i * A.cp + ts] = __fmul_rn(v[j][i], v[j][i]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; i++) v[j][i] = 0.f;
      }
    }
    consumers_sync();
    if (w == 0) {
      const float sc = rms_scale(A.xc, A.cp, K, p.eps, p.rsq);
      if (lane == 0) red[0] = sc;
    }
    consumers_sync();
    const float scale = red[0];
#pragma unroll
    for (int j = 0; j < RMS_SLOTS; j++) {
      const int s = t + j * nt;
      if (j * nt >= nslot) break;  // uniform: no live slot for any thread
#pragma unroll
      for (int i = 0; i < 8; i++) v[j][i] = __fmul_rn(__fmul_rn(v[j][i], wpre[j][i]), scale);
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
  return __fsub_rn(__int_as_float(0x4B400000 + v), 12582912.0f);
}

// Q4_K: lane (bl = lane/4, g = lane%4) owns qs bytes [32g, 32g+32) of block bl
// of the chunk: low nibbles are sub-block 2g (A), high nibbles sub-block 2g+1
// (B) (src/quant.c:163-229). The lane's activation slice of one chunk (64
// int8 codes, two scales, two code sums) fits in registers.
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

// The lane's term of each of NR rows (rows past nrows re-read row 0, result
// unused; lanes of blocks past m give 0, unused): per pair of sub-blocks
// (A, B) of a super-block, q4k_vec_dot as built (src/quant.c:228-231 under
// -O3 -ffast-math with FMA):
//   tA = fma(sA, d*iqxA, -(mA*(dmin*ixA)))     tB likewise
//   v  = fma(tB, xsB, tA*xsA)
// which the row's running sum then takes with one rounded add (q4k_chain).
// The integer sums are exact dp4a results.
// Sum of the four products of unsigned bytes of a with signed bytes of b,
// plus c (PTX dp4a.u32.s32).
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

template <int NR = 4>
__device__ __forceinline__ void q4k_pairs(const uint8_t* st, int rstride, int nrows, int m, const Q4X& X,
                                          float v[4]) {
  const int lane = threadIdx.x & 31, bl = lane >> 2, g = lane & 3;
#pragma unroll
  for (int r = 0; r < 4; r++) v[r] = 0.f;
  if (bl >= m) return;
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
  const float fxa = i22_to_float(X.sma), fxb = i22_to_float(X.smb);
#pragma unroll
  for (int r = 0; r < NR; r++) {
    const uint32_t qw[8] = {q0[r].x, q0[r].y, q0[r].z, q0[r].w, q1[r].x, q1[r].y, q1[r].z, q1[r].w};
    // exact integer sums, in two independent chains each (shorter
    // dependency chains); the high nibbles stay in place (16 * q) through
    // an unsigned x signed dp4a and the sum is divided by 16 at the end
    int ia0 = 0, ia1 = 0, ib0 = 0, ib1 = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      ia0 = __dp4a((int)(qw[i] & 0x0F0F0F0Fu), X.a[i], ia0);
      ia1 = __dp4a((int)(qw[i + 4] & 0x0F0F0F0Fu), X.a[i + 4], ia1);
      ib0 = dp4a_us(qw[i] & 0xF0F0F0F0u, X.b[i], ib0);
      ib1 = dp4a_us(qw[i + 4] & 0xF0F0F0F0u, X.b[i + 4], ib1);
    }
    const int ia = ia0 + ia1, ib = (ib0 + ib1) >> 4;
    const float d = half_bits_to_float(hd[r].x), dmin = half_bits_to_float(hd[r].x >> 16);
    // get_scale_min_k4 (src/quant.c:57-66) for j = 2g, 2g+1, branch-free:
    // scales[0..3] in hd.y, [4..7] in hd.z, [8..11] in hd.w
    const uint32_t Y = hd[r].y >> shf, Z = hd[r].z >> shf, W = hd[r].w >> shf;
    const uint32_t Y1 = Y >> 8, Z1 = Z >> 8, W1 = W >> 8;
    const int sa = low ? (Y & 63) : ((W & 15) | ((Y >> 2) & 0x30));
    const int ma = low ? (Z & 63) : (((W >> 4) & 15) | ((Z >> 2) & 0x30));
    const int sb = low ? (Y1 & 63) : ((W1 & 15) | ((Y1 >> 2) & 0x30));
    const int mb = low ? (Z1 & 63) : (((W1 >> 4) & 15) | ((Z1 >> 2) & 0x30));
    const float2 p = mul2(make_float2(d, d), make_float2(i22_to_float(ia), i22_to_float(ib)));
    const float2 mq = mul2(make_float2(i22_to_float(ma), i22_to_float(mb)),
                           mul2(make_float2(dmin, dmin), make_float2(fxa, fxb)));
    const float2 tt = fma2(make_float2(i22_to_float(sa), i22_to_float(sb)), p, make_float2(-mq.x, -mq.y));
    const float vv = __fmaf_rn(tt.y, X.xsb, __fmul_rn(tt.x, X.xsa));
    v[r] = r < nrows ? vv : 0.f;
  }
}

// Continues rows 0..3's running sums (lanes 0..3 hold them in `acc`) with
// the pair terms of one chunk, pair 0 (lane 0) first: the terms go through
// the warp's scratch tr (4 x 36 floats) to the row lanes.
__device__ __forceinline__ float q4k_chain(const float v[4], int m, float acc, float* tr) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
#pragma unroll
  for (int r = 0; r < 4; r++) tr[r * 36 + lane] = v[r];
  __syncwarp();
  if (lane < 4) {
    const float4* row = reinterpret_cast<const float4*>(tr + lane * 36);
    for (int j = 0; j < m; j++) {
      const float4 w = row[j];
      acc = __fadd_rn(acc, w.x); acc = __fadd_rn(acc, w.y);
      acc = __fadd_rn(acc, w.z); acc = __fadd_rn(acc, w.w);
    }
  }
  return acc;
}

// Whole Q4_K rows: st points at the unit's first row (all chunks), rows
// rstride bytes apart. Lanes 0..nrows-1 return their row's dot product.
template <int NR = 4>
__device__ __forceinline__ float q4k_rows(const uint8_t* st, int rstride, int nrows, int nb, const Act& A, float* tr) {
  float acc = 0.f;
  const int nch = n_chunks(nb);
  for (int c = 0; c < nch; c++) {
    const int m = q6_chunk_blocks(nb, c);
    const Q4X X = q4x_load(A.xq, A.xs, A.xsum, c, nb);
    float v[4];
    q4k_pairs<NR>(st + (size_t)c * Q4K_CHUNK, rstride, nrows, m, X, v);
    acc = q4k_chain(v, m, acc, tr);
  }
  return acc;
}

// Whole Q6_K rows x the fp32 activation as the reference's generic path
// computes them (src/nn.c:84-95 as built): lane l of the 8-lane accumulator
// adds the rounded products w[i] * x[i] of the elements i = 8t + l one at a
// time in increasing t; the 8 lanes fold at the end (fold8_lanes). Here
// thread (r, l) = (lane / 8, lane % 8) runs that chain for row r over the
// whole row, reading its class's code bytes (device body layout,
// hakm_internal.h) and x by class (Act::xc). w = (q - 32) * (d * sc) is
// exact in fp32 (at most 6 + 18 significant bits), as in dequant_q6_K.
// The products go in pairs (packed fp32) over positions (t0, t2), (t1, t3)
// of each group of four; the next block's bytes load while this one is
// worked. Lanes 8r (r < nrows) return row r's dot product.
struct Q6Blk {
  uint2 w0, w1, w2;  // the class's 24 code bytes
  uint4 sc;          // the 16 int8 scales
  uint32_t dh;       // fp16 d
};
// Block j of a chunk of m blocks, class l's code bytes.
__device__ __forceinline__ Q6Blk q6_blk_load_chunk(const uint8_t* chunk, int m, int j, int l) {
  const uint8_t* body = chunk + j * Q6K_BODY;
  const uint2* wp = reinterpret_cast<const uint2*>(body + 24 * l);
  Q6Blk B;
  B.w0 = wp[0];
  B.w1 = wp[1];
  B.w2 = wp[2];
  B.sc = *reinterpret_cast<const uint4*>(body + 192);
  B.dh = *reinterpret_cast<const uint16_t*>(chunk + m * Q6K_BODY + 2 * j);
  return B;
}
__device__ __forceinline__ Q6Blk q6_blk_load(const uint8_t* row, int nb, int b, int l) {
  const int c = b >> 3;
  return q6_blk_load_chunk(row + (size_t)c * Q6K_CHUNK, q6_chunk_blocks(nb, c), b & 7, l);
}
// float(v) of byte k of w as a signed int8, without a conversion instruction
__device__ __forceinline__ float s8_val(uint32_t w, int k) {
  return __uint_as_float(__byte_perm(w ^ 0x80808080u, 0x4B000000u, 0x7650u | (uint32_t)k)) - 8388736.0f;
}

// The 16 products of half n of a block, in chain order (positions
// 16n + 4k + b for k, b = 0..3): w = (q - 32) * (d * sc) exact, times x.
__device__ __forceinline__ void q6_half_products(const Q6Blk& B, int n, const float* xh, float p[16]) {
  const float2 bias2 = make_float2(-8388640.0f, -8388640.0f);  // -(2^23 + 32)
  const float d = half_bits_to_float(B.dh);
  const float2 dd = make_float2(d, d);
  const uint32_t W0 = n ? B.w1.y : B.w0.x, W1 = n ? B.w2.x : B.w0.y, WH = n ? B.w2.y : B.w1.x;
  const uint32_t scw0 = n ? B.sc.z : B.sc.x, scw1 = n ? B.sc.w : B.sc.y;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    uint32_t q;
    if (k == 0) q = (W0 & 0x0F0F0F0Fu) | ((WH << 4) & 0x30303030u);
    else if (k == 1) q = (W1 & 0x0F0F0F0Fu) | ((WH << 2) & 0x30303030u);
    else if (k == 2) q = ((W0 >> 4) & 0x0F0F0F0Fu) | (WH & 0x30303030u);
    else q = ((W1 >> 4) & 0x0F0F0F0Fu) | ((WH >> 2) & 0x30303030u);
    // groups g = 8n + 2k (codes b = 0, 1) and g + 1 (b = 2, 3): bytes
    // 2(k&1), 2(k&1)+1 of scale word 2n + k/2
    const uint32_t sw = (k >> 1) ? scw1 : scw0;
    const float2 ds = mul2(make_float2(s8_val(sw, 2 * (k & 1)), s8_val(sw, 2 * (k & 1) + 1)), dd);
    // x at positions (b0, b2, b1, b3) of this group of four
    const float4 x4 = *reinterpret_cast<const float4*>(xh + 4 * k);
    const float2 q02 = add2(make_float2(__uint_as_float(__byte_perm(q, 0x4B000000u, 0x7650)),
                                        __uint_as_float(__byte_perm(q, 0x4B000000u, 0x7652))), bias2);
    const float2 q13 = add2(make_float2(__uint_as_float(__byte_perm(q, 0x4B000000u, 0x7651)),
                                        __uint_as_float(__byte_perm(q, 0x4B000000u, 0x7653))), bias2);
    const float2 p02 = mul2(mul2(q02, ds), make_float2(x4.x, x4.y));
    const float2 p13 = mul2(mul2(q13, ds), make_float2(x4.z, x4.w));
    p[4 * k + 0] = p02.x;
    p[4 * k + 1] = p13.x;
    p[4 * k + 2] = p02.y;
    p[4 * k + 3] = p13.y;
  }
}

// NRL = 1: the chain runs one half-block behind the products, so each
// half's 16 products are formed while the previous half's are being added.
// NRL = 2: a lane runs the chains of two rows (r and r + 4 of an 8-row
// unit), their adds interleaved so one chain's add latency hides behind the
// other's (no half-block lag: it would not fit the registers); for phases
// with many rows per CTA (the lm_head). out[i] of lanes 8r is row
// (r + 4i)'s dot product.
template <int NRL>
__device__ __forceinline__ void q6k_rows(const uint8_t* st, int rstride, int nrows, int nb, const Act& A,
                                         float out[NRL]) {
  const int lane = threadIdx.x & 31, r = lane >> 3, l = lane & 7;
  const float* xl = A.xc + l * A.cp;
  if constexpr (NRL == 1) {
    // the loop body has no branch, so the scheduler can interleave each
    // half's adds with the next half's products (the last block is peeled)
    const uint8_t* row = st + (size_t)(r < nrows ? r : 0) * rstride;
    float acc = 0.f;
    Q6Blk B = q6_blk_load(row, nb, 0, l);
    float pv[16];
    q6_half_products(B, 0, xl, pv);
    int b = 0;
    for (; b + 1 < nb; b++) {
      float pc[16];
      q6_half_products(B, 1, xl + 32 * b + 16, pc);
      B = q6_blk_load(row, nb, b + 1, l);
#pragma unroll
      for (int i = 0; i < 16; i++) acc = __fadd_rn(acc, pv[i]);
      q6_half_products(B, 0, xl + 32 * (b + 1), pv);
#pragma unroll
      for (int i = 0; i < 16; i++) acc = __fadd_rn(acc, pc[i]);
    }
    {
      float pc[16];
      q6_half_products(B, 1, xl + 32 * b + 16, pc);
#pragma unroll
      for (int i = 0; i < 16; i++) acc = __fadd_rn(acc, pv[i]);
#pragma unroll
      for (int i = 0; i < 16; i++) acc = __fadd_rn(acc, pc[i]);
    }
    out[0] = fold8_lanes(acc);
  } else {
    const uint8_t* row0 = st + (size_t)(r < nrows ? r : 0) * rstride;
    const uint8_t* row1 = st + (size_t)(r + 4 < nrows ? r + 4 : 0) * rstride;
    float a0 = 0.f, a1 = 0.f;
    Q6Blk B0 = q6_blk_load(row0, nb, 0, l), B1 = q6_blk_load(row1, nb, 0, l);
    for (int b = 0; b < nb; b++) {
#pragma unroll
      for (int n = 0; n < 2; n++) {
        float p0[16], p1[16];
        q6_half_products(B0, n, xl + 32 * b + 16 * n, p0);
        q6_half_products(B1, n, xl + 32 * b + 16 * n, p1);
        if (n == 1 && b + 1 < nb) {
          B0 = q6_blk_load(row0, nb, b + 1, l);
          B1 = q6_blk_load(row1, nb, b + 1, l);
        }
#pragma unroll
        for (int i = 0; i < 16; i++) {
          a0 = __fadd_rn(a0, p0[i]);
          a1 = __fadd_rn(a1, p1[i]);
        }
      }
    }
    out[0] = fold8_lanes(a0);
    out[1] = fold8_lanes(a1);
  }
}

// Chunk c of the unit's rows (rows rstride bytes apart, each holding only
// that chunk: a chunk-streamed stage) continues the lane's chain `acc`, in
// the order and with the roundings of q6k_rows<1>; the caller folds the
// lanes after the last chunk.
__device__ __forceinline__ float q6k_rows_chunk(const uint8_t* st, int rstride, int nrows, int nb, int c,
                                                const Act& A, float acc) {
  const int lane = threadIdx.x & 31, r = lane >> 3, l = lane & 7;
  const uint8_t* chunk = st + (size_t)(r < nrows ? r : 0) * rstride;
  const int m = q6_chunk_blocks(nb, c);
  const float* xl = A.xc + l * A.cp + 32 * CHUNK_BLOCKS * c;
  Q6Blk B = q6_blk_load_chunk(chunk, m, 0, l);
  float pv[16];
  q6_half_products(B, 0, xl, pv);
  int j = 0;
  for (; j + 1 < m; j++) {
    float pc[16];
    q6_half_products(B, 1, xl + 32 * j + 16, pc);
    B = q6_blk_load_chunk(chunk, m, j + 1, l);
#pragma unroll
    for (int i = 0; i < 16; i++) acc = __fadd_rn(acc, pv[i]);
    q6_half_products(B, 0, xl + 32 * (j + 1), pv);
#pragma unroll
    for (int i = 0; i < 16; i++) acc = __fadd_rn(acc, pc[i]);
  }
  float pc[16];
  q6_half_products(B, 1, xl + 32 * j + 16, pc);
#pragma unroll
  for (int i = 0; i < 16; i++) acc = __fadd_rn(acc, pv[i]);
#pragma unroll
  for (int i = 0; i < 16; i++) acc = __fadd_rn(acc, pc[i]);
  return acc;
}

// ------------------------------------------------------------------ epilogue

__device__ __forceinline__ float row_total(const float* part, const SegRange& r, int row) {
  return part[r.part_base + (row - r.row0)];
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
          S.out[dr >> 1] = swiglu_exact(a0, a1);
        } else {
          const float x0 = S.bias ? __fadd_rn(a0, S.bias[dr]) : a0;
          const float x1 = S.bias ? __fadd_rn(a1, S.bias[dr + 1]) : a1;
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
          case EPI_STORE: S.out[row] = S.bias ? __fadd_rn(v, S.bias[row]) : v; break;
          case EPI_RESID: S.out[row] = __fadd_rn(__ldcg(S.out + row), v); break;
          case EPI_V_CACHE: {
            const float o = S.bias ? __fadd_rn(v, S.bias[row]) : v;
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
