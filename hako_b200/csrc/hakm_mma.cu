// hakm_mma.cu — Q4_K x q8_32 matmul on the 5th-generation tensor cores
// (tcgen05.mma kind::i8), for batches of activations (batched decode,
// prompt processing).
//
// out[n][r] = q4k_vec_dot(row r, xq[n], xs[n]) with the arithmetic of the
// reference as built (src/quant.c:150-232 under gcc -O3 -ffast-math with
// FMA): per pair of 32-element sub-blocks (A, B) = (2g, 2g+1) of a
// super-block with scales d, dmin and 6-bit (s, m) per sub-block,
//   t  = fma(s, fl(d * isum), -fl(m * fl(dmin * ix)))   for A and B,
//   acc = acc + fma(tB, xsB, tA * xsA),
// pairs in order along the row, where isum = sum(q * xq) over the sub-block
// (q the 4-bit weight codes) and ix = sum(xq). The per-sub-block integer
// sums come from the tensor cores, exact (int32 accumulators in tensor
// memory, one fresh accumulator per sub-block: K = 32 per MMA); the fp32
// steps run in the epilogue warps, about eleven packed (f32x2) operations
// per two outputs and sub-block pair, and, not the MMA, bound the kernel.
// The row is never split along K (the sum order is the row's order).
//
// CTA tile: 128 weight rows x BN activations, the whole K. Warp roles:
//   warp 0      producer: per 256-element super-block one 2-D tensor copy of
//               the tile's 128 raw Q4_K blocks (144 B each), 16 copies of
//               the activation codes (16-byte K slices, so the slices land
//               in the tensor cores' K-major core-matrix layout), one copy
//               of the activation scales; a ring of 2-3 such stages and a
//               ring of 2 converted stages, mbarriers between the roles.
//   warp 1      allocates tensor memory; one lane issues the MMAs (one per
//               sub-block into one of 512/BN accumulator buffers) and
//               commits them to mbarriers.
//   warps 2-5   converters (thread = row): unpack the nibbles into int8 A
//               tiles in the core-matrix layout, the row's d, dmin and
//               (s, m) per sub-block as floats, and per activation the code
//               sums ix and the scales transposed to [sub-block][n].
//   warps 6-13  epilogue: warp w reads tensor-memory lanes 32*(w%4).. (its
//               rows) and half of the columns, accumulates the fp32 result
//               in registers, and writes out + bias at the end.
// Every wait is bounded; a timeout sets the error flag and the CTA winds
// down (all issued MMAs and copies complete before tensor memory is freed
// and the CTA exits).
#include "hakm_gemv.cuh"
#include "hakm_tmap.h"

#include <atomic>

namespace hakm {

constexpr int MM_ROWS = 128;
constexpr int MM_CONV = 128;          // converter threads (one row each)
constexpr int MM_THREADS = 14 * 32;  // producer, MMA, 4 converter and 8 epilogue warps; 128 registers
constexpr int MM_RAW = MM_ROWS * Q4K_BYTES;  // 18,432
constexpr int MM_A = MM_ROWS * QK;           // 32,768: 8 sub-blocks x 4 KB
// per row: d, -1.5*2^23*d, dmin, s[8], -m[8] as [19][128] floats
constexpr int MM_SC_D = 0, MM_SC_DNEG = 1, MM_SC_DMIN = 2, MM_SC_S = 3, MM_SC_NM = 11;
constexpr int MM_SC = 19 * MM_ROWS * 4;
constexpr uint32_t MM_BIAS = 0x4B400000u;    // bits of 1.5 * 2^23 (see the epilogue)

template <int BN>
struct MmaLayout {
  // ring of tensor copies: raw Q4_K blocks; activation codes as two
  // 128-byte K blocks [2][BN][128 B] in the 128-byte swizzle (the tensor
  // copy writes it, the MMA descriptor reads it); scales [BN][8]. 1 KB
  // aligned (the swizzle atom).
  static constexpr int B = BN * QK, XS = BN * 8 * 4;
  static constexpr int T_RAW = 0, T_B = MM_RAW, T_XS = T_B + B;
  static constexpr int TX = T_XS + XS;  // bytes the copies deliver per stage
  static constexpr int T_STAGE = (TX + 1023) & ~1023;
  // ring of converted operands: A tiles, row scales, activation scales and sums [8][BN + 4]
  static constexpr int XP = BN + 4;
  static constexpr int C_A = 0, C_SC = MM_A, C_XT = C_SC + MM_SC, C_STAGE = C_XT + 2 * 8 * XP * 4;
  // rings as deep as fit: converted stages first (the MMAs and the epilogue
  // trail the converters), then copies; two super-blocks of accumulators
  static_assert(BN == 16 || BN == 32, "the epilogue takes whole sub-block pairs per tensor-memory round trip");
  static constexpr int NT = 3, NC = 3;
  static constexpr int NBUF = 16;                       // accumulator buffers in tensor memory
  static constexpr int TMEM_COLS = NBUF * BN;           // 256 or 512
  static constexpr int HC = BN / 2;                     // columns per epilogue warp
  static constexpr int LDC = HC;                        // columns per tensor-memory load
  // 1 KB of alignment slack, 1 KB header, the two rings
  static constexpr size_t SMEM = 2048 + (size_t)NT * T_STAGE + (size_t)NC * C_STAGE;
  static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
  static_assert((2 * NT + 2 * NC + 2 * NBUF) * 8 <= 1000, "mbarriers before the tensor-memory slot");
};

struct MmaArgs {
  float* out;   // [n_batch][n_out]
  const float* bias;
  int* err_flag;
  int n_out, n_in, n_batch;
};


// Shared-memory matrix descriptor, K-major. No swizzle (layout 0): core
// matrices of 8 rows x 16 bytes (rows 16 B apart); lbo = bytes between the
// two 16-byte K halves of a 32-byte K step, sbo = bytes between 8-row
// groups. 128-byte swizzle (layout 2): rows of 128 bytes, 16-byte chunks
// permuted by row % 8; sbo = 1024 (8 rows), lbo unused (16); a K step
// inside the 128 bytes advances the start address by 32 bytes.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout = 0) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

// Instruction descriptor: D s32, A and B s8, both K-major, M = 128, N = BN.
template <int BN>
__host__ __device__ constexpr uint32_t mma_idesc() {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(MM_ROWS >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Loads without the wait (several in flight, then tmem_wait_ld).
template <int N>
__device__ __forceinline__ void tmem_ld_issue(uint32_t taddr, uint32_t* r) {
  if constexpr (N == 8) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
  }
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Bounded wait that also gives up once another role has failed; the thread
// sleeps in the barrier between tests.
__device__ __forceinline__ bool mm_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > WAIT_LIMIT) {
      *abort = 1;
      return false;
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(MM_THREADS, 1)
    q4k_mma_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ CUtensorMap smap, const __grid_constant__ MmaArgs a) {
  using L = MmaLayout<BN>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // the 128-byte swizzle needs 1 KB aligned stages
  uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  uint64_t* t_full = reinterpret_cast<uint64_t*>(smem);  // [NT] copies landed
  uint64_t* t_free = t_full + L::NT;                      // [NT] converters + MMAs done with the copies
  uint64_t* c_full = t_free + L::NT;                      // [NC] converted operands ready
  uint64_t* c_free = c_full + L::NC;                      // [NC] MMAs + epilogue done with them
  uint64_t* d_full = c_free + L::NC;                      // [NBUF] accumulator ready
  uint64_t* d_empty = d_full + L::NBUF;                   // [NBUF] accumulator read and reset
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 1000);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + 1004);
  uint8_t* tring = smem + 1024;
  uint8_t* cring = tring + L::NT * L::T_STAGE;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * MM_ROWS, n0 = blockIdx.y * BN;
  const int nsb = a.n_in / QK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::NT; i++) {
      mbar_init(smem_addr(&t_full[i]), 1);
      mbar_init(smem_addr(&t_free[i]), MM_CONV + 1);
    }
    for (int i = 0; i < L::NC; i++) {
      mbar_init(smem_addr(&c_full[i]), MM_CONV);
      mbar_init(smem_addr(&c_free[i]), 1 + 8);
    }
    for (int i = 0; i < L::NBUF; i++) {
      mbar_init(smem_addr(&d_full[i]), 1);
      mbar_init(smem_addr(&d_empty[i]), 8);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(L::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();  // activations come from the preceding kernel

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int b = 0;
      for (; b < nsb; b++) {
        const int s = b % L::NT;
        if (b >= L::NT && !mm_wait(smem_addr(&t_free[s]), ((b / L::NT) - 1) & 1, abort)) break;
        uint8_t* st = tring + s * L::T_STAGE;
        const uint32_t bar = smem_addr(&t_full[s]);
        const int g = b;
        mbar_expect_tx(bar, L::TX);
        tma_2d_stream(smem_addr(st + L::T_RAW), &wmap, g * (Q4K_BYTES / 8), row0, bar);
        tma_2d(smem_addr(st + L::T_B), &xmap, g * QK, n0, bar);
        tma_2d(smem_addr(st + L::T_B + BN * 128), &xmap, g * QK + 128, n0, bar);
        tma_2d(smem_addr(st + L::T_XS), &smap, g * 8, n0, bar);
      }
      // the copies in flight land before the CTA may exit
      for (int j = (b > L::NT ? b - L::NT : 0); j < b; j++) {
        const uint32_t bar = smem_addr(&t_full[j % L::NT]);
        const long long t0 = clock64();
        while (!mbar_try_wait(bar, (j / L::NT) & 1) && clock64() - t0 < WAIT_LIMIT) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = mma_idesc<BN>();
      int q = 0, issued = 0;
      for (int b = 0; b < nsb; b++) {
        const int ts = b % L::NT, cs = b % L::NC;
        if (!mm_wait(smem_addr(&c_full[cs]), (b / L::NC) & 1, abort)) break;
        tc_fence_after();
        const uint8_t* tst = tring + ts * L::T_STAGE;
        const uint8_t* cst = cring + cs * L::C_STAGE;
        bool ok = true;
        for (int j = 0; j < 8; j++, q++) {
          const int buf = q % L::NBUF;
          // phase 0 of d_empty: the epilogue's start-up arrival
          if (!mm_wait(smem_addr(&d_empty[buf]), (q / L::NBUF) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = smem_desc(smem_addr(cst + L::C_A + j * 4096), 2048, 128);
          const uint64_t bd = smem_desc(smem_addr(tst + L::T_B + (j >> 2) * BN * 128 + (j & 3) * 32), 16, 1024, 2);
          mma_i8(tmem + buf * BN, ad, bd, idesc, 0u);
          mma_commit(smem_addr(&d_full[buf]));
          issued = q + 1;
        }
        if (!ok) break;
        mma_commit(smem_addr(&t_free[ts]));  // activation codes read
        mma_commit(smem_addr(&c_free[cs]));  // A tiles read
      }
      // every MMA issued has completed before tensor memory is released
      if (issued > 0) {
        const int last = issued - 1, buf = last % L::NBUF;
        const long long t0 = clock64();
        while (!mbar_try_wait(smem_addr(&d_full[buf]), (last / L::NBUF) & 1) && clock64() - t0 < WAIT_LIMIT) {
        }
      }
    }
  } else if (warp < 6) {
    // ---------------- converters ----------------
    const int t0 = threadIdx.x - 64;  // row of the tile
    for (int b = 0; b < nsb; b++) {
      const int ts = b % L::NT, cs = b % L::NC;
      if (!mm_wait(smem_addr(&t_full[ts]), (b / L::NT) & 1, abort)) break;
      if (b >= L::NC && !mm_wait(smem_addr(&c_free[cs]), ((b / L::NC) - 1) & 1, abort)) break;
      const uint8_t* tst = tring + ts * L::T_STAGE;
      uint8_t* cst = cring + cs * L::C_STAGE;
      const int t = t0;
      const uint8_t* blk = tst + L::T_RAW + t * Q4K_BYTES;
      // all of the row's block first (nine 16-byte loads in flight)
      uint4 q[9];
#pragma unroll
      for (int i = 0; i < 9; i++) q[i] = reinterpret_cast<const uint4*>(blk)[i];
      const uint4 hd = q[0];
      uint8_t* A = cst + L::C_A + (t >> 3) * 128 + (t & 7) * 16;
#pragma unroll
      for (int g = 0; g < 4; g++) {
        const uint4 q0 = q[1 + 2 * g], q1 = q[2 + 2 * g];
        const uint4 lo0 = make_uint4(q0.x & 0x0F0F0F0Fu, q0.y & 0x0F0F0F0Fu, q0.z & 0x0F0F0F0Fu, q0.w & 0x0F0F0F0Fu);
        const uint4 lo1 = make_uint4(q1.x & 0x0F0F0F0Fu, q1.y & 0x0F0F0F0Fu, q1.z & 0x0F0F0F0Fu, q1.w & 0x0F0F0F0Fu);
        const uint4 hi0 = make_uint4((q0.x >> 4) & 0x0F0F0F0Fu, (q0.y >> 4) & 0x0F0F0F0Fu, (q0.z >> 4) & 0x0F0F0F0Fu,
                                     (q0.w >> 4) & 0x0F0F0F0Fu);
        const uint4 hi1 = make_uint4((q1.x >> 4) & 0x0F0F0F0Fu, (q1.y >> 4) & 0x0F0F0F0Fu, (q1.z >> 4) & 0x0F0F0F0Fu,
                                     (q1.w >> 4) & 0x0F0F0F0Fu);
        // sub-block 2g: low nibbles; 2g+1: high nibbles (src/quant.c:74-90)
        *reinterpret_cast<uint4*>(A + (2 * g) * 4096) = lo0;
        *reinterpret_cast<uint4*>(A + (2 * g) * 4096 + 2048) = lo1;
        *reinterpret_cast<uint4*>(A + (2 * g + 1) * 4096) = hi0;
        *reinterpret_cast<uint4*>(A + (2 * g + 1) * 4096 + 2048) = hi1;
      }
      // the row's scales (get_scale_min_k4, src/quant.c:57-66); the 12
      // scale bytes are hd.y, hd.z, hd.w
      const float d = half_bits_to_float(hd.x), dmin = half_bits_to_float(hd.x >> 16);
      const uint32_t sw[3] = {hd.y, hd.z, hd.w};
      float* ds = reinterpret_cast<float*>(cst + L::C_SC);
      ds[MM_SC_D * MM_ROWS + t] = d;
      ds[MM_SC_DNEG * MM_ROWS + t] = -12582912.0f * d;  // exact: d has 11 significant bits
      ds[MM_SC_DMIN * MM_ROWS + t] = dmin;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        auto byte = [&](int i) { return (int)((sw[i >> 2] >> (8 * (i & 3))) & 0xFF); };
        int sv, mv;
        if (j < 4) {
          sv = byte(j) & 63;
          mv = byte(j + 4) & 63;
        } else {
          sv = (byte(j + 4) & 15) | ((byte(j - 4) >> 6) << 4);
          mv = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
        }
        ds[(MM_SC_S + j) * MM_ROWS + t] = (float)sv;
        ds[(MM_SC_NM + j) * MM_ROWS + t] = -(float)mv;
      }
      // per activation and sub-block: code sum and scale, as [j][n] rows of BN + 4
      const float* xs_in = reinterpret_cast<const float*>(tst + L::T_XS);
      float* xs_t = reinterpret_cast<float*>(cst + L::C_XT);
      float* ix_t = xs_t + 8 * L::XP;
      for (int p = t0; p < 8 * BN; p += MM_CONV) {
        const int j = p / BN, n = p - j * BN;
        // 16-byte chunks 2(j%4), 2(j%4)+1 of row n of K block j/4, swizzled
        const uint8_t* rowp = tst + L::T_B + (j >> 2) * BN * 128 + n * 128;
        const int ch = 2 * (j & 3);
        const uint4 c0 = *reinterpret_cast<const uint4*>(rowp + ((ch ^ (n & 7)) << 4));
        const uint4 c1 = *reinterpret_cast<const uint4*>(rowp + (((ch + 1) ^ (n & 7)) << 4));
        int sum = 0;
        sum = __dp4a((int)c0.x, 0x01010101, sum);
        sum = __dp4a((int)c0.y, 0x01010101, sum);
        sum = __dp4a((int)c0.z, 0x01010101, sum);
        sum = __dp4a((int)c0.w, 0x01010101, sum);
        sum = __dp4a((int)c1.x, 0x01010101, sum);
        sum = __dp4a((int)c1.y, 0x01010101, sum);
        sum = __dp4a((int)c1.z, 0x01010101, sum);
        sum = __dp4a((int)c1.w, 0x01010101, sum);
        ix_t[j * L::XP + n] = (float)sum;
      }
      for (int p = t0; p < 8 * BN; p += MM_CONV) {
        const int n = p >> 3, j = p & 7;
        xs_t[j * L::XP + n] = xs_in[p];
      }
      // generic-proxy writes of the A tiles become visible to the tensor cores
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(smem_addr(&c_full[cs]));
      mbar_arrive(smem_addr(&t_free[ts]));  // raw blocks, codes and scales read
    }
  } else {
    // ---------------- epilogue ----------------
    // A result word w is isum (|isum| < 2^22); 1.5*2^23 + isum is exact as
    // the float with bits 0x4B400000 + w, and fma(that, d, -1.5*2^23*d) is
    // the correctly rounded d*isum. G sub-blocks (whole pairs) share one
    // round trip to tensor memory (G x HC = 32 result words a thread);
    // columns go two at a time through the packed fp32 operations.
    constexpr int HC = L::HC, LDC = L::LDC, G = 32 / HC;
    static_assert(G % 2 == 0, "sub-block pairs");
    const int quad = warp & 3, half = (warp - 6) >> 2;
    const int r = 32 * quad + lane;  // tile row = tensor-memory lane
    const uint32_t lane_base = (uint32_t)(32 * quad) << 16;
    // phase 0 of every d_empty: the buffers start free
    if (lane == 0)
      for (int buf = 0; buf < L::NBUF; buf++) mbar_arrive(smem_addr(&d_empty[buf]));
    float2 acc[HC / 2];
#pragma unroll
    for (int c = 0; c < HC / 2; c++) acc[c] = make_float2(0.f, 0.f);
    bool ok = true;
    int q = 0;
    for (int b = 0; b < nsb && ok; b++) {
      const int cs = b % L::NC;
      const uint8_t* cst = cring + cs * L::C_STAGE;
      const float* ds = reinterpret_cast<const float*>(cst + L::C_SC);
      const float* xs_t = reinterpret_cast<const float*>(cst + L::C_XT);
      const float* ix_t = xs_t + 8 * L::XP;
      // the converters' writes for this stage are visible
      if (!mm_wait(smem_addr(&c_full[cs]), (b / L::NC) & 1, abort)) break;
      const float d = ds[MM_SC_D * MM_ROWS + r], dneg = ds[MM_SC_DNEG * MM_ROWS + r];
      const float dmin = ds[MM_SC_DMIN * MM_ROWS + r];
      const float2 d2 = make_float2(d, d), dneg2 = make_float2(dneg, dneg), dmin2 = make_float2(dmin, dmin);
      for (int j0 = 0; j0 < 8; j0 += G, q += G) {
        for (int g = 0; g < G && ok; g++)
          if (!mm_wait(smem_addr(&d_full[(q + g) % L::NBUF]), ((q + g) / L::NBUF) & 1, abort)) ok = false;
        if (!ok) break;
        tc_fence_after();
        uint32_t v[G * HC];
#pragma unroll
        for (int g = 0; g < G; g++)
          tmem_ld_issue<LDC>(tmem + lane_base + ((q + g) % L::NBUF) * BN + half * HC, &v[g * HC]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
          for (int g = 0; g < G; g++) mbar_arrive(smem_addr(&d_empty[(q + g) % L::NBUF]));
#pragma unroll
        for (int g = 0; g < G; g += 2) {
          const int jA = j0 + g, jB = jA + 1;
          const float sA = ds[(MM_SC_S + jA) * MM_ROWS + r], nmA = ds[(MM_SC_NM + jA) * MM_ROWS + r];
          const float sB = ds[(MM_SC_S + jB) * MM_ROWS + r], nmB = ds[(MM_SC_NM + jB) * MM_ROWS + r];
          const float2 sA2 = make_float2(sA, sA), nmA2 = make_float2(nmA, nmA);
          const float2 sB2 = make_float2(sB, sB), nmB2 = make_float2(nmB, nmB);
#pragma unroll
          for (int c4 = 0; c4 < HC / 4; c4++) {
            const int c = half * HC + 4 * c4;
            const float4 xA = *reinterpret_cast<const float4*>(xs_t + jA * L::XP + c);
            const float4 iA = *reinterpret_cast<const float4*>(ix_t + jA * L::XP + c);
            const float4 xB = *reinterpret_cast<const float4*>(xs_t + jB * L::XP + c);
            const float4 iB = *reinterpret_cast<const float4*>(ix_t + jB * L::XP + c);
#pragma unroll
            for (int e = 0; e < 2; e++) {
              const int k = 4 * c4 + 2 * e;
              const float2 xsA = e ? make_float2(xA.z, xA.w) : make_float2(xA.x, xA.y);
              const float2 ixA = e ? make_float2(iA.z, iA.w) : make_float2(iA.x, iA.y);
              const float2 xsB = e ? make_float2(xB.z, xB.w) : make_float2(xB.x, xB.y);
              const float2 ixB = e ? make_float2(iB.z, iB.w) : make_float2(iB.x, iB.y);
              const float2 wA = make_float2(__uint_as_float(MM_BIAS + v[g * HC + k]),
                                            __uint_as_float(MM_BIAS + v[g * HC + k + 1]));
              const float2 wB = make_float2(__uint_as_float(MM_BIAS + v[(g + 1) * HC + k]),
                                            __uint_as_float(MM_BIAS + v[(g + 1) * HC + k + 1]));
              const float2 tA = fma2(sA2, fma2(wA, d2, dneg2), mul2(nmA2, mul2(dmin2, ixA)));
              const float2 tB = fma2(sB2, fma2(wB, d2, dneg2), mul2(nmB2, mul2(dmin2, ixB)));
              acc[k / 2] = add2(acc[k / 2], fma2(tB, xsB, mul2(tA, xsA)));
            }
          }
        }
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&c_free[cs]));  // scales of this stage read
    }
    const int row = row0 + r;
    if (ok && row < a.n_out) {
      const float bv = a.bias ? __ldg(a.bias + row) : 0.f;
#pragma unroll
      for (int c = 0; c < HC; c++) {
        const int n = n0 + half * HC + c;
        const float y = (c & 1) ? acc[c / 2].y : acc[c / 2].x;
        if (n < a.n_batch) a.out[(size_t)n * a.n_out + row] = a.bias ? __fadd_rn(y, bv) : y;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TMEM_COLS) : "memory");
  }
  if (threadIdx.x == 0 && *abort && a.err_flag) atomicExch(a.err_flag, 1);
}

// ------------------------------------------------------------------ host

namespace {

// Activation tile width: 32 when the 32-wide tiles already give every SM a
// CTA, else 16 (twice the CTAs; the weight tile is then read twice, the
// second time mostly from L2).
int mma_bn(int n_out, int n_batch, int num_sms) {
  const int row_tiles = (n_out + MM_ROWS - 1) / MM_ROWS;
  return n_batch > 16 && row_tiles * ((n_batch + 31) / 32) >= num_sms ? 32 : 16;
}

template <int BN>
cudaError_t launch_mma_bn(const uint8_t* w, const int8_t* xq, const float* xs, const MmaArgs& a, cudaStream_t st) {
  using L = MmaLayout<BN>;
  CUtensorMap wm, xm, sm;
  const uint64_t rowB = (uint64_t)(a.n_in / QK) * Q4K_BYTES;
  if (!encode_tmap_2d(&wm, CU_TENSOR_MAP_DATA_TYPE_UINT64, w, rowB / 8, (uint64_t)a.n_out, rowB, Q4K_BYTES / 8, MM_ROWS) ||
      !encode_tmap_2d(&xm, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, (uint64_t)a.n_in, (uint64_t)a.n_batch, (uint64_t)a.n_in, 128,
                 BN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&sm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, xs, (uint64_t)(a.n_in / 32), (uint64_t)a.n_batch,
                 (uint64_t)(a.n_in / 32) * 4, 8, BN))
    return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> ready{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(ready.load() & bit)) {
    e = cudaFuncSetAttribute(q4k_mma_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::SMEM);
    if (e != cudaSuccess) return e;
    ready.fetch_or(bit);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a.n_out + MM_ROWS - 1) / MM_ROWS), (unsigned)((a.n_batch + BN - 1) / BN), 1);
  cfg.blockDim = dim3(MM_THREADS);
  cfg.dynamicSmemBytes = L::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, q4k_mma_kernel<BN>, wm, xm, sm, a);
}

}  // namespace

// Tensor-core batched Q4_K matmul; activation tiles of 16 or 32.
cudaError_t launch_q4k_mma(float* out, const uint8_t* w, const int8_t* xq, const float* xs, const float* bias,
                           int n_out, int n_in, int n_batch, int* err_flag, int num_sms, cudaStream_t st) {
  if (n_out <= 0 || n_batch <= 0 || n_in <= 0 || n_in % QK) return cudaErrorInvalidValue;
  MmaArgs a = {};
  a.out = out;
  a.bias = bias;
  a.err_flag = err_flag;
  a.n_out = n_out;
  a.n_in = n_in;
  a.n_batch = n_batch;
  return mma_bn(n_out, n_batch, num_sms) == 32 ? launch_mma_bn<32>(w, xq, xs, a, st)
                                               : launch_mma_bn<16>(w, xq, xs, a, st);
}

}  // namespace hakm
