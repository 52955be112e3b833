// hakm_batch.cu — Q4_K x q8_32 matmul for a batch of activations.
//
// out[n][r] = q4k_vec_dot(w row r, xq[n], xs[n]) (+ bias[r]) (src/quant.c:150-232)
// for n < n_batch. Every weight byte is read from HBM once per launch and
// used for all (up to 16) activations of the launch, so the HBM cost stays
// that of one vector while the dp4a work grows with the batch.
//
// Work unit = (32-row tile t, 8-block chunk c): 36,864 weight bytes, moved
// by ONE 2-D tensor copy (cp.async.bulk.tensor, tensor map over the rows as
// 8-byte elements; rows and chunk columns past the matrix are zero-filled,
// which contributes exact zeros). Units are ordered chunk-major
// (u = c * n_tiles + t) and each CTA of a persistent grid takes a contiguous
// range, so a CTA sees at most a couple of chunks and keeps their activation
// slices (int8 codes, scales, per-32 code sums) in shared memory for its
// whole range.
//
//   warp 0      producer: one tensor copy per unit into a ring of up to 6
//               slots (as many as fit beside the activation slices),
//               completion on the slot's mbarrier (bounded waits).
//   warps 1..8  consumers: warp w owns rows 4(w-1)..4(w-1)+3 of every tile.
//               Lane (block bl = lane/4, quarter g = lane%4) unpacks the
//               nibbles of sub-blocks 2g and 2g+1 of block bl for its four
//               rows once, then for each activation: 16 dp4a per row and
//               xs*((d*s)*iqx - (dmin*m)*ix) per sub-block (the reference's
//               order of the scale products; d*s and dmin*m are exact in
//               fp32). The 4 x 8 per-lane partials of eight activations are
//               summed over the warp by a transposing butterfly (31
//               shuffles: lane l ends with the total of value l).
//
// Rows of a single chunk are written directly. Otherwise each chunk's
// partial per (row, activation) goes to global memory and a second kernel,
// launched as a programmatic dependent of the first (its launch overlaps the
// first's tail; griddepcontrol.wait orders the reads), sums the chunks in
// order and adds the bias: deterministic for any grid, and no fence or
// ticket in the streaming kernel.
#include "hakm_gemv.cuh"
#include "hakm_tmap.h"

#include <atomic>

namespace hakm {

constexpr int BT_WARPS = 8;                              // consumer warps
constexpr int BT_THREADS = 32 * (BT_WARPS + 1);
constexpr int BT_ROWS = 4 * BT_WARPS;                    // rows per tile
constexpr int BT_MAX_STAGES = 6;  // ring slots: as many as fit beside the activation slices
constexpr int BT_STAGE_BYTES = BT_ROWS * Q4K_CHUNK;      // 36,864
constexpr int BT_ACT_CHUNK = 2048 + 64 * 4 + 64 * 4;     // codes, xs, code sums of one chunk
constexpr int BT_ACT_SLOTS = 32;                         // activations x chunks held per CTA
constexpr int BT_HEADER = 128;
constexpr int BT_BAR = 2;                                // named barrier of the consumers
constexpr int BT_MAX_NB = 16;                            // activations per launch

struct BatchArgs {
  float* out;          // [n_batch][n_out]
  float* part;         // chunk order: [nch][n_batch][n_out]; tile order: [n_tiles][pmax][n_batch][32]
  int* ticket;         // tile order: [n_tiles * BT_WARPS], zero before the launch; left zero
  int* err_flag;       // set on a timed-out wait (may be null)
  const int8_t* xq;    // [n_batch][n_in]
  const float* xs;     // [n_batch][n_in / 32]
  const float* bias;   // [n_out] or null
  int n_out, n_in, n_batch, nch, n_tiles, n_units, span, n_stages;
  int tile_order;      // 1: units tile-major, every chunk's activation held; 0: chunk-major
  int pmax;            // tile order: most CTAs sharing one tile
};

// CTA whose unit range [n_units*b/grid, n_units*(b+1)/grid) holds unit u.
__device__ __forceinline__ int cta_of_unit(int u, int n_units) {
  return (int)((((long long)u + 1) * gridDim.x + n_units - 1) / n_units) - 1;
}

__device__ __forceinline__ void consumers_sync_bt() {
  asm volatile("bar.sync %0, %1;" ::"n"(BT_BAR), "n"(BT_WARPS * 32) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(pol)
      : "memory");
}

// Sum of v[i] over the 32 lanes for every i < V (V a power of two <= 32):
// butterfly steps on the lane bits >= log2(V) add whole vectors; the steps
// below halve the vector, each lane keeping the half its lane bit selects.
// Lane l ends with the total of value (l mod V) in v[0].
template <int V>
__device__ __forceinline__ float warp_transpose_sum(float (&v)[V]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    if (s >= V) {
#pragma unroll
      for (int i = 0; i < V; i++) v[i] += __shfl_xor_sync(0xffffffffu, v[i], s);
    } else {
      const bool up = (lane & s) != 0;
#pragma unroll
      for (int i = 0; i < s; i++) {
        const float send = up ? v[i] : v[i + s];
        const float keep = up ? v[i + s] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
      }
    }
  }
  return v[0];
}

// Tile order: the warp's four rows of tile t are complete for this CTA's
// chunks of t. A tile held by one CTA is written out; otherwise the CTA's
// piece goes to the partial buffer and the warp completing the tile's last
// piece (ticket, reset by that warp) sums the pieces in CTA order.
template <int NB, int NBB>
__device__ __forceinline__ void tile_flush(const BatchArgs& a, int t, int cw, int lane, int rsub, int nsub,
                                           float (&tot)[NB / NBB]) {
  constexpr int V = 4 * NBB;
  const int b0 = cta_of_unit(t * a.nch, a.n_units), b1 = cta_of_unit(t * a.nch + a.nch - 1, a.n_units);
  const int row = t * BT_ROWS + 4 * cw + rsub;
  if (b0 == b1) {
#pragma unroll
    for (int q = 0; q < NB / NBB; q++) {
      const int n = q * NBB + nsub;
      if (lane < V && row < a.n_out && n < a.n_batch)
        a.out[(size_t)n * a.n_out + row] = tot[q] + (a.bias ? __ldg(a.bias + row) : 0.f);
      tot[q] = 0.f;
    }
    return;
  }
  const int p = blockIdx.x - b0;
  float* piece = a.part + (size_t)(t * a.pmax + p) * a.n_batch * BT_ROWS;
#pragma unroll
  for (int q = 0; q < NB / NBB; q++) {
    const int n = q * NBB + nsub;
    if (lane < V && n < a.n_batch) piece[n * BT_ROWS + 4 * cw + rsub] = tot[q];
    tot[q] = 0.f;
  }
  __threadfence();
  __syncwarp();
  int prev = 0;
  if (lane == 0) prev = atomicAdd(a.ticket + t * BT_WARPS + cw, 1);
  prev = __shfl_sync(0xffffffffu, prev, 0);
  if (prev != b1 - b0) return;
  __threadfence();
  const float* pieces = a.part + (size_t)t * a.pmax * a.n_batch * BT_ROWS;
  for (int j = lane; j < 4 * a.n_batch; j += 32) {
    const int r = 4 * cw + (j & 3), n = j >> 2, rr = t * BT_ROWS + r;
    if (rr >= a.n_out) continue;
    float s = 0.f;
    for (int q = 0; q <= b1 - b0; q++) s += __ldcg(pieces + ((size_t)q * a.n_batch + n) * BT_ROWS + r);
    a.out[(size_t)n * a.n_out + rr] = s + (a.bias ? __ldg(a.bias + rr) : 0.f);
  }
  if (lane == 0) a.ticket[t * BT_WARPS + cw] = 0;
}

template <int NB>
__global__ void __launch_bounds__(BT_THREADS, 1)
    q4k_batch_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ BatchArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + BT_MAX_STAGES;
  uint8_t* ring = smem + BT_HEADER;
  const int S = a.n_stages;
  uint8_t* actb = ring + S * BT_STAGE_BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u0 = (int)((long long)a.n_units * blockIdx.x / gridDim.x);
  const int u1 = (int)((long long)a.n_units * (blockIdx.x + 1) / gridDim.x);
  const int c_first = a.tile_order ? 0 : u0 / a.n_tiles;
  // dependents (the chunk-sum kernel, the next call) may launch; each waits
  // for this grid before it reads what this grid writes
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      mbar_init(smem_addr(&full[i]), 1);
      mbar_init(smem_addr(&empty[i]), BT_WARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  bool failed = false;

  if (warp == 0) {
    // ---------------- producer ----------------
    int i = 0;
    for (int u = u0; u < u1; u++, i++) {
      const int slot = i % S;
      if (i >= S) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait(smem_addr(&empty[slot]), ((i / S) - 1) & 1);
        if (!__shfl_sync(0xffffffffu, ok, 0)) { failed = true; break; }
      }
      if (lane == 0) {
        int c, t;
        if (a.tile_order) { t = u / a.nch; c = u - t * a.nch; } else { c = u / a.n_tiles; t = u - c * a.n_tiles; }
        mbar_expect_tx(smem_addr(&full[slot]), BT_STAGE_BYTES);
        tma_load_2d(smem_addr(ring + slot * BT_STAGE_BYTES), &wmap, c * (Q4K_CHUNK / 8), t * BT_ROWS,
                    smem_addr(&full[slot]));
      }
      __syncwarp();
    }
    // every copy this CTA issued lands before the CTA exits
    if (lane == 0)
      for (int j = (i > S ? i - S : 0); j < i; j++)
        if (!mbar_wait(smem_addr(&full[j % S]), (j / S) & 1)) failed = true;
  } else {
    // ---------------- consumers ----------------
    const int ct = threadIdx.x - 32, cw = warp - 1;
    // the preceding kernel's outputs (activations) and reads (of out) are
    // settled before the consumers touch either; weights are constant, so
    // the producer streams them already
    pdl_wait();
    // activation slices of chunks c_first .. c_first + span - 1: per
    // (activation, chunk) 2048 codes, 64 scales, 64 code sums; zeros past
    // n_in and past n_batch
    const int nsb = a.n_in / 32;
    for (int j = ct; j < NB * a.span * 64; j += BT_WARPS * 32) {
      const int n = j / (a.span * 64), rem = j - n * a.span * 64, cc = rem >> 6, sb = rem & 63;
      const int e = (c_first + cc) * 2048 + 32 * sb;  // first element of the 32-block
      uint8_t* ab = actb + (n * a.span + cc) * BT_ACT_CHUNK;
      int4 q0 = make_int4(0, 0, 0, 0), q1 = q0;
      float s = 0.f;
      if (n < a.n_batch && e < a.n_in) {
        const int4* src = reinterpret_cast<const int4*>(a.xq + (size_t)n * a.n_in + e);
        q0 = __ldg(src);
        q1 = __ldg(src + 1);
        s = __ldg(a.xs + (size_t)n * nsb + e / 32);
      }
      int sum = 0;
      const int w8[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
      for (int k = 0; k < 8; k++) sum = __dp4a(w8[k], 0x01010101, sum);
      // 32-block sb = 8*bl + 2*g + h feeds lane L = 4*bl + g as its int4s
      // 2h and 2h+1; int4 k of lane L sits at (32*k + L)*16, so each of the
      // consumer's four 16-byte loads reads 512 contiguous bytes
      const int L = sb >> 1, h = sb & 1;
      int4* dst = reinterpret_cast<int4*>(ab);
      dst[32 * (2 * h) + L] = q0;
      dst[32 * (2 * h + 1) + L] = q1;
      reinterpret_cast<float*>(ab + 2048)[sb] = s;
      reinterpret_cast<int*>(ab + 2048 + 256)[sb] = sum;
    }
    consumers_sync_bt();

    constexpr int NBB = NB < 8 ? NB : 8;  // activations per butterfly
    constexpr int V = 4 * NBB;
    const int bl = lane >> 2, g = lane & 3;
    const int shf = 16 * (g & 1);
    const bool low = g < 2;
    float tot[NB / NBB];  // tile order: this tile's running sum (lane's row and activation per block)
#pragma unroll
    for (int q = 0; q < NB / NBB; q++) tot[q] = 0.f;
    const int rsub = (lane & (V - 1)) / NBB, nsub = (lane & (V - 1)) % NBB;
    int cur_t = -1;
    int i = 0;
    for (int u = u0; u < u1; u++, i++) {
      int c, t;
      if (a.tile_order) { t = u / a.nch; c = u - t * a.nch; } else { c = u / a.n_tiles; t = u - c * a.n_tiles; }
      if (a.tile_order && t != cur_t) {
        if (cur_t >= 0) tile_flush<NB, NBB>(a, cur_t, cw, lane, rsub, nsub, tot);
        cur_t = t;
      }
      const int slot = i % S;
      if (!mbar_wait(smem_addr(&full[slot]), (i / S) & 1)) failed = true;
      if (__any_sync(0xffffffffu, failed)) { failed = true; break; }
      // the four rows' nibbles and scale products, once per unit
      uint32_t lo[4][8], hi[4][8];
      float ds_a[4], ds_b[4], dm_a[4], dm_b[4];
      const uint8_t* st = ring + slot * BT_STAGE_BYTES + (4 * cw) * Q4K_CHUNK + bl * Q4K_BYTES;
#pragma unroll
      for (int r = 0; r < 4; r++) {
        const uint8_t* blk = st + r * Q4K_CHUNK;
        const uint4 hd = *reinterpret_cast<const uint4*>(blk);
        const uint4 q0 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * g);
        const uint4 q1 = *reinterpret_cast<const uint4*>(blk + 32 + 32 * g);
        const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int k = 0; k < 8; k++) {
          lo[r][k] = qw[k] & 0x0F0F0F0Fu;
          hi[r][k] = (qw[k] >> 4) & 0x0F0F0F0Fu;
        }
        const float d = half_bits_to_float(hd.x), dmin = half_bits_to_float(hd.x >> 16);
        // get_scale_min_k4 (src/quant.c:57-66) for sub-blocks 2g, 2g+1
        const uint32_t Y = hd.y >> shf, Z = hd.z >> shf, W = hd.w >> shf;
        const uint32_t Y1 = Y >> 8, Z1 = Z >> 8, W1 = W >> 8;
        const int sa = low ? (Y & 63) : ((W & 15) | ((Y >> 2) & 0x30));
        const int ma = low ? (Z & 63) : (((W >> 4) & 15) | ((Z >> 2) & 0x30));
        const int sb = low ? (Y1 & 63) : ((W1 & 15) | ((Y1 >> 2) & 0x30));
        const int mb = low ? (Z1 & 63) : (((W1 >> 4) & 15) | ((Z1 >> 2) & 0x30));
        ds_a[r] = d * i22_to_float(sa);
        ds_b[r] = d * i22_to_float(sb);
        dm_a[r] = dmin * i22_to_float(ma);
        dm_b[r] = dmin * i22_to_float(mb);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&empty[slot]));  // the stage is in registers

      const int row = t * BT_ROWS + 4 * cw + (lane & (V - 1)) / NBB;
      const uint8_t* ab0 = actb + (c - c_first) * BT_ACT_CHUNK;
#pragma unroll
      for (int nblk = 0; nblk < NB / NBB; nblk++) {
        float v[V];
#pragma unroll
        for (int nl = 0; nl < NBB; nl++) {
          const uint8_t* ab = ab0 + (nblk * NBB + nl) * a.span * BT_ACT_CHUNK;
          const int4* xa = reinterpret_cast<const int4*>(ab) + lane;
          const int4 a0 = xa[0], a1 = xa[32], b0 = xa[64], b1 = xa[96];
          const int xA[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          const int xB[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
          const float2 xs2 = *reinterpret_cast<const float2*>(ab + 2048 + 4 * (8 * bl + 2 * g));
          const int2 sm2 = *reinterpret_cast<const int2*>(ab + 2048 + 256 + 4 * (8 * bl + 2 * g));
          const float fxa = i22_to_float(sm2.x), fxb = i22_to_float(sm2.y);
#pragma unroll
          for (int r = 0; r < 4; r++) {
            int ia = 0, ib = 0;
#pragma unroll
            for (int k = 0; k < 8; k++) {
              ia = __dp4a((int)lo[r][k], xA[k], ia);
              ib = __dp4a((int)hi[r][k], xB[k], ib);
            }
            v[r * NBB + nl] = xs2.x * (ds_a[r] * i22_to_float(ia) - dm_a[r] * fxa) +
                              xs2.y * (ds_b[r] * i22_to_float(ib) - dm_b[r] * fxb);
          }
        }
        const float sum = warp_transpose_sum<V>(v);
        if (a.tile_order) {
          tot[nblk] += sum;  // chunks of a tile arrive in order
        } else {
          const int n = nblk * NBB + nsub;
          if (lane < V && row < a.n_out && n < a.n_batch) {
            if (a.nch == 1) a.out[(size_t)n * a.n_out + row] = sum + (a.bias ? __ldg(a.bias + row) : 0.f);
            else a.part[((size_t)c * a.n_batch + n) * a.n_out + row] = sum;
          }
        }
      }
    }
    if (a.tile_order && cur_t >= 0 && !failed) tile_flush<NB, NBB>(a, cur_t, cw, lane, rsub, nsub, tot);
  }
  if (failed && a.err_flag) atomicExch(a.err_flag, 1);
}

// out[n][r] = sum over chunks c in order of part[c][n][r] (+ bias[r]).
__global__ void __launch_bounds__(256) q4k_batch_sum_kernel(float* out, const float* part, const float* bias,
                                                            int n_out, int n_batch, int nch) {
  pdl_launch_dependents();
  pdl_wait();
  const int total = n_out * n_batch;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < total; j += gridDim.x * blockDim.x) {
    const int r = j % n_out;
    float s = 0.f;
    for (int c = 0; c < nch; c++) s += part[(size_t)c * total + j];
    out[j] = s + (bias ? bias[r] : 0.f);
  }
}

// ------------------------------------------------------------------ host

// The chunk-sum kernel as a programmatic dependent of the kernel before it.
cudaError_t launch_chunk_sum(float* out, const float* part, const float* bias, int n_out, int n_batch, int nch,
                             int num_sms, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  const int total = n_batch * n_out;
  cfg.gridDim = dim3((unsigned)std::min((total + 255) / 256, 4 * num_sms));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, q4k_batch_sum_kernel, out, part, bias, n_out, n_batch, nch);
}

bool encode_tmap_2d(CUtensorMap* m, CUtensorMapDataType type, const void* base, uint64_t d0, uint64_t d1,
                    uint64_t stride1, uint32_t b0, uint32_t b1, CUtensorMapSwizzle swizzle) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  const cuuint64_t dims[2] = {d0, d1};
  const cuuint64_t strides[1] = {stride1};
  const cuuint32_t box[2] = {b0, b1};
  const cuuint32_t es[2] = {1, 1};
  return fn(m, type, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

constexpr size_t BT_SMEM_MAX = 227 * 1024;

// The shared-memory opt-in is set once per device and instance. Launched as
// a programmatic dependent of the preceding kernel: its prologue and weight
// stream overlap that kernel's tail.
template <int NB>
cudaError_t launch_nb(const CUtensorMap& m, const BatchArgs& a, int grid, cudaStream_t st) {
  static std::atomic<unsigned long long> ready{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(ready.load() & bit)) {
    e = cudaFuncSetAttribute(q4k_batch_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BT_SMEM_MAX);
    if (e != cudaSuccess) return e;
    ready.fetch_or(bit);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(BT_THREADS);
  cfg.dynamicSmemBytes = BT_HEADER + (size_t)a.n_stages * BT_STAGE_BYTES + (size_t)NB * a.span * BT_ACT_CHUNK;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, q4k_batch_kernel<NB>, m, a);
}

// Most chunks any CTA's chunk-major unit range touches.
int max_span(int n_units, int n_tiles, int grid) {
  int s = 0;
  for (int b = 0; b < grid; b++) {
    const int u0 = (int)((long long)n_units * b / grid), u1 = (int)((long long)n_units * (b + 1) / grid);
    if (u1 > u0) s = std::max(s, (u1 - 1) / n_tiles - u0 / n_tiles + 1);
  }
  return s;
}

int cta_of_unit_host(int u, int n_units, int grid) {
  return (int)((((long long)u + 1) * grid + n_units - 1) / n_units) - 1;
}

// Activation slots (activations x chunks) that fit beside a 3-slot ring.
constexpr int BT_TILE_SLOTS = (int)((BT_SMEM_MAX - BT_HEADER - 3 * (size_t)BT_STAGE_BYTES) / BT_ACT_CHUNK);

struct BatchPlan {
  int NB, grid, tile_order, span, pmax;
  size_t part_floats;
};

// Launch geometry of one launch of nbt (<= 16) activations. Tile order when
// every chunk's activation fits in shared memory (a CTA then accumulates a
// tile's chunks in registers); chunk order otherwise (partials of every
// chunk, summed by the second kernel).
BatchPlan plan_batch(int n_out, int n_in, int nbt, int num_sms) {
  BatchPlan p = {};
  const int nch = n_chunks(n_in / QK), n_tiles = (n_out + BT_ROWS - 1) / BT_ROWS, n_units = nch * n_tiles;
  p.NB = nbt <= 1 ? 1 : nbt <= 2 ? 2 : nbt <= 4 ? 4 : nbt <= 8 ? 8 : 16;
  p.grid = std::min(n_units, num_sms);
  if (p.NB * nch <= BT_TILE_SLOTS) {
    p.tile_order = 1;
    p.span = nch;
    for (int t = 0; t < n_tiles; t++)
      p.pmax = std::max(p.pmax, cta_of_unit_host(t * nch + nch - 1, n_units, p.grid) -
                                     cta_of_unit_host(t * nch, n_units, p.grid) + 1);
    p.part_floats = p.pmax > 1 ? (size_t)n_tiles * p.pmax * nbt * BT_ROWS : 0;
  } else {
    while (p.NB * max_span(n_units, n_tiles, p.grid) > BT_ACT_SLOTS && p.grid < n_units)
      p.grid = std::min(n_units, 2 * p.grid);
    p.span = max_span(n_units, n_tiles, p.grid);
    p.part_floats = nch > 1 ? (size_t)nch * nbt * n_out : 0;
  }
  return p;
}

size_t ticket_offset(size_t part_floats) { return ((part_floats * 4 + 255) & ~(size_t)255); }

}  // namespace

// Batched Q4_K matmul, up to BT_MAX_NB activations per launch; larger
// batches are split. Returns a CUDA error or cudaErrorInvalidValue for
// unsupported shapes. scratch: q4k_batch_scratch_bytes, its ticket words
// (after the partials) zero; the launches leave them zero.
cudaError_t launch_q4k_batch(float* out, const uint8_t* w, const int8_t* xq, const float* xs, const float* bias,
                             int n_out, int n_in, int n_batch, void* scratch, int* err_flag, int num_sms,
                             cudaStream_t st) {
  const int nb = n_in / QK;
  const size_t rowB = (size_t)nb * Q4K_BYTES;
  CUtensorMap m;
  if (!encode_tmap_2d(&m, CU_TENSOR_MAP_DATA_TYPE_UINT64, w, rowB / 8, (uint64_t)n_out, rowB, Q4K_CHUNK / 8,
                      BT_ROWS))
    return cudaErrorInvalidValue;
  BatchArgs a = {};
  a.err_flag = err_flag;
  a.bias = bias;
  a.n_out = n_out;
  a.n_in = n_in;
  a.nch = n_chunks(nb);
  a.n_tiles = (n_out + BT_ROWS - 1) / BT_ROWS;
  a.n_units = a.nch * a.n_tiles;
  a.part = (float*)scratch;
  a.ticket = (int*)((char*)scratch + q4k_batch_ticket_offset(n_out, n_in, n_batch, num_sms));
  for (int n0 = 0; n0 < n_batch; n0 += BT_MAX_NB) {
    const int nbt = std::min(BT_MAX_NB, n_batch - n0);
    const BatchPlan P = plan_batch(n_out, n_in, nbt, num_sms);
    if (P.NB * P.span > (P.tile_order ? BT_TILE_SLOTS : BT_ACT_SLOTS)) return cudaErrorInvalidValue;
    a.tile_order = P.tile_order;
    a.pmax = P.pmax;
    a.span = P.span;
    const size_t act = (size_t)P.NB * a.span * BT_ACT_CHUNK;
    a.n_stages = (int)std::min<size_t>(BT_MAX_STAGES, (BT_SMEM_MAX - BT_HEADER - act) / BT_STAGE_BYTES);
    a.out = out + (size_t)n0 * n_out;
    a.xq = xq + (size_t)n0 * n_in;
    a.xs = xs + (size_t)n0 * (n_in / 32);
    a.n_batch = nbt;
    cudaError_t e;
    switch (P.NB) {
      case 1: e = launch_nb<1>(m, a, P.grid, st); break;
      case 2: e = launch_nb<2>(m, a, P.grid, st); break;
      case 4: e = launch_nb<4>(m, a, P.grid, st); break;
      case 8: e = launch_nb<8>(m, a, P.grid, st); break;
      default: e = launch_nb<16>(m, a, P.grid, st); break;
    }
    if (e != cudaSuccess) return e;
    if (!P.tile_order && a.nch > 1) {
      e = launch_chunk_sum(a.out, a.part, bias, n_out, nbt, a.nch, num_sms, st);
      if (e != cudaSuccess) return e;
    }
  }
  return cudaSuccess;
}

// Partials of the largest launch, then the tickets.
size_t q4k_batch_scratch_bytes(int n_out, int n_in, int n_batch, int num_sms) {
  size_t part = 0;
  for (int n0 = 0; n0 < n_batch; n0 += BT_MAX_NB)
    part = std::max(part, plan_batch(n_out, n_in, std::min(BT_MAX_NB, n_batch - n0), num_sms).part_floats);
  const int n_tiles = (n_out + BT_ROWS - 1) / BT_ROWS;
  return ticket_offset(part) + (size_t)n_tiles * BT_WARPS * 4;
}

size_t q4k_batch_ticket_offset(int n_out, int n_in, int n_batch, int num_sms) {
  const int n_tiles = (n_out + BT_ROWS - 1) / BT_ROWS;
  return q4k_batch_scratch_bytes(n_out, n_in, n_batch, num_sms) - (size_t)n_tiles * BT_WARPS * 4;
}

}  // namespace hakm
