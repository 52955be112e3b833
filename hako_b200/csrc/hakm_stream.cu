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
//               then each takes 4-row units of a stage (whole rows): Q4_K
//               rows with dp4a integer sub-block sums (src/quant.c:150-232),
//               Q6_K rows as the fp32 dot on the fly (src/nn.c:84-95,
//               src/quant.c:94-123), both with the reference's roundings
//               (hakm_gemv.cuh); one result per row lands in shared memory.
//   epilogue    bias / residual / NeoX RoPE + K append / V append / SwiGLU /
//               logits + greedy argmax, and for the lm_head phase the step
//               finalisation (next token, token log, position + 1).
//
// Every wait on an mbarrier is bounded (clock64); a timeout sets
// PhaseParams::err_flag and the CTA drains its own copies and returns.
#include "hakm_gemv.cuh"

namespace hakm {

// ------------------------------------------------------------------ kernel

// KINDS: bit 0 = Q4_K segments, bit 1 = Q6_K segments.
template <int KINDS>
__global__ void __launch_bounds__(THREADS, 1) stream_kernel(const __grid_constant__ PhaseParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + MAX_STAGES;
  const int S_ = p.n_stages, SB = p.stage_bytes;
  uint8_t* ring = smem + SMEM_HEADER;
  const int K = p.n_in, nb = K / QK, nsb = K / 32;
  uint8_t* act = ring + (size_t)S_ * SB;
  const bool f32 = p.need_q6 || p.act == ACT_RMS;
  const Act A = carve_act(act, K, p.need_q8, f32);
  float* part = reinterpret_cast<float*>(act + act_bytes(K, p.need_q8, f32));
  float* red = part + p.part_floats;
  float* wscr = red + 64;  // per-warp unit scratch
  (void)nsb;

  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) TRACE(0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S_; i++) {
      mbar_init(smem_addr(&full[i]), 1);
      mbar_init(smem_addr(&empty[i]), CONSUMER_WARPS / phase_groups(nb));
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
      const int R = stage_rows(type, nb);
      for (int rt = sr[s].row0; rt < sr[s].row1; rt += R, i++) {
        const int nr = min(R, sr[s].row1 - rt);
        const int slot = i % S_;
        if (i >= S_) {
          bool ok = true;
          if (lane == 0) ok = mbar_wait(smem_addr(&empty[slot]), ((i / S_) - 1) & 1);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) { failed = true; break; }
        }
        if (lane == 0) {
          const uint32_t bytes = (uint32_t)(nr * rowB);
          mbar_expect_tx(smem_addr(&full[slot]), bytes);
          bulk_g2s(smem_addr(ring + (size_t)slot * SB), S.w + (size_t)rt * rowB, bytes, smem_addr(&full[slot]));
        }
        __syncwarp();
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
    build_activation(p, wpre, A, red);
    if (threadIdx.x == 32) TRACE(1);
    const int cw = warp - 1;
    float* tr = wscr + cw * WARP_SCRATCH_FLOATS;
    bool first = true;
    int i = 0;
    unsigned ucount = 0;  // units seen: rotates the units over the warps
    for (int s = 0; s < p.n_seg && !failed; s++) {
      const int type = (KINDS == 1) ? W_Q4K : (KINDS == 2) ? W_Q6K : p.seg[s].type;
      const int rowB = (int)dev_row_bytes(type, nb);
      const int R = stage_rows(type, nb);
      // units of whole rows: 4, or 8 (two a lane) for Q6_K rows by the
      // hundred per CTA (the lm_head)
      const int ur = (type == W_Q6K && R >= 8 && sr[s].row1 - sr[s].row0 >= 8 * CONSUMER_WARPS) ? 8 : 4;
      const int n_units = (R + ur - 1) / ur;
      for (int rt = sr[s].row0; rt < sr[s].row1; rt += R, i++) {
        const int nr = min(R, sr[s].row1 - rt);
        const int slot = i % S_;
        if (!mbar_wait(smem_addr(&full[slot]), (i / S_) & 1)) { failed = true; break; }
        if (first && threadIdx.x == 32) TRACE(2);
        first = false;
        const uint8_t* stage = ring + (size_t)slot * SB;
        const int u0 = (int)((unsigned)(cw + CONSUMER_WARPS) - ucount % CONSUMER_WARPS) % CONSUMER_WARPS;
        for (int u = u0; u < n_units; u += CONSUMER_WARPS) {
          const int t0 = ur * u, nru = min(ur, nr - t0);
          if (nru <= 0) continue;
          const uint8_t* st = stage + (size_t)t0 * rowB;
          float* dst = part + sr[s].part_base + (rt - sr[s].row0 + t0);
          if (type == W_Q4K) {
            if constexpr (KINDS & 1) {
              const float tot = q4k_rows<4>(st, rowB, nru, nb, A, tr);
              if (lane < nru) dst[lane] = tot;
            }
          } else {
            if constexpr (KINDS & 2) {
              if (ur == 8) {
                float tot[2];
                q6k_rows<2>(st, rowB, nru, nb, A, tot);
                if ((lane & 7) == 0 && (lane >> 3) < nru) dst[lane >> 3] = tot[0];
                if ((lane & 7) == 0 && (lane >> 3) + 4 < nru) dst[(lane >> 3) + 4] = tot[1];
              } else {
                float tot[1];
                q6k_rows<1>(st, rowB, nru, nb, A, tot);
                if ((lane & 7) == 0 && (lane >> 3) < nru) dst[lane >> 3] = tot[0];
              }
            }
          }
        }
        ucount += (unsigned)n_units;
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&empty[slot]));
      }
    }
    consumers_sync();
    if (threadIdx.x == 32) TRACE(3);
    if (!failed) epilogue(p, sr, part, red, p.pos_dev ? *p.pos_dev : 0);
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
  size_t slot = 0;
  int part = 0;
  for (int s = 0; s < q.n_seg; s++) {
    const size_t sb = (size_t)stage_rows(q.seg[s].type, nb) * dev_row_bytes(q.seg[s].type, nb);
    slot = sb > slot ? sb : slot;
    const int G = (q.seg[s].n_rows + 3) / 4;
    part += ((G + grid - 1) / grid) * 4;
  }
  q.stage_bytes = (int)slot;
  q.part_floats = (part + 3) & ~3;
  const size_t fixed = SMEM_HEADER + act_bytes(K, q.need_q8, q.need_q6 || q.act == ACT_RMS) +
                       (size_t)q.part_floats * 4 + 64 * 4 + WARP_SCRATCH_BYTES;
  // Stage i lives in slot i % S and is consumed by group i % groups. S must
  // be a multiple of groups: then every slot belongs to one group, which waits
  // on that slot's phases strictly in order — a parity wait can never see a
  // phase two behind and alias.
  const int groups = phase_groups(nb);
  const long avail = (long)PHASE_BUDGET - (long)fixed;
  int k = (int)(avail / ((long)groups * q.stage_bytes));
  const int kmax = groups == 1 ? 6 : 3;
  k = k < 1 ? 1 : (k > kmax ? kmax : k);
  if (groups == 1 && k < 2 && avail >= 2L * q.stage_bytes) k = 2;
  q.n_stages = k * groups;
  return fixed + (size_t)q.n_stages * q.stage_bytes;
}

size_t phase_smem_bytes(const PhaseParams& p, int grid) {
  PhaseParams q = p;
  return plan(q, grid);
}

template <int KINDS>
static cudaError_t launch_k(const PhaseParams& p, int grid, size_t smem, cudaStream_t s, bool pdl) {
  static unsigned done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 32 && !(done & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(stream_kernel<KINDS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
  return cudaLaunchKernelEx(&cfg, stream_kernel<KINDS>, p);
}

cudaError_t launch_phase(const PhaseParams& p0, int num_sms, cudaStream_t s, bool pdl) {
  PhaseParams p = p0;
  if (p.act == ACT_RMS && p.n_in > 8 * RMS_SLOTS * CONSUMER_WARPS * 32) return cudaErrorInvalidValue;
  const int grid = phase_grid_size(p, num_sms);
  const size_t smem = plan(p, grid);
  if (smem > (size_t)PHASE_SMEM_MAX || p.n_stages > MAX_STAGES) return cudaErrorInvalidValue;
  if (p.act == ACT_RMS && !p.rsq) return cudaErrorInvalidValue;
  const int kinds = phase_kinds(p);
  if (kinds == 1) return launch_k<1>(p, grid, smem, s, pdl);
  if (kinds == 2) return launch_k<2>(p, grid, smem, s, pdl);
  return launch_k<3>(p, grid, smem, s, pdl);
}

}  // namespace hakm
