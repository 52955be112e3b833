// hakm_step.cu — the persistent decode-step kernel.
//
// One cooperative launch (one CTA per SM) runs n_steps whole decode steps of
// hakm_forward (src/model.c:93-165): embedding, then per layer the qkv,
// attention, attn-output, ffn gate/up and ffn down phases, then lm_head with
// the greedy pick. The phase list of one step is a device-resident program
// built by the runtime.
//
//   warp 0      producer: walks the program for all steps and streams every
//               GEMV phase's weight rows for this CTA through one ring of
//               shared-memory slots (cp.async.bulk + mbarrier). It waits
//               only for free slots, so the next phases' weights are loading
//               while the consumers wait for inputs, run attention or write
//               an epilogue.
//   warps 1..11 consumers: per phase, fetch the inputs, rebuild the
//               activation (norm weights fetched first), consume the phase's
//               stages, run the epilogue. Every consumer warp visits every
//               stage (waits its full barrier, does the 4-row units that fall
//               to it, arrives on its empty barrier), so each slot's phases
//               are waited strictly in order whatever mix of phases shares
//               the ring.
//
// Phases hand vectors to each other as tagged words (hakm_ll.cuh): a reader
// polls the words it needs until they carry the writing phase's tag, so
// there is no grid barrier between phases. Every GEMV phase needs all of its
// input vector and every output of a phase feeds some later phase, so a CTA
// that has read phase p's input knows that every CTA has finished reading
// phase p-2's: the residual therefore alternates between two buffers and the
// other vectors need one.
//
// One grid barrier (monotonic counter, release add / acquire poll) remains
// per step: the greedy pick of step s is an atomicMax over all CTAs into
// keys[s % 3], read after the barrier that ends step s, and the barrier also
// orders the K/V cache rows written in one step before the attention of the
// next. The first n_forced steps can take forced input tokens (a prompt), so
// prompt + generation is one launch; their lm_head phase is skipped except on
// the last forced step, whose pick is the first generated token.
//
// Every wait is bounded; a timeout, or the error flag raised by another CTA,
// makes the CTA stop issuing work, wait for its own copies and return.
#include <algorithm>
#include <cstdlib>

#include "hakm_attn.cuh"
#include "hakm_gemv.cuh"
#include "hakm_ll.cuh"

namespace hakm {

struct ConsumerSync {
  __device__ void operator()() const { consumers_sync(); }
};

// consumers_sync that also ORs a flag over the 384 consumer threads.
__device__ __forceinline__ bool consumers_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.or.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(BAR_CONSUMERS), "n"(CONSUMER_WARPS * 32)
      : "memory");
  return r != 0;
}

// Called by one thread after a consumers_sync. The release add is cumulative:
// the CTA's writes that this thread observed through the named barrier are
// visible to whoever acquires the count. System scope (here and in
// grid_wait): with tensor parallelism the writes include other GPUs' memory
// and the waiters include other GPUs' threads; once per step, so the cost of
// the wider scope does not matter.
__device__ __forceinline__ void grid_arrive(unsigned* bar) {
  asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
}

// Bounded poll of a step counter (relaxed loads, one acquire fence once it
// is reached); the error flag is looked at every 2^12 cycles.
__device__ __forceinline__ bool grid_wait(const unsigned* bar, unsigned target, const int* err) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
  if (v < target) {
    const long long t0 = clock64();
    long long next = t0 + 4096;
    for (;;) {
      asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
      if (v >= target) break;
      const long long now = clock64();
      if (now > next) {
        if (ll_aborted(err) || now - t0 > WAIT_LIMIT) return false;
        next = now + 4096;
      }
    }
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  return true;
}

__device__ __forceinline__ bool mbar_wait_or_abort(uint32_t bar, uint32_t parity, const int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  long long next = t0 + 4096;
  while (!mbar_try_wait_sleep(bar, parity)) {
    const long long now = clock64();
    if (now > next) {
      if (ll_aborted(err) || now - t0 > WAIT_LIMIT) return false;
      next = now + 4096;
    }
  }
  return true;
}

__device__ __forceinline__ int key_pick(const unsigned long long* key) {
  return argmax_key_index(__ldcg(key));
}

// Address p (in region `region` of this GPU) in rank r's copy.
template <class T>
__device__ __forceinline__ T* on_rank(const StepArgs& A, T* p, int region, int r) {
  return reinterpret_cast<T*>(reinterpret_cast<char*>(p) + A.tp_delta[r][region]);
}
// GPUs an output goes to: compile-time 1 in the single-GPU kernel instance.
template <bool TP>
__device__ __forceinline__ int n_ranks(const StepArgs& A) { return TP ? A.tp_world : 1; }
// A tagged word to every GPU's copy of an exchange vector.
template <bool TP>
__device__ __forceinline__ void put_all(const StepArgs& A, uint64_t* p, uint64_t w) {
  if (!TP) { ll_st1(p, w); return; }
  for (int r = 0; r < A.tp_world; r++) ll_st1(on_rank(A, p, XR_LL, r), w);
}

__device__ __forceinline__ bool phase_runs(const StepArgs& A, int ph, int step) {
  return !(A.skip_last && ph == A.n_phases - 1 && step + 1 < A.n_forced);
}

// Copy of a phase descriptor into shared memory by the first 32 consumer
// threads (read-only path): consumers read descriptors from there, never
// in a chain of dependent global loads.
__device__ __forceinline__ void stage_desc(PhaseDesc* dst, const PhaseDesc* src, int t) {
  constexpr int W = (int)(sizeof(PhaseDesc) / 16);
  static_assert(sizeof(PhaseDesc) % 16 == 0, "descriptor copied as uint4");
  for (int i = t; i < W; i += 32) reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
}

// This CTA's rows of program phase ph (host-computed table) into shared
// memory, by the threads of the second consumer warp.
__device__ __forceinline__ void stage_ranges(SegRange* dst, const SegRange* table, int ph, int t, unsigned grid,
                                             unsigned cta) {
  const int i = t - 32;
  if (i >= 0 && i < MAX_SEGS)
    reinterpret_cast<int4*>(dst)[i] = __ldg(reinterpret_cast<const int4*>(table + ((size_t)ph * grid + cta) * MAX_SEGS) + i);
}

// Epilogue operands that do not depend on the phase's results, loaded at the
// start of the phase for this thread's first item: the RoPE pair's biases
// and (cos, sin), the V row's bias.
struct EpiPre {
  float b0 = 0.f, b1 = 0.f, bv = 0.f;
  float2 cs = make_float2(0.f, 0.f);
};

// Per-segment stage geometry of this CTA, computed once per phase: R whole
// rows per stage (one bulk copy), units of ur (4, or 2) whole rows.
struct SegGeo {
  int type, rowB, R, nch, chunkB, rn, ur;
  int cr;           // chunk-stream rows (0: whole-row stages)
  const void* map;  // its two tensor maps
};
// Read from the descriptor (computed by plan_step on the host).
__device__ __forceinline__ SegGeo seg_geo(const PhaseDesc& D, int s) {
  SegGeo g;
  g.type = D.g.seg[s].type;
  g.rowB = D.st_row_bytes[s];
  g.R = D.st_rows[s];
  g.nch = D.st_nch[s];
  g.chunkB = g.type == W_Q4K ? Q4K_CHUNK : Q6K_CHUNK;
  g.rn = D.st_rn[s];
  g.ur = D.st_unit_rows[s];
  g.cr = D.st_chunk_rows[s];
  g.map = D.st_map[s];
  return g;
}

// Ring position of the next stage: slot = i % S, parity = (i / S) & 1.
struct Ring {
  int slot = 0;
  uint32_t par = 0;
  bool lapped = false;  // a full lap done: slots must be freed before reuse
  __device__ __forceinline__ void advance(int S) {
    if (++slot == S) { slot = 0; par ^= 1u; lapped = true; }
  }
};

// Activation of a GEMV phase from a tagged input vector (as build_activation
// for ACT_RMS / ACT_F32). plain: if set, the raw input is also written there
// as floats. Returns false if a wait gave up.
__device__ bool build_activation_ll(const PhaseParams& p, const uint64_t* x, uint32_t tag,
                                    const float wpre[RMS_SLOTS][8], const Act& A, float* red, const int* err,
                                    float* plain) {
  const int K = p.n_in, nslot = K >> 3;
  const int t = threadIdx.x - 32, nt = CONSUMER_WARPS * 32;
  bool ok = true;
  if (p.act == ACT_RMS) {
    float v[RMS_SLOTS][8];
#pragma unroll
    for (int j = 0; j < RMS_SLOTS; j++) {
      const int s = t + j * nt;
      if (s < nslot) {
        ok &= ll_get<8>(x + 8 * s, tag, v[j], err);
        if (plain) {
#pragma unroll
          for (int i = 0; i < 8; i++) plain[8 * s + i] = v[j][i];
        }
        // squares by lane class for the scale (src/nn.c:15 as built)
        const int ts = cls_slot(s);
#pragma unroll
        for (int i = 0; i < 8; i++) A.xc[i * A.cp + ts] = __fmul_rn(v[j][i], v[j][i]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; i++) v[j][i] = 0.f;
      }
    }
    consumers_sync();
    if (t < 32) {
      const float sc = rms_scale(A.xc, A.cp, K, p.eps, p.rsq);
      if (t == 0) red[0] = sc;
    }
    consumers_sync();
    const float scale = red[0];
    // src/nn.c:17 as built: y = (x * w) * scale
#pragma unroll
    for (int j = 0; j < RMS_SLOTS; j++) {
      const int s = t + j * nt;
      if (j * nt >= nslot) break;  // uniform: no live slot for any thread
#pragma unroll
      for (int i = 0; i < 8; i++) v[j][i] = __fmul_rn(__fmul_rn(v[j][i], wpre[j][i]), scale);
      store_slot(p, s, s < nslot, v[j], A);
    }
  } else {
    constexpr int F32_BATCH = 2;  // slots in flight per thread (raw words held in registers)
    for (int s0 = 0; s0 < nslot; s0 += F32_BATCH * nt) {
      float v[F32_BATCH][8];
      uint64_t w[F32_BATCH][8];
      // all slots' loads in flight before the first tag check
#pragma unroll
      for (int j = 0; j < F32_BATCH; j++) {
        const int s = s0 + j * nt + t;
        if (s < nslot) ll_issue8(x + 8 * s, w[j]);
      }
#pragma unroll
      for (int j = 0; j < F32_BATCH; j++) {
        const int s = s0 + j * nt + t;
        if (s < nslot) {
          ok &= ll_finish8(x + 8 * s, tag, w[j], v[j], err);
        } else {
#pragma unroll
          for (int i = 0; i < 8; i++) v[j][i] = 0.f;
        }
      }
#pragma unroll
      for (int j = 0; j < F32_BATCH; j++) {
        if (s0 + j * nt >= nslot) break;  // uniform
        const int s = s0 + j * nt + t;
        store_slot(p, s, s < nslot, v[j], A);
      }
    }
  }
  return ok;
}

// Epilogue record of one thread for one segment: its first output item,
// prepared at the start of the phase (off the critical path) so that after
// the last unit only the partial sums remain to be read. kind: 0 none, else
// an Epi code (EPI_ROPE_QK split into q and k by EPI_ROPE_K) | nch << 8.
constexpr int EPI_ROPE_K = 16;
struct __align__(16) EpiRec {
  int kind, pidx, o0, o1;
  float f0, f1, f2, f3;  // ROPE: bias pair, (cos, sin); RESID: residual; V / STORE: bias
};
constexpr int EPI_RECS = 2;  // segments with records

__device__ __forceinline__ EpiRec epi_prepare(const PhaseDesc& D, const SegRange* sr, int s, int pos, int t,
                                              uint32_t res_tag, bool& ok, const int* err) {
  const PhaseParams& p = D.g;
  const Seg& S = p.seg[s];
  const SegRange& r = sr[s];
  EpiRec e = {0, 0, 0, 0, 0.f, 0.f, 0.f, 0.f};
  if (S.epi == EPI_ROPE_QK || S.epi == EPI_SWIGLU) {
    if (2 * t + 1 >= r.row1 - r.row0) return e;
    const int dr = r.row0 + 2 * t;
    e.pidx = r.part_base + 2 * t;
    if (S.epi == EPI_SWIGLU) {
      e.kind = EPI_SWIGLU | (1 << 8);
      e.o0 = dr >> 1;
      return e;
    }
    const bool is_k = dr >= S.split;
    const int lr = is_k ? dr - S.split : dr;
    const int hd = p.head_dim, half = hd >> 1;
    const int head = lr / hd, pi = (lr % hd) >> 1;
    e.kind = (is_k ? EPI_ROPE_K : EPI_ROPE_QK) | (1 << 8);
    e.o0 = head * hd + pi;
    e.o1 = e.o0 + half;
    if (S.bias) { e.f0 = __ldg(S.bias + dr); e.f1 = __ldg(S.bias + dr + 1); }
    const float2 cs = __ldg(reinterpret_cast<const float2*>(p.rope_cs) + (size_t)pos * half + pi);
    e.f2 = cs.x;
    e.f3 = cs.y;
    return e;
  }
  const int row = r.row0 + t;
  if (row >= r.row1 || S.epi == EPI_ARGMAX) return e;
  e.kind = S.epi | (1 << 8);
  e.pidx = r.part_base + t;
  e.o0 = row;
  if (S.epi == EPI_RESID) ok &= ll_get1(D.res_ll + row, res_tag, e.f0, err);
  else if (S.bias) e.f0 = __ldg(S.bias + row);
  return e;
}

// The prepared first items: partial sums, arithmetic, stores.
template <bool TP>
__device__ __forceinline__ void epi_apply(const StepArgs& A, const PhaseDesc& D, int s, const EpiRec& e,
                                          const float* part, int pos, uint32_t tag) {
  const int kind = e.kind & 255, nch = e.kind >> 8;
  if (!kind) return;
  const PhaseParams& p = D.g;
  const float* pp = part + e.pidx;
  float a0 = pp[0];
  for (int c = 1; c < nch; c++) a0 += pp[c];
  if (kind == EPI_SWIGLU || kind == EPI_ROPE_QK || kind == EPI_ROPE_K) {
    float a1 = pp[nch];
    for (int c = 1; c < nch; c++) a1 += pp[nch + c];
    if (kind == EPI_SWIGLU) {
      // src/model.c:154 with silu_f (src/nn.c:29)
      put_all<TP>(A, D.out_ll[s] + e.o0, ll_word(swiglu_exact(a0, a1), tag));
      return;
    }
    const float x0 = __fadd_rn(a0, e.f0), x1 = __fadd_rn(a1, e.f1);
    // src/nn.c:38-40
    const float2 rr = rope_rotate(x0, x1, e.f2, e.f3);
    const float r0 = rr.x, r1 = rr.y;
    const bool is_k = kind == EPI_ROPE_K;
    uint64_t* dst = is_k ? D.out2_ll : D.out_ll[s];
    put_all<TP>(A, dst + e.o0, ll_word(r0, tag));
    put_all<TP>(A, dst + e.o1, ll_word(r1, tag));
    if (is_k) {
      float* kc = p.seg[s].cache + A.kv_off + (size_t)pos * p.kv_dim;
      for (int r = 0; r < n_ranks<TP>(A); r++) {
        on_rank(A, kc, XR_KCACHE, r)[e.o0] = r0;
        on_rank(A, kc, XR_KCACHE, r)[e.o1] = r1;
      }
    }
    return;
  }
  const float o = __fadd_rn(a0, e.f0);  // residual or bias (0 when none)
  put_all<TP>(A, D.out_ll[s] + e.o0, ll_word(o, tag));
  if (kind == EPI_V_CACHE) {
    float* vc = p.seg[s].cache + A.kv_off + (size_t)pos * p.kv_dim + e.o0;
    for (int r = 0; r < n_ranks<TP>(A); r++) *on_rank(A, vc, XR_VCACHE, r) = o;
  }
}

// Epilogue of a GEMV phase of the step program: as epilogue(), with the
// vector outputs written as tagged words. res: this thread's prefetched
// previous residual for row r.row0 + t (EPI_RESID). Returns false if a wait
// gave up.
template <bool TP>
__device__ bool epilogue_ll(const StepArgs& A, const PhaseDesc& D, const SegRange* sr, const float* part, int pos,
                            unsigned long long* key, uint32_t tag, uint32_t res_tag, float res, const EpiPre& pre,
                            const int* err, int n_done = 0) {
  const int W = n_ranks<TP>(A);
  const PhaseParams& p = D.g;
  const int t = threadIdx.x - 32, nt = CONSUMER_WARPS * 32;
  unsigned long long best = 0ull;
  bool ok = true;
  for (int s = 0; s < p.n_seg; s++) {
    const Seg& S = p.seg[s];
    const SegRange& r = sr[s];
    uint64_t* out = D.out_ll[s];
    const int first = s < n_done ? nt : 0;  // items done from the records
    if (S.epi == EPI_ROPE_QK || S.epi == EPI_SWIGLU) {
      for (int q = t + first; 2 * q + 1 < r.row1 - r.row0; q += nt) {
        const int dr = r.row0 + 2 * q;
        const float a0 = row_total(part, r, dr), a1 = row_total(part, r, dr + 1);
        if (S.epi == EPI_SWIGLU) {
          // src/model.c:154 with silu_f (src/nn.c:29)
          put_all<TP>(A, out + (dr >> 1), ll_word(swiglu_exact(a0, a1), tag));
        } else {
          const bool first = q == t;
          const float x0 = S.bias ? __fadd_rn(a0, first ? pre.b0 : S.bias[dr]) : a0;
          const float x1 = S.bias ? __fadd_rn(a1, first ? pre.b1 : S.bias[dr + 1]) : a1;
          const bool is_k = dr >= S.split;
          const int lr = is_k ? dr - S.split : dr;
          const int hd = p.head_dim, half = hd >> 1;
          const int head = lr / hd, pi = (lr % hd) >> 1;
          const float2 cs = first ? pre.cs : reinterpret_cast<const float2*>(p.rope_cs)[(size_t)pos * half + pi];
          // src/nn.c:38-40
          const float2 rr = rope_rotate(x0, x1, cs.x, cs.y);
          const float r0 = rr.x, r1 = rr.y;
          const int o0 = head * hd + pi, o1 = o0 + half;
          uint64_t* dst = is_k ? D.out2_ll : out;
          put_all<TP>(A, dst + o0, ll_word(r0, tag));
          put_all<TP>(A, dst + o1, ll_word(r1, tag));
          if (is_k) {
            float* kc = S.cache + A.kv_off + (size_t)pos * p.kv_dim;
            for (int r = 0; r < W; r++) {
              on_rank(A, kc, XR_KCACHE, r)[o0] = r0;
              on_rank(A, kc, XR_KCACHE, r)[o1] = r1;
            }
          }
        }
      }
    } else {
      for (int row = r.row0 + t + (S.epi == EPI_ARGMAX ? 0 : first); row < r.row1; row += nt) {
        const float v = row_total(part, r, row);
        switch (S.epi) {
          case EPI_RESID: {
            float old = res;
            if (row != r.row0 + t) ok &= ll_get1(D.res_ll + row, res_tag, old, err);
            put_all<TP>(A, out + row, ll_word(__fadd_rn(old, v), tag));
            break;
          }
          case EPI_V_CACHE: {
            const float o = S.bias ? __fadd_rn(v, row == r.row0 + t ? pre.bv : S.bias[row]) : v;
            put_all<TP>(A, out + row, ll_word(o, tag));
            float* vc = S.cache + A.kv_off + (size_t)pos * p.kv_dim + row;
            for (int rr = 0; rr < W; rr++) *on_rank(A, vc, XR_VCACHE, rr) = o;
            break;
          }
          case EPI_ARGMAX: {
            if (S.out)
              for (int rr = 0; rr < W; rr++) on_rank(A, S.out, XR_LOGITS, rr)[row] = v;
            const unsigned long long kk = argmax_key(v, row);
            best = kk > best ? kk : best;
            break;
          }
          default:
            put_all<TP>(A, out + row, ll_word(S.bias ? __fadd_rn(v, S.bias[row]) : v, tag));
            break;
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
    if ((t & 31) == 0 && best) {
      if (W == 1) atomicMax(key, best);
      else
        for (int r = 0; r < W; r++) atomicMax_system(on_rank(A, key, XR_KEYS, r), best);
    }
  }
  return ok;
}

template <int HD, bool TP>
__global__ void __launch_bounds__(THREADS, 1) step_kernel(const __grid_constant__ StepArgs A) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + MAX_STAGES;
  const int S_ = A.n_stages, SB = A.slot_bytes;
  uint8_t* ring = smem + SMEM_HEADER;
  uint8_t* region = ring + (size_t)S_ * SB;  // activation of a GEMV phase / attention tiles
  float* part = reinterpret_cast<float*>(region + A.region_bytes);
  float* red = part + A.part_floats;
  float* wscr = red + 64;  // per-warp unit scratch (WARP_SCRATCH_FLOATS each)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned grid = gridDim.x, vcta = blockIdx.x;
  const int NP = A.n_phases + 1;  // tags per step: embedding + program

  if (threadIdx.x == 0) {
    for (int i = 0; i < S_; i++) {
      mbar_init(smem_addr(&full[i]), 1);
      mbar_init(smem_addr(&empty[i]), CONSUMER_WARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    Ring rp;
    int issued = 0;
    bool ok = true;
    for (int step = 0; step < A.n_steps && ok; step++) {
      for (int ph = 0; ph < A.n_phases && ok; ph++) {
        const PhaseDesc& D = A.prog[ph];
        if (D.kind != PK_GEMV || !phase_runs(A, ph, step)) continue;
        const SegRange* rtab = A.ranges + ((size_t)ph * grid + vcta) * MAX_SEGS;
        for (int s = 0; s < D.g.n_seg && ok; s++) {
          const SegGeo G = seg_geo(D, s);
          const uint8_t* w = D.g.seg[s].w;
          const int4 rr = __ldg(reinterpret_cast<const int4*>(rtab + s));
          if (G.cr > 0) {
            // chunk stages: the CTA's rows x chunk c, one tensor copy each
            if (rr.x >= rr.y) continue;
            const bool fewer = rr.y - rr.x <= G.cr - 4;
            const void* map = reinterpret_cast<const uint8_t*>(G.map) + (fewer ? 128 : 0);
            const uint32_t bytes = (uint32_t)((fewer ? G.cr - 4 : G.cr) * Q6K_CHUNK);
            for (int c = 0; c < G.nch && ok; c++) {
              if (rp.lapped) {
                bool wok = true;
                if (lane == 0) wok = mbar_wait_or_abort(smem_addr(&empty[rp.slot]), rp.par ^ 1u, A.err_flag);
                if (!__shfl_sync(0xffffffffu, wok, 0)) { ok = false; break; }
              }
              if (lane == 0) {
                mbar_expect_tx(smem_addr(&full[rp.slot]), bytes);
                tma_2d_stream(smem_addr(ring + (size_t)rp.slot * SB), map, c * (Q6K_CHUNK / 8), rr.x - rr.z,
                       smem_addr(&full[rp.slot]));
              }
              __syncwarp();
              rp.advance(S_);
              issued++;
            }
            continue;
          }
          for (int rt = rr.x; rt < rr.y; rt += G.R) {
            const int nr = min(G.R, rr.y - rt);
            if (rp.lapped) {
              bool wok = true;
              if (lane == 0) wok = mbar_wait_or_abort(smem_addr(&empty[rp.slot]), rp.par ^ 1u, A.err_flag);
              if (!__shfl_sync(0xffffffffu, wok, 0)) { ok = false; break; }
            }
            if (lane == 0) {
              const uint32_t bytes = (uint32_t)(nr * G.rowB);
              mbar_expect_tx(smem_addr(&full[rp.slot]), bytes);
              bulk_g2s(smem_addr(ring + (size_t)rp.slot * SB), w + (size_t)(rt - rr.z) * G.rowB, bytes,
                       smem_addr(&full[rp.slot]));
            }
            __syncwarp();
            rp.advance(S_);
            issued++;
          }
        }
      }
    }
    if (lane == 0) {
      if (!ok) atomicExch(A.err_flag, 1);
      // drain: every copy this CTA issued lands before the CTA exits
      for (int j = (issued > S_ ? issued - S_ : 0); j < issued; j++)
        if (!mbar_wait(smem_addr(&full[j % S_]), (j / S_) & 1)) atomicExch(A.err_flag, 1);
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int t = threadIdx.x - 32, nt = CONSUMER_WARPS * 32, cw = warp - 1;
  Ring rc;              // next stage to consume (the producer's order)
  unsigned ucount = 0;  // 4-row units seen; rotates units over the warps
  int kph = 0;          // phases run (trace index)
  bool bad = false;     // a wait of this thread gave up
  const int* err = A.err_flag;
  __shared__ int s_ok;
  // phase descriptors, staged one phase ahead: executed phase e uses buffer
  // e % 3; the buffer written during phase e was last read in phase e - 2,
  // which every consumer left before the barrier of phase e - 1
  __shared__ __align__(16) PhaseDesc s_desc[3];
  __shared__ SegRange s_sr[3][MAX_SEGS];  // this CTA's rows of each staged phase
  __shared__ int s_didx[3];
  int e = 0;
  if (t < 3) s_didx[t] = -1;
  consumers_sync();

  auto stamp = [&](int j) {
    if (A.trace && t == 0 && kph < A.trace_k)
      A.trace[((size_t)blockIdx.x * A.trace_k + kph) * 4 + j] = gtime();
  };
  auto tag_of = [&](int step, int idx) -> uint32_t { return A.tag_base + (uint32_t)(step * NP + idx); };

  for (int step = 0; step < A.n_steps; step++) {
    const int pos = A.pos0 + step;
    // ---- step barrier: the previous step's pick and K/V rows are complete
    // (with tensor parallelism: on every GPU, through the cross-GPU counter)
    if (step > 0) {
      if (t == 0)
        s_ok = A.tp_world == 1 ? grid_wait(A.bar, (unsigned)step * grid, err)
                               : grid_wait(A.xbar, (A.xbar_base + (unsigned)step) * (unsigned)A.tp_world, err);
      consumers_sync();
      if (!s_ok) bad = true;
    }
    if (consumers_sync_or(bad)) goto fail;
    stamp(0);
    // ---- embedding of this step's input token (deq_row, src/nn.c:55-59)
    {
      int token;
      if (step < A.n_forced) token = A.forced[step];
      else if (step == 0) token = __ldcg(A.token_dev);
      else token = key_pick(A.keys + (step - 1) % 3);
      if (vcta == 0 && t == 0) {
        const int j = step - 1 - A.log_base;
        if (step >= 1 && A.token_log && j >= 0 && j < A.token_log_cap)
          A.token_log[j] = key_pick(A.keys + (step - 1) % 3);
        // keys[(step + 1) % 3]: last read at the start of step - 1, first
        // written in step + 1, after a barrier this CTA arrives at later
        A.keys[(step + 1) % 3] = 0ull;
      }
      const int nbD = A.D / QK;
      const uint8_t* row = A.tok_embd + (size_t)token * dev_row_bytes(W_Q6K, nbD);
      const int gc = A.tp_rank * (int)grid + (int)vcta, n_gc = A.tp_world * (int)grid;
      const int per = (A.D + n_gc - 1) / n_gc;
      const int e1 = min(A.D, (gc + 1) * per);
      const uint32_t tg = tag_of(step, 0);
      for (int e = gc * per + t; e < e1; e += nt)
        put_all<TP>(A, A.xb_ll + e, ll_word(q6k_dequant_packed(row, nbD, e), tg));
    }
    stamp(3);
    kph++;

    for (int ph = 0; ph < A.n_phases; ph++) {
      if (!phase_runs(A, ph, step)) continue;
      const int b = e % 3;
      if (s_didx[b] != ph) {  // not staged ahead (first phase, or after a skipped one)
        stage_desc(&s_desc[b], &A.prog[ph], t);
        stage_ranges(s_sr[b], A.ranges, ph, t, grid, vcta);
        if (t == 0) s_didx[b] = ph;
        consumers_sync();
      }
      {
        int nx = ph + 1;
        if (nx >= A.n_phases || !phase_runs(A, nx, step)) nx = 0;
        const int nb = (e + 1) % 3;
        stage_desc(&s_desc[nb], &A.prog[nx], t);
        stage_ranges(s_sr[nb], A.ranges, nx, t, grid, vcta);
        if (t == 0) s_didx[nb] = nx;
      }
      e++;
      const PhaseDesc& D = s_desc[b];
      const uint32_t tag = tag_of(step, ph + 1);
      stamp(0);
      if (D.kind == PK_GEMV) {
        const PhaseParams& P = D.g;
        const int K = P.n_in, nb = K / QK;
        const SegRange* sr = s_sr[b];
        // inputs that do not depend on the previous phase first: norm
        // weights, and the residual rows of this CTA (written two or more
        // phases back)
        float wpre[RMS_SLOTS][8];
#pragma unroll
        for (int j = 0; j < RMS_SLOTS; j++) {
          const int s = t + j * nt;
          if (P.act == ACT_RMS && s < K / 8) {
            const float4* w4 = reinterpret_cast<const float4*>(P.norm_w);
            const float4 a = w4[2 * s], b = w4[2 * s + 1];
            wpre[j][0] = a.x; wpre[j][1] = a.y; wpre[j][2] = a.z; wpre[j][3] = a.w;
            wpre[j][4] = b.x; wpre[j][5] = b.y; wpre[j][6] = b.z; wpre[j][7] = b.w;
          } else {
#pragma unroll
            for (int q = 0; q < 8; q++) wpre[j][q] = 0.f;
          }
        }
        float res = 0.f;
        bool ok_pre = true;
        const uint32_t res_tag = tag_of(step, D.res_src);
        // epilogue records of this thread (its own slots: no barrier needed)
        int n_rec = 0;
        EpiRec* recs = nullptr;
        EpiPre pre;
        if (D.epi_rec_off >= 0) {
          recs = reinterpret_cast<EpiRec*>(region + D.epi_rec_off) + t * EPI_RECS;
          n_rec = min(P.n_seg, EPI_RECS);
          for (int s = 0; s < n_rec; s++) recs[s] = epi_prepare(D, sr, s, pos, t, res_tag, ok_pre, err);
        } else {
          // no room for records: the first items' operands in registers
          if (P.seg[0].epi == EPI_RESID && sr[0].row0 + t < sr[0].row1)
            bad |= !ll_get1(D.res_ll + sr[0].row0 + t, res_tag, res, err);
          if (P.seg[0].epi == EPI_ROPE_QK && 2 * t + 1 < sr[0].row1 - sr[0].row0) {
            const Seg& S0 = P.seg[0];
            const int dr = sr[0].row0 + 2 * t;
            if (S0.bias) { pre.b0 = __ldg(S0.bias + dr); pre.b1 = __ldg(S0.bias + dr + 1); }
            const int lr = dr >= S0.split ? dr - S0.split : dr;
            const int half = P.head_dim >> 1;
            pre.cs = __ldg(reinterpret_cast<const float2*>(P.rope_cs) + (size_t)pos * half + ((lr % P.head_dim) >> 1));
          }
          if (P.n_seg > 1 && P.seg[1].epi == EPI_V_CACHE && P.seg[1].bias && sr[1].row0 + t < sr[1].row1)
            pre.bv = __ldg(P.seg[1].bias + sr[1].row0 + t);
        }
        const Act X = carve_act(region, K, P.need_q8, P.need_q6 || P.act == ACT_RMS);
        float* plain =
            (P.seg[0].epi == EPI_ARGMAX && vcta == 0) ? A.xb_plain : nullptr;
        bad |= !build_activation_ll(P, D.x_ll, tag_of(step, D.x_src), wpre, X, red, err, plain);
        if (consumers_sync_or(bad)) goto fail;
        stamp(1);
        bool failed = false;
        for (int s = 0; s < P.n_seg && !failed; s++) {
          const SegGeo G = seg_geo(D, s);
          float* ps = part + sr[s].part_base;
          if (G.cr > 0) {
            // chunk stages: warp cw runs rows 4cw.. of the CTA's range, its
            // lane chains carried from chunk to chunk
            const int nr = sr[s].row1 - sr[s].row0;
            if (nr <= 0) continue;
            const bool mine = 4 * cw < nr;
            const int nru = min(4, nr - 4 * cw);
            float acc = 0.f;
            for (int c = 0; c < G.nch; c++) {
              const bool got = mbar_wait_or_abort(smem_addr(&full[rc.slot]), rc.par, err);
              if (!__all_sync(0xffffffffu, got)) {  // the warp leaves together
                failed = true;
                break;
              }
              const uint8_t* stage = ring + (size_t)rc.slot * SB;
              if (mine) acc = q6k_rows_chunk(stage + (size_t)4 * cw * Q6K_CHUNK, Q6K_CHUNK, nru, nb, c, X, acc);
              __syncwarp();
              if (lane == 0) mbar_arrive(smem_addr(&empty[rc.slot]));
              rc.advance(S_);
            }
            if (mine && !failed) {
              const float tot = fold8_lanes(acc);
              if ((lane & 7) == 0 && (lane >> 3) < nru) ps[4 * cw + (lane >> 3)] = tot;
            }
            continue;
          }
          // units of ur whole rows (every chunk, in order: the row sums are
          // sequential over the row, as the reference's are)
          const int n_units_full = (G.R + G.ur - 1) / G.ur;
          float* tr = wscr + cw * WARP_SCRATCH_FLOATS;
          for (int rt = sr[s].row0; rt < sr[s].row1; rt += G.R) {
            if (!mbar_wait_or_abort(smem_addr(&full[rc.slot]), rc.par, err)) {
              failed = true;
              break;
            }
            const int nr = min(G.R, sr[s].row1 - rt);
            const uint8_t* stage = ring + (size_t)rc.slot * SB;
            // this warp's units: u = first, first + 11, ... (rotated by ucount)
            const int first = (int)((unsigned)(cw + CONSUMER_WARPS) - ucount % CONSUMER_WARPS) % CONSUMER_WARPS;
            for (int u = first; u < n_units_full; u += CONSUMER_WARPS) {
              const int t0 = G.ur * u, nru = min(G.ur, nr - t0);
              if (nru <= 0) continue;
              const uint8_t* st = stage + t0 * G.rowB;
              float* dst = ps + (rt - sr[s].row0 + t0);
              if (G.type == W_Q4K) {
                const float tot = G.ur == 2 ? q4k_rows<2>(st, G.rowB, nru, nb, X, tr)
                                            : q4k_rows<4>(st, G.rowB, nru, nb, X, tr);
                if (lane < nru) dst[lane] = tot;
              } else if (G.ur == 8) {
                float tot[2];
                q6k_rows<2>(st, G.rowB, nru, nb, X, tot);
                if ((lane & 7) == 0 && (lane >> 3) < nru) dst[lane >> 3] = tot[0];
                if ((lane & 7) == 0 && (lane >> 3) + 4 < nru) dst[(lane >> 3) + 4] = tot[1];
              } else {
                float tot[1];
                q6k_rows<1>(st, G.rowB, nru, nb, X, tot);
                if ((lane & 7) == 0 && (lane >> 3) < nru) dst[lane >> 3] = tot[0];
              }
            }
            ucount += (unsigned)n_units_full;
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&empty[rc.slot]));
            rc.advance(S_);
          }
        }
        if (failed) { atomicExch(A.err_flag, 1); bad = true; }
        if (consumers_sync_or(bad)) goto fail;
        stamp(2);
        for (int s = 0; s < n_rec; s++) epi_apply<TP>(A, D, s, recs[s], part, pos, tag);
        bad |= !ok_pre;
        bad |= !epilogue_ll<TP>(A, D, sr, part, pos, P.argmax_key ? A.keys + step % 3 : nullptr, tag, res_tag, res, pre,
                                err, n_rec);
        // the next phase's activation may be built over these records
        if (n_rec) consumers_sync();
      } else {
        consumers_sync();  // the next descriptor is staged; CTAs without items have no other barrier here
        AttnLL T;
        T.q = D.x_ll;
        T.k = D.res_ll;
        T.v = D.v_ll;
        T.out = D.out_ll[0];
        T.in_tag = tag_of(step, D.x_src);
        T.out_tag = tag;
        T.err = err;
        T.n_dst = n_ranks<TP>(A);
        T.out_delta = &A.tp_delta[0][XR_LL];
        T.delta_stride = XR_COUNT;
        T.kv_off = A.kv_off;
        T.sc_cap = A.region_bytes / 4 - (int)(attn_smem_bytes(HD) / 4);
        // (query head, dimension slice) units; with tensor parallelism this
        // GPU runs units rank, rank + world, ...
        const int n_loc = attn_units_local(attn_units(D.a.n_heads, HD), A.tp_rank, A.tp_world);
        float* sm = reinterpret_cast<float*>(region);
        for (int it = (int)vcta; it < n_loc; it += grid)
          bad |= !attn_item<HD, true>(D.a, attn_unit_of(A.tp_rank, A.tp_world, it), pos, sm, t, nt, ConsumerSync(), T);
        // the next phase writes the shared region (activation, epilogue
        // records): every thread must be done with the attention tiles
        consumers_sync();
      }
      stamp(3);
      kph++;
    }
    // ---- end of step: every CTA's pick and cache rows are in
    if (consumers_sync_or(bad)) goto fail;
    if (t == 0) {
      grid_arrive(A.bar);
      if (A.tp_world > 1 && vcta == 0) {
        // this GPU's CTAs are done: signal every GPU's cross-GPU counter
        if (grid_wait(A.bar, (unsigned)(step + 1) * grid, err)) {
          for (int r = 0; r < A.tp_world; r++)
            asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(on_rank(A, A.xbar, XR_XBAR, r)) : "memory");
        } else {
          atomicExch(A.err_flag, 1);
        }
      }
    }
  }
  // the last step's pick: next input token, token log, position
  if (vcta == 0 && t == 0) {
    const bool done = A.tp_world == 1
                          ? grid_wait(A.bar, (unsigned)A.n_steps * grid, err)
                          : grid_wait(A.xbar, (A.xbar_base + (unsigned)A.n_steps) * (unsigned)A.tp_world, err);
    if (done) {
      const int tok = key_pick(A.keys + (A.n_steps - 1) % 3);
      *A.token_dev = tok;
      const int j = A.n_steps - 1 - A.log_base;
      if (A.token_log && j >= 0 && j < A.token_log_cap) A.token_log[j] = tok;
      *A.pos_dev = A.pos0 + A.n_steps;
    } else {
      atomicExch(A.err_flag, 1);
    }
  }
  return;
fail:
  if (t == 0) atomicExch(A.err_flag, 1);
}

__global__ void ll_unpack_kernel(float* out, const uint64_t* in, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = ll_value(in[i]);
}

// ---------------------------------------------------------------------- host

// Host copy of cta_ranges (hakm_gemv.cuh): a segment's 4-row groups split
// evenly over the grid, each segment's split rotated by the groups before it.
void step_ranges(const PhaseDesc* prog, int n_phases, int grid, int cta0, int n_ctas, SegRange* out) {
  for (int ph = 0; ph < n_phases; ph++)
    for (int lc = 0; lc < n_ctas; lc++) {
      const int cta = cta0 + lc;
      SegRange* sr = out + ((size_t)ph * n_ctas + lc) * MAX_SEGS;
      for (int s = 0; s < MAX_SEGS; s++) sr[s] = SegRange{0, 0, 1, 0};
      if (prog[ph].kind != PK_GEMV) continue;
      const PhaseParams& p = prog[ph].g;
      unsigned goff = 0;
      int pbase = 0;
      for (int s = 0; s < p.n_seg; s++) {
        const int n = p.seg[s].n_rows;
        const unsigned G = (unsigned)(n + 3) / 4;
        const unsigned idx = ((unsigned)cta + grid - goff % grid) % grid;
        const int g0 = (int)(idx * G / grid), g1 = (int)((idx + 1) * G / grid);
        sr[s].row0 = 4 * g0;
        sr[s].row1 = std::min(4 * g1, n);
        const Seg& S = p.seg[s];
        sr[s].wdelta = (S.w_rows > 0 && S.w_rows < n) ? (sr[s].row0 >= S.w_row0 ? S.w_row0 : S.w_row0 - n) : 0;
        sr[s].part_base = pbase;
        pbase += sr[s].row1 - sr[s].row0;
        goff += G;
      }
    }
}

size_t step_smem_bytes(const StepArgs& a) {
  return SMEM_HEADER + (size_t)a.n_stages * a.slot_bytes + a.region_bytes + (size_t)a.part_floats * 4 + 64 * 4 +
         WARP_SCRATCH_BYTES;
}

// Q6_K segments that stream chunk by chunk (see PhaseDesc::st_chunk_rows):
// more than one chunk per row and at most one 4-row group per consumer warp.
static int chunk_rows_of(const PhaseDesc& D, int s, int grid) {
  const Seg& S = D.g.seg[s];
  const int nb = D.g.n_in / QK, max_groups = ((S.n_rows + 3) / 4 + grid - 1) / grid;
  return (S.type == W_Q6K && nb > CHUNK_BLOCKS && max_groups <= CONSUMER_WARPS) ? 4 * max_groups : 0;
}

bool plan_step(PhaseDesc* prog, int n_phases, int grid, StepArgs& a, bool chunked) {
  size_t region = 0, max_row = 0, chunk_stage = 0;
  int part = 0;
  for (int ph = 0; ph < n_phases; ph++) {
    const PhaseDesc& D = prog[ph];
    if (D.kind == PK_ATTN) {
      if (D.a.n_heads % D.a.n_kv || !D.a.part || D.a.score_stride < 1) return false;
      if (D.a.head_dim != 64 && D.a.head_dim != 128) return false;
      region = std::max(region, attn_smem_bytes(D.a.head_dim));
      continue;
    }
    const PhaseParams& P = D.g;
    if (P.n_in % QK || (P.act != ACT_RMS && P.act != ACT_F32) ||
        (P.act == ACT_RMS && (P.n_in > 8 * RMS_SLOTS * CONSUMER_WARPS * 32 || !P.rsq)))
      return false;
    const int nb = P.n_in / QK;
    region = std::max(region, act_bytes(P.n_in, P.need_q8, P.need_q6 || P.act == ACT_RMS));
    int pf = 0;
    for (int s = 0; s < P.n_seg; s++) {
      const int cr = chunked ? chunk_rows_of(D, s, grid) : 0;
      if (cr) chunk_stage = std::max(chunk_stage, (size_t)cr * Q6K_CHUNK);
      else max_row = std::max(max_row, dev_row_bytes(P.seg[s].type, nb));
      const int G = (P.seg[s].n_rows + 3) / 4;
      pf += ((G + grid - 1) / grid) * 4;
    }
    part = std::max(part, pf);
  }
  if (max_row == 0) max_row = Q6K_CHUNK;
  a.region_bytes = (int)((region + 127) & ~(size_t)127);
  a.part_floats = (part + 3) & ~3;
  const long ring =
      (long)STEP_SMEM_MAX - SMEM_HEADER - a.region_bytes - (long)a.part_floats * 4 - 64 * 4 - WARP_SCRATCH_BYTES;
  if (ring < 2L * (long)max_row) return false;
  // slots of at least 4 of the longest rows (and a whole chunk stage) while
  // that leaves 2 slots; HAKMC_STEP_STAGES overrides the slot count
  // (measurement)
  int S = (int)(ring / std::max(4L * (long)max_row, (long)chunk_stage));
  S = std::max(2, std::min(S, 8));
  if (const char* e = getenv("HAKMC_STEP_STAGES")) {
    const int v = atoi(e);
    if (v >= 2 && v <= MAX_STAGES) S = v;
  }
  long slot = (ring / S) & ~127L;
  if (slot < (long)max_row) {
    S = (int)(ring / (long)max_row);
    if (S < 2) return false;
    slot = (ring / S) & ~127L;
  }
  if (slot < (long)chunk_stage) return plan_step(prog, n_phases, grid, a, false);
  a.n_stages = S;
  a.slot_bytes = (int)slot;
  for (int ph = 0; ph < n_phases; ph++) {
    PhaseDesc& D = prog[ph];
    D.epi_rec_off = -1;
    if (D.kind != PK_GEMV) continue;
    {
      // per-thread epilogue records past the activation, when they fit
      const size_t act = (act_bytes(D.g.n_in, D.g.need_q8, D.g.need_q6 || D.g.act == ACT_RMS) + 15) & ~(size_t)15;
      const size_t recs = (size_t)CONSUMER_WARPS * 32 * EPI_RECS * sizeof(EpiRec);
      if (act + recs <= (size_t)a.region_bytes) D.epi_rec_off = (int)act;
    }
    const int nb = D.g.n_in / QK;
    for (int s = 0; s < D.g.n_seg; s++) {
      D.st_chunk_rows[s] = chunked ? chunk_rows_of(D, s, grid) : 0;
      D.st_rows[s] = D.st_chunk_rows[s] ? D.st_chunk_rows[s] : stage_rows_for(D.g.seg[s].type, nb, a.slot_bytes);
      D.st_row_bytes[s] = (int)dev_row_bytes(D.g.seg[s].type, nb);
      D.st_nch[s] = n_chunks(nb);
      D.st_rn[s] = (65536 + D.st_nch[s] - 1) / D.st_nch[s];
      if (D.st_rows[s] < 1) return false;
      // a Q4_K segment that gives each CTA a single 4-row unit runs as two
      // 2-row units on two warps: half the latency. With more units per CTA
      // the extra activation loads cost more (measured).
      const int max_groups = ((D.g.seg[s].n_rows + 3) / 4 + grid - 1) / grid;
      D.st_unit_rows[s] = (max_groups == 1 && D.g.seg[s].type == W_Q4K) ? 2 : 4;
      // Q6_K rows by the hundred per CTA (the lm_head): two rows a lane
      if (D.g.seg[s].type == W_Q6K && 4 * max_groups >= 8 * CONSUMER_WARPS && D.st_rows[s] >= 8)
        D.st_unit_rows[s] = 8;
    }
  }
  return step_smem_bytes(a) <= (size_t)STEP_SMEM_MAX;
}

template <int HD, bool TP>
static cudaError_t launch_step_hd(const StepArgs& a, int grid, cudaStream_t s) {
  static unsigned done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 32 && !(done & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(step_kernel<HD, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, STEP_SMEM_MAX);
    if (e != cudaSuccess) return e;
    done |= 1u << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = step_smem_bytes(a);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the barrier and tags need it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, step_kernel<HD, TP>, a);
}

cudaError_t launch_step(const StepArgs& a, int grid, cudaStream_t s) {
  const bool tp = a.tp_world > 1;
  if (a.head_dim == 128) return tp ? launch_step_hd<128, true>(a, grid, s) : launch_step_hd<128, false>(a, grid, s);
  if (a.head_dim == 64) return tp ? launch_step_hd<64, true>(a, grid, s) : launch_step_hd<64, false>(a, grid, s);
  return cudaErrorInvalidValue;
}

cudaError_t launch_ll_unpack(float* out, const uint64_t* in, int n, cudaStream_t s) {
  ll_unpack_kernel<<<(n + 255) / 256, 256, 0, s>>>(out, in, n);
  return cudaGetLastError();
}

}  // namespace hakm
