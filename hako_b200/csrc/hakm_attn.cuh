// hakm_attn.cuh — GQA decode attention over the fp32 KV cache
// (src/model.c:124-142, softmax src/nn.c:20-27) with the reference's own
// roundings, as a device routine run by a range of threads of one CTA: the
// standalone attention kernel and the persistent decode-step kernel both
// call it.
//
// The reference scores every position, takes one softmax over all of them
// and then accumulates the weighted V rows position by position, with an FMA
// per dimension. Those orders are kept:
//  - score t = (q . k_t) * scale, the dot as gcc vectorizes it: lane i % 8
//    of an 8-lane accumulator sums the rounded products q[i]*k[i] in order,
//    then the lanes fold (fold8_lanes);
//  - softmax: the max, exp(s - max) by element index through libmvec's
//    8-wide, then 4-wide, then glibc's scalar expf (exp_softmax), the sum in
//    the vectorized loop's order, one IEEE reciprocal and a multiply;
//  - out[d] = fma(p_t, v_t[d], out[d]) for t = 0 .. pos, from +0.
// Work unit = (query head, slice of ATTN_SLICE dimensions): every unit
// scores its head's positions itself (the score work is small next to the
// V chain, which is sequential in t) and runs the V chains of its slice,
// one dimension per lane of warp 0, while the other warps stage the next
// tile of V rows in shared memory. Scores live in a global scratch row per
// unit (score_stride floats), or in shared memory past the V tiles when the
// caller has room for them (tagged-word mode, AttnLL::sc_cap). Inputs are
// read with L2-coherent loads: other SMs may have written them earlier in
// the same kernel.
#pragma once
#include "hakm_device.cuh"
#include "hakm_exact.cuh"
#include "hakm_ll.cuh"

namespace hakm {

constexpr int ATTN_VT = 64;  // positions per staged V tile

// Tagged-word mode (persistent step kernel): q and the current position's k
// and v rows come from tagged words of the qkv phase (the cache rows before
// it were written in earlier steps), and the output goes out as tagged words.
struct AttnLL {
  const uint64_t* q;
  const uint64_t* k;
  const uint64_t* v;
  uint64_t* out;
  uint32_t in_tag, out_tag;
  const int* err;
  int n_dst;                      // GPUs the output goes to (tensor parallelism), 1 otherwise
  // byte offset of GPU r's copy of `out`: out_delta[r * delta_stride] (a
  // pointer into the kernel's parameters, so no per-thread copy is made)
  const long long* out_delta;
  int delta_stride;
  long long kv_off;  // elements from the cache pointers to this sequence's cache (0: the first)
  // shared floats past the attention tiles (attn_smem_bytes): rows of at
  // most this many positions keep their scores there instead of in the
  // global scratch row
  int sc_cap = 0;
};

// Tagged output word to every destination GPU.
__device__ __forceinline__ void attn_put1(const AttnLL& T, uint64_t* p, uint64_t w) {
  if (T.n_dst == 1) { ll_st1(p, w); return; }
  for (int r = 0; r < T.n_dst; r++)
    ll_st1(reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(p) + T.out_delta[r * T.delta_stride]), w);
}

__host__ __device__ inline size_t attn_smem_bytes(int hd) {
  return (size_t)(hd + 64 + 2 * ATTN_VT * ATTN_SLICE) * 4;
}

// Softmax of sc[0 .. n) in place (src/nn.c:20-27 as built): the max, the
// exps by element index (exp_softmax), their sum in the vectorized loop's
// order (8 lane chains over the first 8*floor(n/8) elements, folded to 4 by
// adding lanes k and k+4, one 4-lane step when at least 4 remain, the fold
// of those, then scalar adds), one IEEE reciprocal and a multiply. Run by
// threads [0, nthr) (a multiple of 32) that sync() synchronises; red: 33
// floats of shared scratch. Ends with a sync().
template <class Sync>
__device__ __forceinline__ void softmax_exact(float* sc, int n, float* red, int tid, int nthr, Sync sync) {
  const int lane = tid & 31, warp = tid >> 5, nw = nthr >> 5;
  float mx = -CUDART_INF_F;
  for (int t = tid; t < n; t += nthr) mx = fmaxf(mx, sc[t]);
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  sync();
  mx = red[0];
  for (int w = 1; w < nw; w++) mx = fmaxf(mx, red[w]);
  for (int t = tid; t < n; t += nthr) sc[t] = exp_softmax(__fsub_rn(sc[t], mx), t, n);
  sync();
  if (warp == 0) {
    const int n8 = n & ~7, rem = n - n8;
    float c = 0.f;
    if (lane < 8)
      for (int t = lane; t < n8; t += 8) c = __fadd_rn(c, sc[t]);
    // lanes 0..3: c_k + c_{k+4}, the 4 lanes the remainder step continues
    const float c4 = __fadd_rn(c, __shfl_xor_sync(0xffffffffu, c, 4));
    const float u2 = __fadd_rn(c4, __shfl_xor_sync(0xffffffffu, c4, 2));
    float sum = __fadd_rn(u2, __shfl_xor_sync(0xffffffffu, u2, 1));
    if (rem >= 4) {
      const float uk = __fadd_rn(sc[n8 + (lane & 3)], c4);
      const float a2 = __fadd_rn(uk, __shfl_xor_sync(0xffffffffu, uk, 2));
      sum = __fadd_rn(a2, __shfl_xor_sync(0xffffffffu, a2, 1));
    }
    if (lane == 0) {
      for (int t = rem >= 4 ? n8 + 4 : n8; t < n; t++) sum = __fadd_rn(sum, sc[t]);
      red[32] = __fdiv_rn(1.0f, sum);
    }
  }
  sync();
  const float inv = red[32];
  for (int t = tid; t < n; t += nthr) sc[t] = __fmul_rn(sc[t], inv);
  sync();
}

// tid in [0, nthr), nthr a multiple of 32 and at least 64; sync()
// synchronises exactly those nthr threads. In tagged mode returns false if a
// wait for a tagged input gave up.
template <int HD, bool LL, class Sync>
__device__ bool attn_item(const AttnParams& a, int unit, int pos, float* sm, int tid, int nthr, Sync sync,
                          const AttnLL& T = AttnLL()) {
  constexpr int NSL = HD / ATTN_SLICE;
  const int h = unit / NSL, sl = unit % NSL;
  const int kvh = h / (a.n_heads / a.n_kv);
  const int kv_dim = a.n_kv * HD, n = pos + 1;
  const int lane = tid & 31, warp = tid >> 5, nw = nthr >> 5;
  float* qs = sm;          // [HD]
  float* red = qs + HD;    // [64]
  float* vt = red + 64;    // [2][ATTN_VT][ATTN_SLICE]
  float* sc = a.part + (size_t)unit * a.score_stride;
  if (LL && n <= T.sc_cap) sc = vt + 2 * ATTN_VT * ATTN_SLICE;
  const long long kv_off = LL ? T.kv_off : 0;
  const float* kb = a.k_cache + kv_off + kvh * HD;
  const float* vb = a.v_cache + kv_off + kvh * HD + sl * ATTN_SLICE;
  bool ok = true;
  const int l = lane & 7;

  // V rows of the first tile into buffer 0; in tagged-word mode the row of
  // this position comes from a tagged word of the qkv phase and waits for
  // the softmax (fill_pos_row), the others are cache rows of earlier steps
  // and load at once
  auto stage = [&](int tile, int buf, int t_lo, int t_n, bool skip_pos) {
    float* dst = vt + buf * ATTN_VT * ATTN_SLICE;
    const int t0 = tile * ATTN_VT, cnt = min(ATTN_VT, n - t0);
    for (int i = t_lo; i < cnt * (ATTN_SLICE / 4); i += t_n) {
      const int r = i / (ATTN_SLICE / 4), c4 = i % (ATTN_SLICE / 4), t = t0 + r;
      float4 v;
      if (LL && t == pos) {
        if (skip_pos) continue;
        float w[4];
        ok &= ll_get<4>(T.v + kvh * HD + sl * ATTN_SLICE + 4 * c4, T.in_tag, w, T.err);
        v = make_float4(w[0], w[1], w[2], w[3]);
      } else {
        v = __ldcg(reinterpret_cast<const float4*>(vb + (size_t)t * kv_dim) + c4);
      }
      reinterpret_cast<float4*>(dst)[i] = v;
    }
  };
  if constexpr (LL) {
    // the K rows this thread will score into L2 (no registers held across
    // the wait for q): lanes 0..HD/32-1 of each position one 128-byte line
    if (l < HD / 32)
      for (int t = 4 * warp + (lane >> 3); t < n; t += 4 * nw)
        if (t != pos) asm volatile("prefetch.global.L2 [%0];" ::"l"(kb + (size_t)t * kv_dim + 32 * l));
    stage(0, 0, tid, nthr, true);
  }

  for (int i = tid; i < HD; i += nthr) {
    float v;
    if constexpr (LL) ok &= ll_get1(T.q + (size_t)h * HD + i, T.in_tag, v, T.err);
    else v = __ldcg(a.q + (size_t)h * HD + i);
    qs[i] = v;
  }
  sync();

  // scores: lane (p, l) = (lane / 8, lane % 8) runs chain l of position
  // 4 * (iteration) + p; the 8 chains of a position fold over its lanes
  {
    float qv[HD / 8];
#pragma unroll
    for (int j = 0; j < HD / 8; j++) qv[j] = qs[8 * j + l];
    for (int t0 = 4 * warp; t0 < n; t0 += 4 * nw) {
      const int t = t0 + (lane >> 3);
      float acc = 0.f;
      if (t < n) {
        float kv[HD / 8];
        if (LL && t == pos) {
          ok &= ll_get_strided<HD / 8>(T.k + kvh * HD + l, 8, T.in_tag, kv, T.err);
        } else {
          const float* kr = kb + (size_t)t * kv_dim + l;
#pragma unroll
          for (int j = 0; j < HD / 8; j++) kv[j] = __ldcg(kr + 8 * j);
        }
#pragma unroll
        for (int j = 0; j < HD / 8; j++) acc = __fadd_rn(acc, __fmul_rn(qv[j], kv[j]));
      }
      const float dot = fold8_lanes(acc);
      if (t < n && l == 0) sc[t] = __fmul_rn(dot, a.scale);
    }
  }
  sync();

  softmax_exact(sc, n, red, tid, nthr, sync);

  // weighted V: warp 0 lane d runs out[d] over the staged tiles; the other
  // warps stage tile i + 1 while it works on tile i
  const int n_tiles = (n + ATTN_VT - 1) / ATTN_VT;
  if constexpr (LL) {
    // tile 0 was staged before q but for this position's row
    if (pos < ATTN_VT && tid < ATTN_SLICE / 4) {
      float w[4];
      ok &= ll_get<4>(T.v + kvh * HD + sl * ATTN_SLICE + 4 * tid, T.in_tag, w, T.err);
      reinterpret_cast<float4*>(vt)[pos * (ATTN_SLICE / 4) + tid] = make_float4(w[0], w[1], w[2], w[3]);
    }
  } else {
    stage(0, 0, tid, nthr, false);
  }
  sync();
  float acc = 0.f;
  for (int tile = 0; tile < n_tiles; tile++) {
    if (warp == 0) {
      const float* src = vt + (tile & 1) * ATTN_VT * ATTN_SLICE + lane;
      const int t0 = tile * ATTN_VT, cnt = min(ATTN_VT, n - t0);
      for (int r = 0; r < cnt; r++) acc = __fmaf_rn(sc[t0 + r], src[r * ATTN_SLICE], acc);
    } else if (tile + 1 < n_tiles) {
      stage(tile + 1, (tile + 1) & 1, tid - 32, nthr - 32, false);
    }
    sync();
  }
  if (warp == 0) {
    const int o = h * HD + sl * ATTN_SLICE + lane;
    if constexpr (LL) attn_put1(T, T.out + o, ll_word(acc, T.out_tag));
    else a.out[o] = acc;
  }
  return ok;
}

}  // namespace hakm
