// hakm_attn.cuh — GQA decode attention over the fp32 KV cache
// (src/model.c:124-142, softmax src/nn.c:20-27), as a device routine run by a
// range of threads of one CTA: the standalone attention kernel and the
// persistent decode-step kernel both call it.
//
// One work item = (kv head, group of its query heads, chunk of ATTN_CHUNK
// positions). The chunk's K and V rows are staged in shared memory with every
// load in flight at once (rows padded by 4 floats so float4 reads down a
// column of positions are bank-conflict free); scores, softmax and the
// weighted V sum run out of shared memory. Chunks combine flash-decode style
// (max / sum rescale); the last item of a (kv head, head group) to finish
// (atomic ticket) merges them. Inputs are read with L2-coherent loads:
// other SMs may have written them earlier in the same kernel.
#pragma once
#include "hakm_device.cuh"
#include "hakm_ll.cuh"

namespace hakm {

constexpr int ATTN_MAXG = 8;

// Tagged-word mode (persistent step kernel): q and the current position's k
// and v rows come from tagged words of the qkv phase (the cache rows before
// it were written in earlier steps), the output goes out as tagged words,
// and split tickets are monotonic: the item that brings the kv head's
// counter to `ticket_target` merges.
struct AttnLL {
  const uint64_t* q;
  const uint64_t* k;
  const uint64_t* v;
  uint64_t* out;
  uint32_t in_tag, out_tag;
  unsigned ticket_target;
  const int* err;
  int n_dst;                      // GPUs the output goes to (tensor parallelism), 1 otherwise
  // byte offset of GPU r's copy of `out`: out_delta[r * delta_stride] (a
  // pointer into the kernel's parameters, so no per-thread copy is made)
  const long long* out_delta;
  int delta_stride;
  long long kv_off;  // elements from the cache pointers to this sequence's cache (0: the first)
};

// Tagged output words to every destination GPU.
__device__ __forceinline__ void attn_put1(const AttnLL& T, uint64_t* p, uint64_t w) {
  if (T.n_dst == 1) { ll_st1(p, w); return; }
  for (int r = 0; r < T.n_dst; r++)
    ll_st1(reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(p) + T.out_delta[r * T.delta_stride]), w);
}
__device__ __forceinline__ void attn_put2(const AttnLL& T, uint64_t* p, float a, float b) {
  if (T.n_dst == 1) { ll_put2(p, a, b, T.out_tag); return; }
  for (int r = 0; r < T.n_dst; r++)
    ll_put2(reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(p) + T.out_delta[r * T.delta_stride]), a, b,
            T.out_tag);
}

// Most splits the merge can combine: their statistics (2 per split and
// head, plus one per head) live in the space of the staged K/V tiles.
__host__ __device__ inline int attn_max_splits(int hd, int group) {
  return (ATTN_CHUNK * (2 * hd + 4) - group) / (2 * group);
}

__host__ __device__ inline size_t attn_smem_bytes(int hd) {
  return (size_t)(ATTN_MAXG * hd + ATTN_CHUNK * (hd + 4) + ATTN_CHUNK * hd + ATTN_MAXG * ATTN_CHUNK +
                  2 * ATTN_MAXG + 4) * 4;
}

// tid in [0, nthr); sync() synchronises exactly those nthr threads. In
// tagged mode returns false if a wait for a tagged input gave up.
// Work unit u = (kv head, group of a.head_group query heads): query heads
// [u * head_group, (u + 1) * head_group), all of kv head u / (groups per kv
// head).
template <int HD, bool LL, class Sync>
__device__ bool attn_item(const AttnParams& a, int u, int split, int pos, float* sm, int tid, int nthr,
                          Sync sync, const AttnLL& T = AttnLL()) {
  bool ok = true;
  constexpr int KP = HD + 4, R4 = HD / 4;
  const int G = a.head_group;  // query heads of this item
  const int kvh = u / (a.n_heads / a.n_kv / G);
  const int kv_dim = a.n_kv * HD;
  const int lane = tid & 31, warp = tid >> 5, nw = nthr >> 5;
  float* qs = sm;                          // [G][HD]
  float* ks = qs + ATTN_MAXG * HD;         // [ATTN_CHUNK][KP]
  float* vs = ks + ATTN_CHUNK * KP;        // [ATTN_CHUNK][HD]
  float* sc = vs + ATTN_CHUNK * HD;        // [G][ATTN_CHUNK]
  float* stat_m = sc + ATTN_MAXG * ATTN_CHUNK;
  float* stat_l = stat_m + ATTN_MAXG;
  int* last = reinterpret_cast<int*>(stat_l + ATTN_MAXG);
  const int s0 = split * ATTN_CHUNK;
  const int ns = min(ATTN_CHUNK, pos + 1 - s0);  // may be <= 0 for chunks past pos

  // stage q, K and V (all loads issued before any use)
  if constexpr (LL) {
    for (int i = tid; i < G * R4; i += nthr) {
      float v4[4];
      ok &= ll_get<4>(T.q + (size_t)u * G * HD + 4 * i, T.in_tag, v4, T.err);
      reinterpret_cast<float4*>(qs)[i] = make_float4(v4[0], v4[1], v4[2], v4[3]);
    }
  } else {
    const float4* q4 = reinterpret_cast<const float4*>(a.q + (size_t)u * G * HD);
    for (int i = tid; i < G * R4; i += nthr) reinterpret_cast<float4*>(qs)[i] = __ldcg(q4 + i);
  }
  if (ns > 0) {
    const float* kb = a.k_cache + T.kv_off + (size_t)s0 * kv_dim + kvh * HD;
    const float* vb = a.v_cache + T.kv_off + (size_t)s0 * kv_dim + kvh * HD;
    for (int i = tid; i < ns * R4; i += nthr) {
      const int r = i / R4, c4 = i % R4;
      float4 kv, vv;
      if (LL && s0 + r == pos) {
        float k4[4], w4[4];
        ok &= ll_get<4>(T.k + kvh * HD + 4 * c4, T.in_tag, k4, T.err);
        ok &= ll_get<4>(T.v + kvh * HD + 4 * c4, T.in_tag, w4, T.err);
        kv = make_float4(k4[0], k4[1], k4[2], k4[3]);
        vv = make_float4(w4[0], w4[1], w4[2], w4[3]);
      } else {
        kv = __ldcg(reinterpret_cast<const float4*>(kb + (size_t)r * kv_dim + 4 * c4));
        vv = __ldcg(reinterpret_cast<const float4*>(vb + (size_t)r * kv_dim + 4 * c4));
      }
      *reinterpret_cast<float4*>(ks + r * KP + 4 * c4) = kv;
      *reinterpret_cast<float4*>(vs + r * HD + 4 * c4) = vv;
    }
  }
  sync();

  // scores: one (head, position) pair per thread iteration, positions fastest
  for (int i = tid; i < G * ATTN_CHUNK; i += nthr) {
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
  sync();

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
  sync();

  // weighted V: one (head, 4 dims) pair per thread iteration
  const bool single = (a.n_split == 1);
  for (int i = tid; i < G * R4; i += nthr) {
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
      if constexpr (LL) {
        uint64_t* dst = T.out + (size_t)(u * G + g) * HD + 4 * c4;
        attn_put2(T, dst, o.x, o.y);
        attn_put2(T, dst + 2, o.z, o.w);
      } else {
        *reinterpret_cast<float4*>(a.out + (size_t)(u * G + g) * HD + 4 * c4) = o;
      }
    } else {
      float* pp = a.part + ((size_t)(u * a.n_split + split) * G + g) * (HD + 2);
      pp[2 + 4 * c4] = acc.x; pp[3 + 4 * c4] = acc.y; pp[4 + 4 * c4] = acc.z; pp[5 + 4 * c4] = acc.w;
      if (c4 == 0) { pp[0] = ns > 0 ? stat_m[g] : -CUDART_INF_F; pp[1] = ns > 0 ? stat_l[g] : 0.f; }
    }
  }
  if (!single) {
    sync();
    if (tid == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(&a.counters[u], 1u);
      *last = LL ? (prev + 1u == T.ticket_target) : (prev == (unsigned)a.n_split - 1);
    }
    sync();
    if (*last) {
      __threadfence();
      // merge: every split's (max, exp-sum) into shared memory at once,
      // one rescale weight per (split, head), then the weighted sum of the
      // partial vectors with independent L2 loads. The staged K/V tiles are
      // no longer needed: their space holds the statistics.
      const int ns_all = a.n_split * G;
      float* mw = ks;               // [n_split * G]: split max, then its weight
      float* ls = ks + ns_all;      // [n_split * G]: split exp-sum
      float* head_l = ls + ns_all;  // [G]: merged exp-sum
      for (int i = tid; i < ns_all; i += nthr) {
        const float* pp = a.part + ((size_t)u * a.n_split * G + i) * (HD + 2);
        mw[i] = __ldcg(pp);
        ls[i] = __ldcg(pp + 1);
      }
      sync();
      for (int g = warp; g < G; g += nw) {
        float m = -CUDART_INF_F;
        for (int sp = lane; sp < a.n_split; sp += 32) m = fmaxf(m, mw[sp * G + g]);
        m = warp_max(m);
        float l = 0.f;
        for (int sp = lane; sp < a.n_split; sp += 32) {
          const float li = ls[sp * G + g];
          const float f = li > 0.f ? expf(mw[sp * G + g] - m) : 0.f;
          mw[sp * G + g] = f;
          l += li * f;
        }
        l = warp_sum(l);
        if (lane == 0) head_l[g] = l;
      }
      sync();
      for (int i = tid; i < G * HD; i += nthr) {
        const int g = i / HD, d = i % HD;
        const float* pp = a.part + ((size_t)u * a.n_split * G + g) * (HD + 2) + 2 + d;
        float acc = 0.f;
        for (int sp = 0; sp < a.n_split; sp++) {
          const float f = mw[sp * G + g];
          if (f != 0.f) acc = fmaf(f, __ldcg(pp + (size_t)sp * G * (HD + 2)), acc);
        }
        const float o = acc / head_l[g];
        if constexpr (LL) attn_put1(T, T.out + (u * G + g) * HD + d, ll_word(o, T.out_tag));
        else a.out[(u * G + g) * HD + d] = o;
      }
      if (!LL && tid == 0) a.counters[u] = 0u;
    }
    sync();
  }
  return ok;
}

}  // namespace hakm
