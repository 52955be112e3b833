// hakm_ll.cuh — tagged words for exchanging vectors between the phases of
// the persistent step kernel without a grid barrier.
//
// A word is (tag << 32) | float bits, written and read as single 8-byte
// relaxed accesses at system scope (pairs of words as one 16-byte vector
// access, each aligned 8-byte element single-copy atomic), the flag-in-data
// scheme of NCCL's LL protocol. System scope, because with tensor
// parallelism the writer may sit on another GPU (peer stores over NVLink). A reader that sees the
// tag it expects sees the value written with it; it polls until every word
// it needs carries that tag. Tags grow by one per phase instance, so a stale
// word can never match.
#pragma once
#include <cstdint>

#include "hakm_device.cuh"

namespace hakm {

constexpr long long LL_WAIT_LIMIT = 4000000000LL;  // ~2 s of SM clock

__device__ __forceinline__ bool ll_aborted(const int* err) { return *(volatile const int*)err != 0; }

__device__ __forceinline__ uint64_t ll_word(float v, uint32_t tag) {
  return ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
}
__device__ __forceinline__ float ll_value(uint64_t w) { return __uint_as_float((uint32_t)w); }
__device__ __forceinline__ bool ll_has(uint64_t w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }

__device__ __forceinline__ void ll_ld2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ void ll_st2(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ll_st1(uint64_t* p, uint64_t a) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(a) : "memory");
}
__device__ __forceinline__ void ll_put2(uint64_t* p, float a, float b, uint32_t tag) {
  ll_st2(p, ll_word(a, tag), ll_word(b, tag));
}

// N (even) consecutive tagged floats from p (16-byte aligned). While the
// first word lacks `tag` only that word is polled (8 bytes per poll, a short
// sleep between polls), so waiting readers put little load on L2; then all N
// are read and any word still without the tag is read again. Gives up
// (values 0, returns false) after LL_WAIT_LIMIT cycles or once the error flag
// is set (looked at every 2^12 cycles). Everything stays inline: a call
// would save the caller's registers to local memory.
template <int N>
__device__ __forceinline__ bool ll_get(const uint64_t* p, uint32_t tag, float* out, const int* err) {
  uint64_t w[N];
  bool ok = true;
#pragma unroll
  for (int i = 0; i < N; i += 2) {
    ll_ld2(p + i, w[i], w[i + 1]);
    ok = ok && ll_has(w[i], tag) && ll_has(w[i + 1], tag);
  }
  if (!ok) {
    const long long t0 = clock64();
    long long next = t0 + 4096;
    for (;;) {
      if (!ll_has(w[0], tag)) {
        __nanosleep(64);
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w[0]) : "l"(p) : "memory");
      } else {
        ok = true;
#pragma unroll
        for (int i = 0; i < N; i += 2) {
          if (!(ll_has(w[i], tag) && ll_has(w[i + 1], tag))) ll_ld2(p + i, w[i], w[i + 1]);
          ok = ok && ll_has(w[i], tag) && ll_has(w[i + 1], tag);
        }
        if (ok) break;
      }
      const long long now = clock64();
      if (now > next) {
        if (ll_aborted(err) || now - t0 > LL_WAIT_LIMIT) {
#pragma unroll
          for (int i = 0; i < N; i++) out[i] = 0.f;
          return false;
        }
        next = now + 4096;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < N; i++) out[i] = ll_value(w[i]);
  return true;
}

// Split form of ll_get<8> for several slots in flight at once: ll_issue8
// starts the loads, ll_finish8 checks the tags and polls what is missing.
__device__ __forceinline__ void ll_issue8(const uint64_t* p, uint64_t w[8]) {
#pragma unroll
  for (int i = 0; i < 8; i += 2) ll_ld2(p + i, w[i], w[i + 1]);
}
__device__ __forceinline__ bool ll_finish8(const uint64_t* p, uint32_t tag, uint64_t w[8], float* out,
                                           const int* err) {
  bool ok = true;
#pragma unroll
  for (int i = 0; i < 8; i++) ok = ok && ll_has(w[i], tag);
  if (!ok) return ll_get<8>(p, tag, out, err);
#pragma unroll
  for (int i = 0; i < 8; i++) out[i] = ll_value(w[i]);
  return true;
}

// N tagged floats p[0], p[stride], ..., p[(N-1)*stride]: all N loads in
// flight before the first tag check (a loop of ll_get1 would wait for each
// load's answer before it issues the next), then only the words still
// lacking the tag are read again, a short sleep between rounds. Gives up as
// ll_get does.
template <int N>
__device__ __forceinline__ bool ll_get_strided(const uint64_t* p, int stride, uint32_t tag, float* out,
                                               const int* err) {
  uint64_t w[N];
#pragma unroll
  for (int i = 0; i < N; i++)
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w[i]) : "l"(p + (size_t)i * stride) : "memory");
  bool ok = true;
#pragma unroll
  for (int i = 0; i < N; i++) ok = ok && ll_has(w[i], tag);
  if (!ok) {
    const long long t0 = clock64();
    long long next = t0 + 4096;
    for (;;) {
      __nanosleep(64);
#pragma unroll
      for (int i = 0; i < N; i++)
        if (!ll_has(w[i], tag))
          asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w[i]) : "l"(p + (size_t)i * stride) : "memory");
      ok = true;
#pragma unroll
      for (int i = 0; i < N; i++) ok = ok && ll_has(w[i], tag);
      if (ok) break;
      const long long now = clock64();
      if (now > next) {
        if (ll_aborted(err) || now - t0 > LL_WAIT_LIMIT) {
#pragma unroll
          for (int i = 0; i < N; i++) out[i] = 0.f;
          return false;
        }
        next = now + 4096;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < N; i++) out[i] = ll_value(w[i]);
  return true;
}

// One tagged float (p 8-byte aligned).
__device__ __forceinline__ bool ll_get1(const uint64_t* p, uint32_t tag, float& out, const int* err) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  if (!ll_has(w, tag)) {
    const long long t0 = clock64();
    long long next = t0 + 4096;
    while (!ll_has(w, tag)) {
      __nanosleep(64);
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
      const long long now = clock64();
      if (now > next) {
        if (ll_aborted(err) || now - t0 > LL_WAIT_LIMIT) { out = 0.f; return false; }
        next = now + 4096;
      }
    }
  }
  out = ll_value(w);
  return true;
}

}  // namespace hakm
