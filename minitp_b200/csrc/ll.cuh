// LL ("low-latency") words for exchanges between CTAs and ranks.
//
// An LL word is 8 bytes {payload (32 bit), sequence number (32 bit)} written
// by one aligned 64-bit store. Such a store is single-copy atomic, so a
// reader (64-bit loads) that sees the expected sequence number in a word also
// sees that word's payload: no memory fence and no separate flag is needed.
// Readers spin (bounded) on the words themselves. The 16-byte forms carry two
// words, each of which validates itself.
#pragma once

#include "common.cuh"

namespace mtpb {

__device__ __forceinline__ void ll_put(uint64_t* dst, uint32_t payload, uint32_t seq) {
  const uint64_t w = (uint64_t(seq) << 32) | payload;
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(dst), "l"(w) : "memory");
}
// two words {a, seq}, {b, seq} in one 16-byte store (two 64-bit elements,
// each of which validates itself)
__device__ __forceinline__ void ll_put2(uint64_t* dst, uint32_t a, uint32_t b, uint32_t seq) {
  const uint64_t w0 = (uint64_t(seq) << 32) | a, w1 = (uint64_t(seq) << 32) | b;
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(w0), "l"(w1) : "memory");
}
__device__ __forceinline__ uint2 ll_ld(const uint64_t* src) {
  uint64_t w;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(src) : "memory");
  return make_uint2(uint32_t(w), uint32_t(w >> 32));
}
// {payload0, seq0, payload1, seq1}
__device__ __forceinline__ uint4 ll_ld2(const uint64_t* src) {
  uint64_t a, b;
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(src) : "memory");
  return make_uint4(uint32_t(a), uint32_t(a >> 32), uint32_t(b), uint32_t(b >> 32));
}
__device__ __forceinline__ bool ll_ok2(const uint4& v, uint32_t seq) { return v.y == seq && v.w == seq; }

// Re-poll one word / one 16-byte pair until it carries seq (the slow path,
// kept out of line; results come back by value so the callers' arrays stay in
// registers). ok == 0 when the CTA's abort flag is raised or `budget_ns`
// passed.
struct LLSpin {
  uint4 v;
  uint32_t ok;
};
static __device__ __noinline__ LLSpin ll_spin_any(const uint64_t* src, uint32_t seq, int wide, uint64_t budget_ns,
                                           volatile int* abort, uint32_t backoff_ns) {
  LLSpin r;
  const uint64_t t0 = global_ns();
  for (uint32_t n = 1;; ++n) {
    if (backoff_ns) __nanosleep(backoff_ns);
    if (wide) {
      r.v = ll_ld2(src);
      if (ll_ok2(r.v, seq)) break;
    } else {
      const uint2 a = ll_ld(src);
      r.v = make_uint4(a.x, a.y, 0u, 0u);
      if (a.y == seq) break;
    }
    if ((n & 15) == 0 && (*abort || global_ns() - t0 > budget_ns)) {
      r.ok = 0;
      return r;
    }
  }
  r.ok = 1;
  return r;
}

// T values per LL word and their packing (bf16: two values, low half first)
template <typename T> struct LLPack;
template <> struct LLPack<float> {
  static constexpr int kPer = 1;
  __device__ static uint32_t pack(const float* v) { return __float_as_uint(v[0]); }
  __device__ static void unpack(uint32_t w, float* v) { v[0] = __uint_as_float(w); }
};
template <> struct LLPack<bf16> {
  static constexpr int kPer = 2;
  __device__ static uint32_t pack(const float* v) {
    const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(v[0]));
    const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(v[1]));
    return lo | (hi << 16);
  }
  __device__ static void unpack(uint32_t w, float* v) {
    v[0] = __uint_as_float(w << 16);
    v[1] = __uint_as_float(w & 0xFFFF0000u);
  }
};


// Poll up to NB 16-byte LL pairs (or 8-byte words) until all carry seq.
// Every round issues the loads of all that are still missing, so a round
// costs one memory round trip however many are late. False on timeout or
// abort.
template <int NB, typename Addr>
__device__ __forceinline__ bool ll_wait2(uint64_t budget_ns, uint32_t spin_ns, Addr addr, int n, uint32_t seq, uint4 (&v)[NB],
                                         volatile int* abort) {
  uint32_t pend = 0;
#pragma unroll
  for (int b = 0; b < NB; ++b)
    if (b < n) v[b] = ll_ld2(addr(b));
#pragma unroll
  for (int b = 0; b < NB; ++b)
    if (b < n && !ll_ok2(v[b], seq)) pend |= 1u << b;
  if (!pend) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (spin_ns) __nanosleep(spin_ns);
#pragma unroll
    for (int b = 0; b < NB; ++b)
      if (pend & (1u << b)) v[b] = ll_ld2(addr(b));
#pragma unroll
    for (int b = 0; b < NB; ++b)
      if ((pend & (1u << b)) && ll_ok2(v[b], seq)) pend &= ~(1u << b);
    if (!pend) return true;
    if ((it & 15) == 0 && (*abort || global_ns() - t0 > budget_ns)) return false;
  }
}
template <int NB, typename Addr>
__device__ __forceinline__ bool ll_wait1(uint64_t budget_ns, uint32_t spin_ns, Addr addr, int n, uint32_t seq, uint2 (&v)[NB],
                                         volatile int* abort) {
  uint32_t pend = 0;
#pragma unroll
  for (int b = 0; b < NB; ++b)
    if (b < n) v[b] = ll_ld(addr(b));
#pragma unroll
  for (int b = 0; b < NB; ++b)
    if (b < n && v[b].y != seq) pend |= 1u << b;
  if (!pend) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (spin_ns) __nanosleep(spin_ns);
#pragma unroll
    for (int b = 0; b < NB; ++b)
      if (pend & (1u << b)) v[b] = ll_ld(addr(b));
#pragma unroll
    for (int b = 0; b < NB; ++b)
      if ((pend & (1u << b)) && v[b].y == seq) pend &= ~(1u << b);
    if (!pend) return true;
    if ((it & 15) == 0 && (*abort || global_ns() - t0 > budget_ns)) return false;
  }
}

}  // namespace mtpb
