// Shared device helpers for the minitp_b200 kernels (sm_100a only).
//
// * 16-byte vector loads/stores and bf16 <-> fp32 conversion.
// * Programmatic dependent launch (PDL): every kernel calls pdl_launch() and
//   pdl_wait() unconditionally in every CTA, so "grid N completed" implies
//   "grids before N completed" along the whole stream.
// * System-scope release/acquire flags for NVLink peer signalling, with
//   bounded waits: a wait that runs past its budget records an error in the
//   status word and returns; it never spins forever.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef __CUDA_ARCH__
#define MTPB_HOST_ONLY 1
#endif

namespace mtpb {

constexpr int kMaxRanks = 8;

// ---------------------------------------------------------------- status
// Error bits recorded in a device status word (read by the host after a step).
enum : uint32_t {
  kStatusOk = 0,
  kStatusTimeout = 1u << 0,      // a bounded wait on peer flags ran out
  kStatusBadPosition = 1u << 1,  // a position >= KV capacity or RoPE table size
  kStatusBadToken = 1u << 2,     // a token id outside [0, vocab)
};

// ---------------------------------------------------------------- types
using bf16 = __nv_bfloat16;

template <typename T> struct VecTraits;
template <> struct VecTraits<float> { static constexpr int kElems = 4; };
template <> struct VecTraits<bf16> { static constexpr int kElems = 8; };

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(bf16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16_rn(v); }

// Round through the storage type: the value a tensor of type T would hold.
template <typename T> __device__ __forceinline__ float round_t(float v) { return to_f(from_f<T>(v)); }

// Unpack one 16-byte vector into fp32 lanes.
__device__ __forceinline__ void unpack(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ void unpack(const uint4& u, float (&f)[4]) {
  f[0] = __uint_as_float(u.x);
  f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z);
  f[3] = __uint_as_float(u.w);
}

// Pack fp32 lanes into one 16-byte vector of the storage type (round to
// nearest even for bf16).
__device__ __forceinline__ uint4 pack_vec(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i]))) |
           (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i + 1]))) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ uint4 pack_vec(const float (&f)[4]) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
}

// Streaming 16-byte load of read-only data (weights): no L1 allocation.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// 16-byte load through L1 (activations reused by every warp of the CTA).
__device__ __forceinline__ uint4 ld_vec(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// ---------------------------------------------------------------- PDL
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Bulk prefetch of [p, p + bytes) into L2 (p 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Prefetch a byte range into L2 from one thread, in pieces of at most 1 MiB.
__device__ __forceinline__ void prefetch_range_l2(const void* base, size_t bytes) {
  const char* p = static_cast<const char*>(base);
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  uintptr_t lo = (a + 15) & ~uintptr_t(15);
  uintptr_t hi = (a + bytes) & ~uintptr_t(15);
  while (lo < hi) {
    const uintptr_t left = hi - lo, cap = uintptr_t(1) << 20;
    const uint32_t n = static_cast<uint32_t>(left < cap ? left : cap);
    prefetch_l2(reinterpret_cast<const void*>(lo), n);
    lo += n;
  }
}

// ---------------------------------------------------------------- timers, flags
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}

// true when flag value `v` has reached sequence number `seq` (wrap-safe).
__device__ __forceinline__ bool seq_reached(uint32_t v, uint32_t seq) {
  return static_cast<int32_t>(v - seq) >= 0;
}

__device__ __forceinline__ uint4 ld_volatile_v4(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// One warp polls flags[s * src_stride + i] for sources s < nsrc and i < n
// until every flag reached `seq` (wrap-safe); each round issues the loads of
// every source before it tests any (16-byte loads when the flags are 16-byte
// aligned), with a short sleep between rounds so that many CTAs polling at
// once do not flood L2. After success an acquire fence at `sys` (else gpu)
// scope orders the caller's later reads after the producers' releases.
// Bounded: returns false when `timeout_ns` passed, *status became non-zero or
// *abort became non-zero. All lanes of the warp must call it; all return the
// same value.
__device__ __forceinline__ bool warp_poll_flags(const uint32_t* flags, int n, uint32_t seq, bool sys,
                                                uint32_t* status, uint64_t timeout_ns,
                                                const volatile int* abort = nullptr, int nsrc = 1,
                                                size_t src_stride = 0) {
  const int lane = threadIdx.x & 31;
  const bool vec = (reinterpret_cast<uintptr_t>(flags) & 15u) == 0 && (src_stride & 3u) == 0;
  uint64_t t0 = 0;
  uint32_t round = 0;
  while (true) {
    bool mine = true;
    for (int sidx = 0; sidx < nsrc; ++sidx) {
      const uint32_t* f = flags + size_t(sidx) * src_stride;
      if (vec) {
        for (int i = lane * 4; i < n; i += 128) {
          if (i + 3 < n) {
            const uint4 v = ld_volatile_v4(f + i);
            mine &= seq_reached(v.x, seq) & seq_reached(v.y, seq) & seq_reached(v.z, seq) & seq_reached(v.w, seq);
          } else {
            for (int j = i; j < n; ++j) mine &= seq_reached(ld_volatile_u32(f + j), seq);
          }
        }
      } else {
        for (int i = lane; i < n; i += 32) mine &= seq_reached(ld_volatile_u32(f + i), seq);
      }
    }
    if (__all_sync(0xffffffffu, mine)) break;
    ++round;
    if ((round & 7u) == 0) {
      bool bad = false;
      if (lane == 0) {
        if (t0 == 0) t0 = global_ns();
        bad = ld_volatile_u32(status) != 0 || global_ns() - t0 > timeout_ns || (abort && *abort);
      }
      if (__shfl_sync(0xffffffffu, bad ? 1 : 0, 0)) return false;
    }
    if (round > 4) __nanosleep(round > 64 ? 256 : 64);
  }
  if (sys) {
    fence_sys();
  } else {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
  }
  return true;
}

// Block-wide bounded wait until flags[i] >= seq for every i in [0, n).
// Every thread of the block must call it. Returns false (after recording
// kStatusTimeout in *status) when the budget runs out or when another wait
// already failed; the caller then skips its work and returns.
// Every thread of the block calls it; warp 0 polls, the others wait at the
// barrier. Records kStatusTimeout on failure.
__device__ __forceinline__ bool block_wait_flags(const uint32_t* flags, int n, uint32_t seq, bool sys,
                                                 uint32_t* status, uint64_t timeout_ns) {
  __shared__ int s_ok;
  if (threadIdx.x < 32) {
    const bool ok = warp_poll_flags(flags, n, seq, sys, status, timeout_ns);
    if (threadIdx.x == 0) {
      s_ok = ok ? 1 : 0;
      if (!ok) atomicOr(status, kStatusTimeout);
    }
  }
  __syncthreads();
  const bool res = s_ok != 0;
  __syncthreads();
  return res;
}

// ---------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the block; result valid in every thread. `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nwarps; ++i) t += red[i];  // fixed order: deterministic
  return t;
}

// ---------------------------------------------------------------- greedy argmax keys
// Packed argmax key, order-preserving over (value, -id):
//   key32 = bits(v) for v >= +0, (~bits(v) & 0xFFFFFFFF) - 2^31 for v < 0,
//   packed = (int64(key32) << 32) | (0xFFFFFFFF - id).
// The larger packed value has the larger logit; equal logits favour the smaller id.
// -0.0 is normalised to +0.0. NaN handling depends on `nan_wins`: the TP=1
// path follows torch.argmax (NaN beats everything, first NaN wins), the TP>1
// path maps NaN to -inf so a NaN logit cannot win.
__device__ __forceinline__ long long argmax_pack(float v, uint32_t id, bool nan_wins) {
  int64_t key;
  if (v != v) {
    if (nan_wins) {
      key = 0x7FFFFFFFll;
    } else {
      v = -__int_as_float(0x7f800000);
      uint32_t bits = __float_as_uint(v);
      key = static_cast<int64_t>(~bits & 0xFFFFFFFFu) - 0x80000000ll;
    }
  } else {
    if (v == 0.f) v = 0.f;
    uint32_t bits = __float_as_uint(v);
    key = bits < 0x80000000u ? static_cast<int64_t>(bits)
                             : static_cast<int64_t>(~bits & 0xFFFFFFFFu) - 0x80000000ll;
  }
  return static_cast<long long>((static_cast<uint64_t>(key) << 32) |
                                static_cast<uint64_t>(0xFFFFFFFFu - id));
}
__device__ __forceinline__ long long argmax_id(long long packed) {
  return static_cast<long long>(0xFFFFFFFFull - (static_cast<uint64_t>(packed) & 0xFFFFFFFFull));
}
constexpr long long kArgmaxEmpty = (-0x7FFFFFFFFFFFFFFFll - 1);

__device__ __forceinline__ long long warp_max_ll(long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    long long u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  return v;
}

}  // namespace mtpb
