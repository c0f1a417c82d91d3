// Row-wise finish of a flag-protocol AllReduce site: the rank-order sum of
// the partial rows (one-shot) or the owner's reduced slices (two-shot, see
// comm.cuh), then bias, residual and RMSNorm, with 16-byte vectors and every
// load of a row issued before its arithmetic. Shared by the consume pass of
// the model's collective sites (prefill, many-row decode) and the standalone
// fused AllReduce + residual + RMSNorm.
//
// Arithmetic (the reference's rounding points): o = T(sum_r partial_r) in
// rank order, o = T(o + bias), x = T(residual + o), then
// y = T((x * rsqrt(mean(x^2) + eps)) * gain) with the mean from a block sum in
// a fixed order. Every rank computes identical bits.
#pragma once

#include "comm.cuh"

namespace mtpb {

constexpr int kArRowThreads = 256;
constexpr int kArRowVecs = 4;  // 16-byte vectors per thread: H <= 4 * 256 * (8 bf16 | 4 fp32)

// Can a row of H values go through the vector path?
template <typename T>
__host__ __device__ inline bool ar_rows_vec_ok(int H) {
  constexpr int VE = sizeof(T) == 2 ? 8 : 4;
  return H % VE == 0 && H / VE <= kArRowVecs * kArRowThreads;
}

// Two-shot reduce step: this rank's slice (ts columns from rank * ts) of row
// m, summed over the sources' slots in rank order, rounded to T and stored
// into data[chan][par][rank] of every rank. Call from all threads of the CTA.
template <typename T>
__device__ __forceinline__ void ar_reduce_slice(const Comm& c, int chan, int par, int ts, int m, int H) {
  constexpr int VE = VecTraits<T>::kElems;
  const int v0 = c.rank * (ts / VE), v1 = min(H / VE, v0 + ts / VE);
  for (int v = v0 + int(threadIdx.x); v < v1; v += blockDim.x) {
    const size_t off = size_t(m) * H + size_t(v) * VE;
    uint4 u[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < c.world)
        u[r] = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(c.data(c.rank, chan, par, r)) + off));
    float s[VE];
#pragma unroll
    for (int e = 0; e < VE; ++e) s[e] = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r < c.world) {
        float f[VE];
        unpack(u[r], f);
#pragma unroll
        for (int e = 0; e < VE; ++e) s[e] += f[e];
      }
    }
    const uint4 o = pack_vec(s);
    for (int d = 0; d < c.world; ++d)
      *reinterpret_cast<uint4*>(reinterpret_cast<T*>(c.data(d, chan, par, c.rank)) + off) = o;
  }
}

// Finish row m: the AllReduce result from the site's slots (or from `direct`
// when there is no exchange), + bias, + residual -> res_out, and the RMSNorm
// -> out_norm (when gain is set). Call from all threads of the CTA.
template <typename T>
__device__ __forceinline__ void ar_finish_row(const Comm& c, int chan, int par, int ts, const T* direct, int m, int H,
                                              const T* bias, const T* res_in, T* res_out, const T* gain, float eps,
                                              T* out_norm, float* red) {
  constexpr int VE = VecTraits<T>::kElems;
  const int nv = H / VE;
  float x[kArRowVecs][VE];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kArRowVecs; ++i) {
    const int v = int(threadIdx.x) + i * int(blockDim.x);
    if (v < nv) {
      const size_t off = size_t(m) * H + size_t(v) * VE;
      float o[VE];
      if (direct) {
        unpack(ld_vec(direct + off), o);
      } else if (ts > 0) {
        const int own = ts_owner(v * VE, ts, c.world);
        unpack(__ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(c.data(c.rank, chan, par, own)) + off)),
               o);
      } else {
        uint4 u[kMaxRanks];
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
          if (r < c.world)
            u[r] = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(c.data(c.rank, chan, par, r)) + off));
#pragma unroll
        for (int e = 0; e < VE; ++e) o[e] = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r) {
          if (r < c.world) {
            float f[VE];
            unpack(u[r], f);
#pragma unroll
            for (int e = 0; e < VE; ++e) o[e] += f[e];
          }
        }
#pragma unroll
        for (int e = 0; e < VE; ++e) o[e] = round_t<T>(o[e]);
      }
      if (bias) {
        float b[VE];
        unpack(ld_vec(bias + size_t(v) * VE), b);
#pragma unroll
        for (int e = 0; e < VE; ++e) o[e] = round_t<T>(o[e] + b[e]);
      }
      if (res_in) {
        float rr[VE];
        unpack(ld_vec(res_in + off), rr);
#pragma unroll
        for (int e = 0; e < VE; ++e) o[e] = round_t<T>(rr[e] + o[e]);
      }
#pragma unroll
      for (int e = 0; e < VE; ++e) {
        x[i][e] = o[e];
        ss += o[e] * o[e];
      }
      *reinterpret_cast<uint4*>(res_out + off) = pack_vec(o);
    }
  }
  if (!gain) return;
  const float tot = block_sum(ss, red);
  const float rinv = rsqrtf(tot / float(H) + eps);
#pragma unroll
  for (int i = 0; i < kArRowVecs; ++i) {
    const int v = int(threadIdx.x) + i * int(blockDim.x);
    if (v < nv) {
      float g[VE], y[VE];
      unpack(ld_vec(gain + size_t(v) * VE), g);
#pragma unroll
      for (int e = 0; e < VE; ++e) y[e] = __fmul_rn(__fmul_rn(x[i][e], rinv), g[e]);
      *reinterpret_cast<uint4*>(out_norm + size_t(m) * H + size_t(v) * VE) = pack_vec(y);
    }
  }
  __syncthreads();  // red is reused by the next row
}

}  // namespace mtpb
