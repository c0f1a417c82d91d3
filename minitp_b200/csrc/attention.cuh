// Split-KV grouped-query attention over the rank's local heads.
//
// Row m of q is token t = m % tpr of batch row b = m / tpr at absolute
// position pos = pos0 + t (pos0 from device memory in the captured decode
// step). It attends to cache positions [0, pos] of its KV head: the causal
// rule of the reference for decode (no mask), prefill (is_causal) and chunked
// prefill (tril(diagonal=cache_len)). The `G = hq / hkv` query heads sharing
// one KV head are processed by the same CTA, so K/V bytes are read once per
// group (no expand / repeat_interleave copies).
//
// grid = (nsplit, hkv, M); each CTA covers one contiguous slice of the
// positions. With nsplit > 1 the partial softmax states (max, sum, o) go to
// scratch and the last CTA of each (row, kv head) merges them.
#pragma once

#include "comm.cuh"

namespace mtpb {

struct AttnParams {
  const void* q;  // [M][hq*hd]
  const void* k_cache;
  const void* v_cache;  // [B][hkv][cap][hd]
  void* out;            // [M][hq*hd]
  int M, tpr, hq, hkv, cap;
  const int* pos_ptr;
  int pos_base;
  float scale;
  int nsplit;
  int chunk_cap;  // max positions per split (sizes the score buffer)
  float* part_o;  // [M][hq][nsplit][hd]
  float* part_ml;  // [M][hq][nsplit][2]
  uint32_t* counters;  // [M][hkv], zero between launches
  uint32_t* status;
};

constexpr int kAttnThreads = 128;
constexpr int kAttnGB = 4;  // heads per PV pass
constexpr int kAttnU = 4;   // K / V rows (and merged splits) whose loads are issued together

template <typename T, int HD>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnParams p) {
  constexpr int VE = VecTraits<T>::kElems;
  constexpr int LPP = HD / VE;  // lanes per key row
  static_assert(LPP >= 1 && LPP <= 32 && (32 % LPP) == 0, "unsupported head_dim");
  constexpr int PPW = 32 / LPP;  // key rows per warp pass
  constexpr int DCH = HD / VE;   // 16-byte chunks per row
  constexpr int NW = kAttnThreads / 32;
  constexpr int NPL = kAttnThreads / DCH;  // position lanes in the PV pass

  extern __shared__ __align__(16) float sm[];
  const int G = p.hq / p.hkv;
  float* qf = sm;                       // [G][HD]
  float* sc = qf + G * HD;              // [G][chunk_cap]
  float* ml = sc + G * p.chunk_cap;     // [G][2]
  float* ro = ml + 2 * G;               // [NPL][kAttnGB][HD]
  __shared__ int s_last;

  pdl_launch();
  pdl_wait();

  const int split = blockIdx.x, kvh = blockIdx.y, m = blockIdx.z;
  const int b = m / p.tpr, t = m - b * p.tpr;
  const int pos = (p.pos_ptr ? *p.pos_ptr : p.pos_base) + t;
  if (pos < 0 || pos >= p.cap) {
    if (threadIdx.x == 0) atomicOr(p.status, kStatusBadPosition);
    return;
  }
  const int L = pos + 1;
  const int chunk = (L + p.nsplit - 1) / p.nsplit;
  const int s0 = min(L, split * chunk), s1 = min(L, s0 + chunk);
  const int n = s1 - s0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const T* kbase = static_cast<const T*>(p.k_cache) + (size_t(b) * p.hkv + kvh) * p.cap * HD;
  const T* vbase = static_cast<const T*>(p.v_cache) + (size_t(b) * p.hkv + kvh) * p.cap * HD;
  const T* qrow = static_cast<const T*>(p.q) + size_t(m) * p.hq * HD + size_t(kvh) * G * HD;
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) qf[i] = to_f(qrow[i]);
  __syncthreads();

  // scores: LPP lanes per key row, PPW rows per warp pass; the K rows of
  // kAttnU passes are loaded before any of them is used
  {
    const int pg = lane / LPP, li = lane - pg * LPP;
    for (int rb = s0 + warp * PPW; rb < s1; rb += NW * PPW * kAttnU) {
      uint4 kv[kAttnU];
#pragma unroll
      for (int u = 0; u < kAttnU; ++u) {
        const int r = rb + u * NW * PPW + pg;
        kv[u] = r < s1 ? ld_vec(kbase + size_t(r) * HD + li * VE) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kAttnU; ++u) {
        const int r = rb + u * NW * PPW + pg;
        const bool ok = r < s1;
        float kf[VE];
        unpack(kv[u], kf);
        for (int g = 0; g < G; ++g) {
          const float* qg = qf + g * HD + li * VE;
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < VE; ++e) d = fmaf(kf[e], qg[e], d);
#pragma unroll
          for (int o = LPP / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
          if (ok && li == 0) sc[g * p.chunk_cap + (r - s0)] = d * p.scale;
        }
      }
    }
  }
  __syncthreads();

  // softmax statistics per head (one warp per head)
  for (int g = warp; g < G; g += NW) {
    float* s = sc + g * p.chunk_cap;
    float mx = -INFINITY;
    for (int i = lane; i < n; i += 32) mx = fmaxf(mx, s[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float e = expf(s[i] - mx);
      s[i] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    if (lane == 0) {
      ml[2 * g] = mx;
      ml[2 * g + 1] = sum;
    }
  }
  __syncthreads();

  // o[g][:] = sum_r p[g][r] * v[r][:], kAttnGB heads per pass
  const int dc = threadIdx.x % DCH, pl = threadIdx.x / DCH;
  const bool single = p.nsplit == 1;
  for (int g0 = 0; g0 < G; g0 += kAttnGB) {
    float acc[kAttnGB][VE];
#pragma unroll
    for (int gg = 0; gg < kAttnGB; ++gg)
#pragma unroll
      for (int e = 0; e < VE; ++e) acc[gg][e] = 0.f;
    for (int rb = pl; rb < n; rb += NPL * kAttnU) {
      uint4 vv[kAttnU];
#pragma unroll
      for (int u = 0; u < kAttnU; ++u) {
        const int r = rb + u * NPL;
        vv[u] = r < n ? ld_vec(vbase + size_t(s0 + r) * HD + dc * VE) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kAttnU; ++u) {
        const int r = rb + u * NPL;
        if (r < n) {
          float vf[VE];
          unpack(vv[u], vf);
#pragma unroll
          for (int gg = 0; gg < kAttnGB; ++gg) {
            if (g0 + gg < G) {
              const float pr = sc[(g0 + gg) * p.chunk_cap + r];
#pragma unroll
              for (int e = 0; e < VE; ++e) acc[gg][e] = fmaf(pr, vf[e], acc[gg][e]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int gg = 0; gg < kAttnGB; ++gg)
#pragma unroll
      for (int e = 0; e < VE; ++e) ro[(pl * kAttnGB + gg) * HD + dc * VE + e] = acc[gg][e];
    __syncthreads();
    for (int i = threadIdx.x; i < kAttnGB * HD; i += blockDim.x) {
      const int gg = i / HD, d = i - gg * HD;
      const int g = g0 + gg;
      if (g < G) {
        float o = 0.f;
        for (int q = 0; q < NPL; ++q) o += ro[(q * kAttnGB + gg) * HD + d];
        const int head = kvh * G + g;
        if (single) {
          static_cast<T*>(p.out)[size_t(m) * p.hq * HD + size_t(head) * HD + d] =
              from_f<T>(o / ml[2 * g + 1]);
        } else {
          p.part_o[((size_t(m) * p.hq + head) * p.nsplit + split) * HD + d] = o;
        }
      }
    }
    __syncthreads();
  }
  if (single) return;

  // publish (max, sum) and merge in the last CTA of this (row, kv head)
  for (int g = threadIdx.x; g < G; g += blockDim.x) {
    const int head = kvh * G + g;
    float* d = p.part_ml + ((size_t(m) * p.hq + head) * p.nsplit + split) * 2;
    d[0] = n > 0 ? ml[2 * g] : -INFINITY;
    d[1] = n > 0 ? ml[2 * g + 1] : 0.f;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* ctr = p.counters + size_t(m) * p.hkv + kvh;
    const uint32_t old = atomicAdd(ctr, 1u);
    s_last = old == uint32_t(p.nsplit - 1);
    if (s_last) *ctr = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
    const int g = i / HD, d = i - g * HD;
    const int head = kvh * G + g;
    const float* mlh = p.part_ml + (size_t(m) * p.hq + head) * p.nsplit * 2;
    const float* oh = p.part_o + (size_t(m) * p.hq + head) * p.nsplit * HD;
    // kAttnU splits' values are loaded before they are combined (in split order)
    float mx = -INFINITY;
    for (int sb = 0; sb < p.nsplit; sb += kAttnU) {
      float t[kAttnU];
#pragma unroll
      for (int u = 0; u < kAttnU; ++u) t[u] = sb + u < p.nsplit ? __ldcg(mlh + 2 * (sb + u)) : -INFINITY;
#pragma unroll
      for (int u = 0; u < kAttnU; ++u) mx = fmaxf(mx, t[u]);
    }
    float num = 0.f, den = 0.f;
    for (int sb = 0; sb < p.nsplit; sb += kAttnU) {
      float ms[kAttnU], ls[kAttnU], os[kAttnU];
#pragma unroll
      for (int u = 0; u < kAttnU; ++u) {
        const bool in = sb + u < p.nsplit;
        ms[u] = in ? __ldcg(mlh + 2 * (sb + u)) : -INFINITY;
        ls[u] = in ? __ldcg(mlh + 2 * (sb + u) + 1) : 0.f;
        os[u] = in ? __ldcg(oh + size_t(sb + u) * HD + d) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kAttnU; ++u) {
        if (ms[u] == -INFINITY) continue;
        const float w = expf(ms[u] - mx);
        num = fmaf(w, os[u], num);
        den = fmaf(w, ls[u], den);
      }
    }
    static_cast<T*>(p.out)[size_t(m) * p.hq * HD + size_t(head) * HD + d] = from_f<T>(num / den);
  }
}

// ---------------------------------------------------------------------------
// Prefill form (tokens per batch row >= kAttnPfMinT, head dim 64 or 128): a
// CTA takes a tile of consecutive query tokens of one batch row and all G
// query heads of one KV head (R = QT * G rows, R <= 16 * RPT), and streams
// the keys [0, last position of the tile] through shared memory in tiles of
// 64 rows, so each K/V row is read once per query tile instead of once per
// query. Scores and P.V run on the CUDA cores from shared memory with an
// online softmax (running max and sum per row, rescaled per key tile):
//   scores  thread (rg = tid / 16, kg = tid % 16): rows rg*RPT.., keys kg + 16 k
//   P.V     thread (rg, dg = tid % 16): rows rg*RPT.., dims dg*HD/16..
// The 16 threads of a row group are one half-warp, so a row's tile max and
// sum are half-warp shuffles and its rescale factor is in every thread that
// holds that row's output. Causal rule as above (key j <= position of the
// query); rows past the batch row's tokens compute on zeros and write nothing.
// ---------------------------------------------------------------------------
constexpr int kAttnPfThreads = 256;
constexpr int kAttnPfKT = 64;    // keys per tile
constexpr int kAttnPfMinT = 16;  // tokens per batch row from which prefill uses this form
constexpr int kAttnPfPad = 4;    // row padding of the shared-memory tiles (floats)

template <int HD, int RPT>
__host__ __device__ constexpr size_t attn_pf_smem() {
  return (size_t(16 * RPT) * (HD + kAttnPfPad) + 2 * size_t(kAttnPfKT) * (HD + kAttnPfPad) +
          size_t(16 * RPT) * (kAttnPfKT + kAttnPfPad)) *
         sizeof(float);
}

template <typename T, int HD, int RPT>
__global__ void __launch_bounds__(kAttnPfThreads, 1) attn_prefill_kernel(const AttnParams p) {
  constexpr int VE = VecTraits<T>::kElems;
  constexpr int R = 16 * RPT;   // rows (query, head) per CTA at most
  constexpr int DPT = HD / 16;  // output dims per thread
  constexpr int QS = HD + kAttnPfPad, KS = HD + kAttnPfPad, PS = kAttnPfKT + kAttnPfPad;
  extern __shared__ __align__(16) float smf[];
  float* qs = smf;                          // [R][QS]
  float* ks = qs + size_t(R) * QS;          // [KT][KS]
  float* vs = ks + size_t(kAttnPfKT) * KS;  // [KT][KS]
  float* ps = vs + size_t(kAttnPfKT) * KS;  // [R][PS]

  pdl_launch();
  pdl_wait();
  const int G = p.hq / p.hkv;
  const int QT = R / G;  // query tokens per CTA
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int t0 = blockIdx.x * QT;
  const int T_ = p.tpr;
  if (t0 >= T_) return;
  const int nq = min(QT, T_ - t0);  // valid query tokens of this tile
  const int pos0 = (p.pos_ptr ? *p.pos_ptr : p.pos_base) + t0;
  const int kend = pos0 + nq;  // keys [0, kend)
  if (pos0 < 0 || kend > p.cap) {
    if (threadIdx.x == 0) atomicOr(p.status, kStatusBadPosition);
    return;
  }
  const int tid = threadIdx.x, rg = tid >> 4, sub = tid & 15;
  const T* kbase = static_cast<const T*>(p.k_cache) + (size_t(b) * p.hkv + kvh) * p.cap * HD;
  const T* vbase = static_cast<const T*>(p.v_cache) + (size_t(b) * p.hkv + kvh) * p.cap * HD;

  // q rows: row r = qi * G + g (zeros past the valid rows)
  for (int i = tid; i < R * (HD / VE); i += kAttnPfThreads) {
    const int r = i / (HD / VE), c = i - r * (HD / VE);
    const int qi = r / G, g = r - qi * G;
    float f[VE];
    if (qi < nq) {
      const size_t m = size_t(b) * T_ + t0 + qi;
      unpack(ld_vec(static_cast<const T*>(p.q) + m * p.hq * HD + size_t(kvh * G + g) * HD + c * VE), f);
    } else {
#pragma unroll
      for (int e = 0; e < VE; ++e) f[e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < VE; ++e) qs[size_t(r) * QS + c * VE + e] = f[e];
  }
  // the last key position each of this thread's rows may see (rows past the
  // valid queries see every key of the range: finite scores, no output)
  int lim[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = rg * RPT + i, qi = r / G;
    lim[i] = qi < nq ? pos0 + qi : kend - 1;
  }
  float mrow[RPT], lrow[RPT], o[RPT][DPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    mrow[i] = -INFINITY;
    lrow[i] = 0.f;
#pragma unroll
    for (int d = 0; d < DPT; ++d) o[i][d] = 0.f;
  }

  for (int j0 = 0; j0 < kend; j0 += kAttnPfKT) {
    __syncthreads();  // the previous tile's K/V/P are consumed (and q is staged)
    for (int i = tid; i < kAttnPfKT * (HD / VE); i += kAttnPfThreads) {
      const int j = i / (HD / VE), c = i - j * (HD / VE);
      float kf[VE], vf[VE];
      if (j0 + j < kend) {
        unpack(ld_vec(kbase + size_t(j0 + j) * HD + c * VE), kf);
        unpack(ld_vec(vbase + size_t(j0 + j) * HD + c * VE), vf);
      } else {
#pragma unroll
        for (int e = 0; e < VE; ++e) kf[e] = vf[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < VE; ++e) {
        ks[size_t(j) * KS + c * VE + e] = kf[e];
        vs[size_t(j) * KS + c * VE + e] = vf[e];
      }
    }
    __syncthreads();
    // scores of rows rg*RPT.. against keys sub + 16 k (consecutive threads on
    // consecutive K rows: conflict-free 16-byte loads)
    float sc[RPT][4];
#pragma unroll
    for (int i = 0; i < RPT; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) sc[i][k] = 0.f;
    for (int d = 0; d < HD; d += 4) {
      float4 kv[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) kv[k] = *reinterpret_cast<const float4*>(ks + size_t(sub + 16 * k) * KS + d);
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const float4 qv = *reinterpret_cast<const float4*>(qs + size_t(rg * RPT + i) * QS + d);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          sc[i][k] = fmaf(qv.w, kv[k].w, fmaf(qv.z, kv[k].z, fmaf(qv.y, kv[k].y, fmaf(qv.x, kv[k].x, sc[i][k]))));
      }
    }
    // online softmax: tile max and sum per row over the half-warp
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      float tm = -INFINITY;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = j0 + sub + 16 * k;
        sc[i][k] = j <= lim[i] ? sc[i][k] * p.scale : -INFINITY;
        tm = fmaxf(tm, sc[i][k]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, off));
      const float mn = fmaxf(mrow[i], tm);  // finite: key 0 is in the first tile of every row
      const float alpha = expf(mrow[i] - mn);
      float ts = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float e = expf(sc[i][k] - mn);
        ps[size_t(rg * RPT + i) * PS + sub + 16 * k] = e;
        ts += e;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) ts += __shfl_xor_sync(0xffffffffu, ts, off);
      lrow[i] = lrow[i] * alpha + ts;
      mrow[i] = mn;
#pragma unroll
      for (int d = 0; d < DPT; ++d) o[i][d] *= alpha;
    }
    __syncwarp();  // a row group's P entries come from the same half-warp
    // P.V: rows rg*RPT.., dims sub*DPT..
    const int kn = min(kAttnPfKT, kend - j0);
    for (int j = 0; j < kn; ++j) {
      float vv[DPT];
#pragma unroll
      for (int d = 0; d < DPT; d += 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(vs + size_t(j) * KS + sub * DPT + d);
        vv[d] = v4.x;
        vv[d + 1] = v4.y;
        vv[d + 2] = v4.z;
        vv[d + 3] = v4.w;
      }
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const float pr = ps[size_t(rg * RPT + i) * PS + j];
#pragma unroll
        for (int d = 0; d < DPT; ++d) o[i][d] = fmaf(pr, vv[d], o[i][d]);
      }
    }
  }
  // normalise and store the valid rows
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = rg * RPT + i, qi = r / G, g = r - qi * G;
    if (qi < nq) {
      const size_t m = size_t(b) * T_ + t0 + qi;
      T* dst = static_cast<T*>(p.out) + m * p.hq * HD + size_t(kvh * G + g) * HD + sub * DPT;
      const float inv = 1.0f / lrow[i];
#pragma unroll
      for (int d = 0; d < DPT; ++d) dst[d] = from_f<T>(o[i][d] * inv);
    }
  }
}

}  // namespace mtpb
