// Weight-streaming GEMV for decode-time linears: y[m, n] = sum_k x[m, k] * W[n, k].
//
// W is the PyTorch Linear layout [N, K] (row-major), streamed once with
// 16-byte non-allocating loads. x is small ([M, K] with M <= a few dozen),
// staged in shared memory when it fits. Accumulation is fp32; results are
// rounded to the storage type T at the same points where the reference
// (F.linear in T, then elementwise ops in T) rounds.
//
// A CTA owns a contiguous range of "units" (a unit is one output row, or a
// row pair for the SwiGLU and RoPE epilogues); each warp computes the dot
// products of RPW units at a time, optionally split along K over `ks` warps.
//
// Prologue (before the previous kernel's results are needed):
//   1. prefetch this CTA's weight rows into L2 (cp.async.bulk.prefetch.L2),
//   2. griddepcontrol.launch_dependents, 3. griddepcontrol.wait.
// Input modes: x from global memory, or "consume": wait for the peers of a
// collective site, reduce their partials (fixed rank order), add the
// residual, write the new residual (CTA 0) and apply RMSNorm into shared
// memory (the fused RowParallel AllReduce -> residual -> RMSNorm chain).
#pragma once

#include "comm.cuh"

namespace mtpb {

enum Epi : int {
  kEpiStore = 0,   // y[m, n] = T(acc + bias[n])
  kEpiSwiglu = 1,  // act[m, j] = T(silu(T(gate_j)) * T(up_j)), rows (j, j + N/2)
  kEpiRope = 2,    // fused QKV: bias, RoPE on q/k, q -> y, k/v -> KV cache
  kEpiPush = 3,    // partial T(acc) pushed to every rank's receive slot + flags
  kEpiArgmax = 4,  // logits T(acc) -> y, running packed argmax -> best[m]
};

struct GemvParams {
  const void* w;
  const void* bias;
  int M, N, K;
  int units;
  int ks;
  int decode;  // a decode step's projection (T = 1): its own tensor-core row threshold
  // input
  int x_mode;  // 0: x from global memory; 1: consume a collective + RMSNorm
  const void* x;
  int ldx;
  int x_smem;  // stage x (mode 0) in shared memory
  // consume mode
  Comm comm;
  SeqRef in_seq;
  int in_chan;
  int in_nprod;
  const void* res_in;
  void* res_out;
  const void* gain;
  const void* ar_bias;
  float eps;
  int has_res;
  // outputs
  void* y;
  int ldy;
  // Store/Argmax output row of row m: (m / tpr) * out_T + out_t0 + m % tpr
  // when out_T > 0 (a token chunk of a longer sequence), else m
  int out_T, out_t0;
  // rope / kv append
  const float* cos_tab;
  const float* sin_tab;
  int rope_len;
  int hd, hq, hkv;
  void* k_cache;
  void* v_cache;
  int kv_cap;
  int tpr;  // tokens per batch row: row m is token (m % tpr) of batch row (m / tpr)
  const int* pos_ptr;         // device slot of token 0 (decode step), or
  int pos_base;               // host slot of token 0
  const long long* rope_pos;  // RoPE position of token t (NULL: the slot)
  // push
  SeqRef out_seq;
  int out_chan;
  int ts_cols;  // > 0: two-shot site, column u goes to rank ts_owner(u) only
  // argmax
  long long* best;
  uint32_t vocab_start;
  int nan_wins;
  // misc
  uint32_t prefetch_cap;
};

template <int EPI> struct EpiTraits { static constexpr int kUR = 1; };
template <> struct EpiTraits<kEpiSwiglu> { static constexpr int kUR = 2; };
template <> struct EpiTraits<kEpiRope> { static constexpr int kUR = 2; };

// row index of the r-th row (r < UR) of unit u
template <int EPI>
__device__ __forceinline__ int unit_row(const GemvParams& p, int u, int r) {
  if constexpr (EPI == kEpiSwiglu) {
    return u + r * (p.N >> 1);
  } else if constexpr (EPI == kEpiRope) {
    const int half = p.hd >> 1;
    const int h = u / half, i = u - h * half;
    return h * p.hd + i + r * half;
  } else {
    return u;
  }
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

// The reference's rotate: x*cos + rotate_half(x)*sin in fp32, products and
// the sum rounded separately (no FMA contraction).
__device__ __forceinline__ float rope_mix(float a, float c, float b, float s) {
  return __fadd_rn(__fmul_rn(a, c), __fmul_rn(b, s));
}

__device__ __forceinline__ int out_row(const GemvParams& p, int m) {
  return p.out_T > 0 ? (m / p.tpr) * p.out_T + p.out_t0 + (m % p.tpr) : m;
}

template <typename T, int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvParams& p, int m, int u, float v0, float v1,
                                              uint32_t out_seq, long long* best_s) {
  if constexpr (EPI == kEpiStore) {
    float v = v0;
    if (p.bias) v += to_f(static_cast<const T*>(p.bias)[u]);
    static_cast<T*>(p.y)[size_t(out_row(p, m)) * p.ldy + u] = from_f<T>(v);
  } else if constexpr (EPI == kEpiSwiglu) {
    const int half = p.N >> 1;
    float g = v0, up = v1;
    if (p.bias) {
      g += to_f(static_cast<const T*>(p.bias)[u]);
      up += to_f(static_cast<const T*>(p.bias)[u + half]);
    }
    g = round_t<T>(g);
    up = round_t<T>(up);
    const float act = round_t<T>(silu_f(g)) * up;
    static_cast<T*>(p.y)[size_t(m) * p.ldy + u] = from_f<T>(act);
  } else if constexpr (EPI == kEpiRope) {
    const int half = p.hd >> 1;
    const int h = u / half, i = u - h * half;
    const int r0 = h * p.hd + i, r1 = r0 + half;
    float a = v0, b = v1;
    if (p.bias) {
      a += to_f(static_cast<const T*>(p.bias)[r0]);
      b += to_f(static_cast<const T*>(p.bias)[r1]);
    }
    a = round_t<T>(a);
    b = round_t<T>(b);
    const int bt = m / p.tpr, t = m - bt * p.tpr;
    const int pos = (p.pos_ptr ? *p.pos_ptr : p.pos_base) + t;  // KV slot
    const long long rp = p.rope_pos ? p.rope_pos[t] : pos;      // RoPE position
    if (pos < 0 || pos >= p.kv_cap || rp < 0 || rp >= p.rope_len) {
      atomicOr(p.comm.status(), kStatusBadPosition);
      return;
    }
    if (h < p.hq + p.hkv) {  // q or k head: rotate
      const float* cs = p.cos_tab + size_t(rp) * p.hd;
      const float* sn = p.sin_tab + size_t(rp) * p.hd;
      const float o0 = rope_mix(a, cs[i], -b, sn[i]);
      const float o1 = rope_mix(b, cs[i + half], a, sn[i + half]);
      if (h < p.hq) {
        T* q = static_cast<T*>(p.y) + size_t(m) * p.ldy + size_t(h) * p.hd;
        q[i] = from_f<T>(o0);
        q[i + half] = from_f<T>(o1);
      } else {
        const int kh = h - p.hq;
        T* k = static_cast<T*>(p.k_cache) + ((size_t(bt) * p.hkv + kh) * p.kv_cap + pos) * p.hd;
        k[i] = from_f<T>(o0);
        k[i + half] = from_f<T>(o1);
      }
    } else {
      const int vh = h - p.hq - p.hkv;
      T* v = static_cast<T*>(p.v_cache) + ((size_t(bt) * p.hkv + vh) * p.kv_cap + pos) * p.hd;
      v[i] = from_f<T>(a);
      v[i + half] = from_f<T>(b);
    }
  } else if constexpr (EPI == kEpiPush) {
    const T val = from_f<T>(v0);
    const int par = out_seq & 1;
    const size_t off = size_t(m) * p.N + u;
    if (p.ts_cols > 0) {
      const int d = ts_owner(u, p.ts_cols, p.comm.world);
      reinterpret_cast<T*>(p.comm.data(d, p.out_chan, par, p.comm.rank))[off] = val;
    } else {
      for (int d = 0; d < p.comm.world; ++d) {
        reinterpret_cast<T*>(p.comm.data(d, p.out_chan, par, p.comm.rank))[off] = val;
      }
    }
  } else if constexpr (EPI == kEpiArgmax) {
    const float v = round_t<T>(v0);
    static_cast<T*>(p.y)[size_t(out_row(p, m)) * p.ldy + u] = from_f<T>(v);
    const long long pk = argmax_pack(v, p.vocab_start + uint32_t(u), p.nan_wins != 0);
    atomicMax(best_s + m, pk);
  }
}

// ---------------------------------------------------------------------------
// consume prologue: x_norm[m, :] = RMSNorm(residual + sum_r partial_r) into xs
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ bool consume_norm(const GemvParams& p, T* xs, float* red) {
  const int H = p.K;
  const Comm& c = p.comm;
  const uint32_t seq = resolve_seq(c, p.in_seq);
  if (!wait_peers(c, p.in_chan, seq, p.in_nprod)) return false;
  const int par = seq & 1;
  const T* gain = static_cast<const T*>(p.gain);
  for (int m = 0; m < p.M; ++m) {
    float ss = 0.f;
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
      const size_t off = size_t(m) * H + j;
      float s = 0.f;
      for (int r = 0; r < c.world; ++r) {
        const T* src = reinterpret_cast<const T*>(c.data(c.rank, p.in_chan, par, r));
        s += to_f(__ldcg(src + off));
      }
      float o = round_t<T>(s);  // the reduced tensor is stored in T
      if (p.ar_bias) o = round_t<T>(o + to_f(static_cast<const T*>(p.ar_bias)[j]));
      float x = o;
      if (p.has_res) x = round_t<T>(to_f(static_cast<const T*>(p.res_in)[off]) + o);
      if (blockIdx.x == 0 && p.res_out) static_cast<T*>(p.res_out)[off] = from_f<T>(x);
      xs[off] = from_f<T>(x);
      ss += x * x;
    }
    const float tot = block_sum(ss, red);
    const float rinv = rsqrtf(tot / float(H) + p.eps);
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
      const size_t off = size_t(m) * H + j;
      const float x = to_f(xs[off]);
      xs[off] = from_f<T>(__fmul_rn(__fmul_rn(x, rinv), to_f(gain[j])));
    }
  }
  __syncthreads();
  return true;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kRowsPerWarp = 4;  // rows (not units) per warp task

template <typename T, int EPI, int MT>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvParams p) {
  constexpr int UR = EpiTraits<EPI>::kUR;
  constexpr int RPW = kRowsPerWarp / UR;  // units per warp task
  constexpr int R = RPW * UR;             // rows per warp task
  constexpr int VE = VecTraits<T>::kElems;

  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[32];
  __shared__ long long best_s[64];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // balanced unit partition
  const int G = gridDim.x;
  const int base = p.units / G, rem = p.units % G;
  const int u0 = blockIdx.x * base + min(int(blockIdx.x), rem);
  const int nu = base + (int(blockIdx.x) < rem ? 1 : 0);

  // 1. L2 prefetch of this CTA's weight rows
  if (threadIdx.x == 0 && nu > 0 && p.prefetch_cap > 0) {
    const int rlo = unit_row<EPI>(p, u0, 0);
    const int rhi = unit_row<EPI>(p, u0 + nu - 1, UR - 1);
    const size_t rb = size_t(p.K) * sizeof(T);
    if constexpr (EPI == kEpiSwiglu) {
      const size_t n = min(size_t(nu) * rb, size_t(p.prefetch_cap) / 2);
      prefetch_range_l2(static_cast<const char*>(p.w) + size_t(rlo) * rb, n);
      prefetch_range_l2(static_cast<const char*>(p.w) + size_t(u0 + (p.N >> 1)) * rb, n);
    } else {
      const size_t n = min(size_t(rhi - rlo + 1) * rb, size_t(p.prefetch_cap));
      prefetch_range_l2(static_cast<const char*>(p.w) + size_t(rlo) * rb, n);
    }
  }
  // 2./3. programmatic dependent launch
  pdl_launch();
  pdl_wait();

  if constexpr (EPI == kEpiArgmax) {
    for (int i = threadIdx.x; i < 64; i += blockDim.x) best_s[i] = kArgmaxEmpty;
  }

  // input staging
  T* xs_smem = reinterpret_cast<T*>(smem_raw);
  float* part = reinterpret_cast<float*>(smem_raw + (p.x_smem ? size_t(p.M) * p.K * sizeof(T) : 0));
  const T* xs;
  int ldxs;
  if (p.x_mode == 1) {
    if (!consume_norm<T>(p, xs_smem, red)) return;
    xs = xs_smem;
    ldxs = p.K;
  } else if (p.x_smem) {
    const int vpr = p.K / VE;
    for (int i = threadIdx.x; i < p.M * vpr; i += blockDim.x) {
      const int m = i / vpr, c = i - m * vpr;
      reinterpret_cast<uint4*>(xs_smem)[i] =
          ld_vec(static_cast<const T*>(p.x) + size_t(m) * p.ldx + size_t(c) * VE);
    }
    __syncthreads();
    xs = xs_smem;
    ldxs = p.K;
  } else {
    xs = static_cast<const T*>(p.x);
    ldxs = p.ldx;
  }
  if constexpr (EPI == kEpiArgmax) __syncthreads();

  uint32_t out_seq = 0;
  if constexpr (EPI == kEpiPush) out_seq = resolve_seq(p.comm, p.out_seq);

  const int CPR = p.K / VE;
  const int ks = p.ks;
  const int cps = (CPR + ks - 1) / ks;
  const int ngroups = (nu + RPW - 1) / RPW;
  const int ntasks = ngroups * ks;
  const T* W = static_cast<const T*>(p.w);

  for (int t0 = 0; t0 < ntasks; t0 += kGemvWarps) {
    const int t = t0 + warp;
    const bool active = t < ntasks;
    const int g = active ? t / ks : 0;
    const int s = active ? t - g * ks : 0;
    int rows[R];
    bool valid[RPW];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int u = u0 + g * RPW + j;
      valid[j] = active && (g * RPW + j) < nu;
#pragma unroll
      for (int r = 0; r < UR; ++r) rows[j * UR + r] = valid[j] ? unit_row<EPI>(p, u, r) : 0;
    }
    const int c_beg = s * cps;
    const int c_end = min(CPR, c_beg + cps);

    for (int m0 = 0; m0 < p.M; m0 += MT) {
      float acc[MT][R];
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int r = 0; r < R; ++r) acc[m][r] = 0.f;

      if (active) {
        // U chunks x R rows of 16-byte weight loads in flight per lane
        constexpr int U = (MT <= 2) ? 4 : 2;
        for (int c0 = c_beg + lane; c0 < c_end; c0 += 32 * U) {
          uint4 wv[U][R];
#pragma unroll
          for (int h = 0; h < U; ++h) {
            const int c = c0 + 32 * h;
            const bool okc = c < c_end;
#pragma unroll
            for (int r = 0; r < R; ++r) {
              wv[h][r] = (okc && valid[r / UR]) ? ld_stream(W + size_t(rows[r]) * p.K + size_t(c) * VE)
                                                : make_uint4(0, 0, 0, 0);
            }
          }
#pragma unroll
          for (int h = 0; h < U; ++h) {
            const int c = c0 + 32 * h;
            if (c < c_end) {
              float xf[MT][VE];
#pragma unroll
              for (int m = 0; m < MT; ++m) {
                if (m0 + m < p.M) {
                  unpack(ld_vec(xs + size_t(m0 + m) * ldxs + size_t(c) * VE), xf[m]);
                } else {
#pragma unroll
                  for (int e = 0; e < VE; ++e) xf[m][e] = 0.f;
                }
              }
#pragma unroll
              for (int r = 0; r < R; ++r) {
                float wf[VE];
                unpack(wv[h][r], wf);
#pragma unroll
                for (int m = 0; m < MT; ++m)
#pragma unroll
                  for (int e = 0; e < VE; ++e) acc[m][r] = fmaf(wf[e], xf[m][e], acc[m][r]);
              }
            }
          }
        }
      }
      // warp reduction: every lane ends with every sum
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int r = 0; r < R; ++r) acc[m][r] = warp_sum(acc[m][r]);

      // lane l owns item l = (m, unit j): l = m * RPW + j
      float v0 = 0.f, v1 = 0.f;
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int j = 0; j < RPW; ++j)
          if (lane == m * RPW + j) {
            v0 = acc[m][j * UR];
            if constexpr (UR == 2) v1 = acc[m][j * UR + 1];
          }
      const int it_m = lane / RPW, it_j = lane - (lane / RPW) * RPW;
      const bool item_ok = lane < MT * RPW && (m0 + it_m) < p.M;

      if (ks == 1) {
        if (active && item_ok && it_j < RPW && valid[0] && (g * RPW + it_j) < nu) {
          gemv_epilogue<T, EPI>(p, m0 + it_m, u0 + g * RPW + it_j, v0, v1, out_seq, best_s);
        }
      } else {
        // cross-warp K reduction through shared memory, fixed order
        constexpr int ITEMS = MT * RPW;
        if (lane < ITEMS) {
          part[(warp * ITEMS + lane) * 2] = v0;
          part[(warp * ITEMS + lane) * 2 + 1] = v1;
        }
        __syncthreads();
        const int groups_here = kGemvWarps / ks;
        for (int it = threadIdx.x; it < groups_here * ITEMS; it += blockDim.x) {
          const int gi = it / ITEMS, l = it - gi * ITEMS;
          const int gg = t0 / ks + gi;
          const int m = m0 + l / RPW, j = l % RPW;
          if (gg * RPW + j < nu && gg < ngroups && m < p.M) {
            float a0 = 0.f, a1 = 0.f;
            for (int q = 0; q < ks; ++q) {
              a0 += part[((gi * ks + q) * ITEMS + l) * 2];
              a1 += part[((gi * ks + q) * ITEMS + l) * 2 + 1];
            }
            gemv_epilogue<T, EPI>(p, m, u0 + gg * RPW + j, a0, a1, out_seq, best_s);
          }
        }
        __syncthreads();
      }
    }
  }

  if constexpr (EPI == kEpiPush) signal_peers(p.comm, p.out_chan, out_seq);
  if constexpr (EPI == kEpiArgmax) {
    __syncthreads();
    for (int m = threadIdx.x; m < p.M; m += blockDim.x) {
      if (best_s[m] != kArgmaxEmpty) atomicMax(p.best + m, best_s[m]);
    }
  }
}

}  // namespace mtpb
