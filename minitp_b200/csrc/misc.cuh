// Embedding, greedy-argmax exchange, standalone AllReduce(+residual+RMSNorm)
// and RMSNorm kernels.
#pragma once

#include "ar_rows.cuh"
#include "comm.cuh"
#include "ll.cuh"

namespace mtpb {

// ---------------------------------------------------------------------------
// Vocab-parallel embedding (reference: minitp/parallel/embedding.py:44-50).
// Row m looks up ids[m] when it falls in [vstart, vend), else contributes
// zeros; the rows are pushed into every rank's receive slot of a collective
// site, whose consumer sums them (one non-zero term: bit-exact).
// With `advance_step`, this kernel opens a new model step on channel 0: all
// CTAs use step+1 for their sequence number and the last CTA stores it.
// ---------------------------------------------------------------------------
struct EmbedParams {
  const long long* ids;  // row m reads ids[(m / ids_tpr) * ids_T + ids_t0 + m % ids_tpr] (ids_T > 0), else ids[m]
  int ids_tpr, ids_T, ids_t0;
  const void* table;     // [vend - vstart][H]
  int M, H;
  long long vstart, vend, vtotal;
  Comm comm;
  int chan;
  SeqRef seq;
  int advance_step;
  void* out;  // optional: plain [M][H] output instead of a push (world == 1 only)
};

template <typename T>
__global__ void __launch_bounds__(128) embed_kernel(const EmbedParams p) {
  constexpr int VE = VecTraits<T>::kElems;
  pdl_launch();
  pdl_wait();
  uint32_t seq = 0, step_next = 0;
  if (p.advance_step) {
    step_next = ld_volatile_u32(p.comm.ctl() + kCtlStep) + 1u;
    seq = step_next * p.seq.nsite + p.seq.site + 1u;
  } else {
    seq = resolve_seq(p.comm, p.seq);
  }
  const int par = seq & 1;
  const bool vec = (p.H % VE) == 0;
  for (int m = blockIdx.x; m < p.M; m += gridDim.x) {
    const long long id =
        p.ids[p.ids_T > 0 ? (m / p.ids_tpr) * p.ids_T + p.ids_t0 + (m % p.ids_tpr) : m];
    if (id < 0 || id >= p.vtotal) {
      if (threadIdx.x == 0) atomicOr(p.comm.status(), kStatusBadToken);
    }
    const bool mine = id >= p.vstart && id < p.vend;
    const T* row = static_cast<const T*>(p.table) + size_t(mine ? id - p.vstart : 0) * p.H;
    if (vec) {
      for (int c = threadIdx.x; c < p.H / VE; c += blockDim.x) {
        const uint4 v = mine ? ld_vec(row + size_t(c) * VE) : make_uint4(0, 0, 0, 0);
        if (p.out) {
          reinterpret_cast<uint4*>(static_cast<T*>(p.out) + size_t(m) * p.H)[c] = v;
        } else {
          for (int d = 0; d < p.comm.world; ++d) {
            T* dst = reinterpret_cast<T*>(p.comm.data(d, p.chan, par, p.comm.rank)) + size_t(m) * p.H;
            reinterpret_cast<uint4*>(dst)[c] = v;
          }
        }
      }
    } else {
      for (int j = threadIdx.x; j < p.H; j += blockDim.x) {
        const T v = mine ? row[j] : from_f<T>(0.f);
        if (p.out) {
          static_cast<T*>(p.out)[size_t(m) * p.H + j] = v;
        } else {
          for (int d = 0; d < p.comm.world; ++d)
            reinterpret_cast<T*>(p.comm.data(d, p.chan, par, p.comm.rank))[size_t(m) * p.H + j] = v;
        }
      }
    }
  }
  if (!p.out) signal_peers(p.comm, p.chan, seq);
  if (p.advance_step) advance_counter(p.comm, kCtlStep, kCtlStepDone, step_next);
}

// ---------------------------------------------------------------------------
// Packed-key argmax over logits rows (the local half of the reference's
// distributed_argmax, embedding.py:146-172): part[m * splits + s] = max over
// split s of row m of argmax_pack(logit, vstart + col). grid = (splits, M).
// ---------------------------------------------------------------------------
struct ArgmaxRowsParams {
  const void* logits;
  int M, V;
  long long ld;
  uint32_t vstart;
  int nan_wins;
  long long* part;  // [M][gridDim.x]
};

template <typename T>
__global__ void __launch_bounds__(256) argmax_rows_kernel(const ArgmaxRowsParams p) {
  pdl_launch();
  pdl_wait();
  const int m = blockIdx.y;
  const T* row = static_cast<const T*>(p.logits) + size_t(m) * p.ld;
  const int per = (p.V + gridDim.x - 1) / gridDim.x;
  const int c0 = blockIdx.x * per, c1 = min(p.V, c0 + per);
  long long bst = kArgmaxEmpty;
  for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
    const long long pk = argmax_pack(to_f(row[c]), p.vstart + uint32_t(c), p.nan_wins != 0);
    bst = pk > bst ? pk : bst;
  }
  bst = warp_max_ll(bst);
  __shared__ long long wb[32];
  if ((threadIdx.x & 31) == 0) wb[threadIdx.x >> 5] = bst;
  __syncthreads();
  if (threadIdx.x == 0) {
    long long b = kArgmaxEmpty;
    for (int i = 0; i < int(blockDim.x >> 5); ++i) b = wb[i] > b ? wb[i] : b;
    p.part[size_t(m) * gridDim.x + blockIdx.x] = b;
  }
}

// ---------------------------------------------------------------------------
// Greedy token selection: exchange every rank's packed best per row over
// NVLink (one int64 per row and rank: the O(tp) gather of the reference,
// embedding.py:158-172 with collectives.py:185-214), take the max, decode the
// id. Writes the token to `tok_out[m]` and optionally `out_ids[m, col]`.
// One CTA. The local candidates come either from `best[m]` (filled by atomic
// max in the LM-head GEMV; reset to empty here for the next step) or, when
// nsplit > 0, from the per-split partials part[m * nsplit + s].
// ---------------------------------------------------------------------------
struct ArgmaxFinishParams {
  long long* best;
  const long long* part;
  int nsplit;
  int M;
  Comm comm;
  int chan;
  SeqRef seq;
  int use_coll_counter;  // channel 1: sequence from kCtlColl, advanced here
  long long* tok_out;    // [M]
  long long* out_ids;    // optional [M][ld_out]
  int ld_out;
  int out_col;           // column written when pos_ptr is null
  int* pos_ptr;          // decode step: column = *pos_ptr + 1, then ++*pos_ptr
};

__global__ void __launch_bounds__(64) argmax_finish_kernel(const ArgmaxFinishParams p) {
  pdl_launch();
  pdl_wait();
  const Comm& c = p.comm;
  uint32_t seq;
  if (p.use_coll_counter) {
    seq = ld_volatile_u32(c.ctl() + kCtlColl) + 1u;
  } else {
    seq = resolve_seq(c, p.seq);
  }
  const int par = seq & 1;
  __shared__ long long loc[64];
  for (int m = threadIdx.x; m < p.M; m += blockDim.x) {
    if (p.nsplit > 0) {
      long long b = kArgmaxEmpty;
      for (int s = 0; s < p.nsplit; ++s) {
        const long long u = p.part[size_t(m) * p.nsplit + s];
        b = u > b ? u : b;
      }
      loc[m] = b;
    } else {
      loc[m] = p.best[m];
      p.best[m] = kArgmaxEmpty;
    }
    if (c.world > 1) {
      for (int d = 0; d < c.world; ++d)
        reinterpret_cast<long long*>(c.data(d, p.chan, par, c.rank))[m] = loc[m];
    }
  }
  bool ok = true;
  if (c.world > 1) {
    signal_peers(c, p.chan, seq);
    ok = wait_peers(c, p.chan, seq, 1);
  }
  __syncthreads();
  const int col = p.pos_ptr ? *p.pos_ptr + 1 : p.out_col;
  for (int m = threadIdx.x; m < p.M && ok; m += blockDim.x) {
    long long v = loc[m];
    if (c.world > 1) {
      v = kArgmaxEmpty;
      for (int r = 0; r < c.world; ++r) {
        const long long u = __ldcg(reinterpret_cast<const long long*>(c.data(c.rank, p.chan, par, r)) + m);
        v = u > v ? u : v;
      }
    }
    const long long tok = argmax_id(v);
    p.tok_out[m] = tok;
    if (p.out_ids) p.out_ids[size_t(m) * p.ld_out + col] = tok;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (p.pos_ptr) *p.pos_ptr += 1;
    if (p.use_coll_counter) c.ctl()[kCtlColl] = seq;
  }
}

// ---------------------------------------------------------------------------
// Standalone one-shot AllReduce, optionally fused with bias + residual add +
// RMSNorm (RowParallelLinear.forward linear.py:111-122, then the decoder's
// residual add layer.py:64 and RMSNorm layer.py:36-42). Channel 1.
// CTA c owns rows [c*rpc, (c+1)*rpc): it pushes its partial rows to every
// rank, raises its flag, waits for CTA c of every rank, and reduces in rank
// order. out_res = T(res + T(sum)) (or T(sum) without residual);
// out_norm = T(out_res * rsqrt(mean(out_res^2) + eps) * gain).
// ---------------------------------------------------------------------------
struct ArNormParams {
  const void* partial;
  const void* residual;
  const void* gain;
  const void* bias;
  void* out_res;
  void* out_norm;
  int rows, H, rpc;
  float eps;
  Comm comm;
  int chan;
};

template <typename T>
__global__ void __launch_bounds__(256) ar_norm_kernel(const ArNormParams p) {
  constexpr int VE = VecTraits<T>::kElems;
  __shared__ float red[32];
  pdl_launch();
  pdl_wait();
  const Comm& c = p.comm;
  const uint32_t seq = ld_volatile_u32(c.ctl() + kCtlColl) + 1u;
  const int par = seq & 1;
  const int r0 = blockIdx.x * p.rpc, r1 = min(p.rows, r0 + p.rpc);
  const bool vec = ar_rows_vec_ok<T>(p.H);
  if (c.world > 1) {
    const size_t e0 = size_t(r0) * p.H, e1 = size_t(r1) * p.H;
    const T* src = static_cast<const T*>(p.partial);
    if (vec) {
      for (size_t i = e0 / VE + threadIdx.x; i < e1 / VE; i += blockDim.x) {
        const uint4 v = ld_vec(src + i * VE);
        for (int d = 0; d < c.world; ++d)
          reinterpret_cast<uint4*>(c.data(d, p.chan, par, c.rank))[i] = v;
      }
    } else {
      for (size_t i = e0 + threadIdx.x; i < e1; i += blockDim.x) {
        const T v = src[i];
        for (int d = 0; d < c.world; ++d) reinterpret_cast<T*>(c.data(d, p.chan, par, c.rank))[i] = v;
      }
    }
    signal_peers(c, p.chan, seq);
    if (!wait_peers_cta(c, p.chan, seq, blockIdx.x)) return;
  }
  const T* gain = static_cast<const T*>(p.gain);
  if (vec) {
    for (int row = r0; row < r1; ++row)
      ar_finish_row<T>(c, p.chan, par, 0, c.world > 1 ? nullptr : static_cast<const T*>(p.partial), row, p.H,
                       static_cast<const T*>(p.bias), static_cast<const T*>(p.residual), static_cast<T*>(p.out_res),
                       p.out_norm ? gain : nullptr, p.eps, static_cast<T*>(p.out_norm), red);
    advance_counter(c, kCtlColl, kCtlCollDone, seq);
    return;
  }
  for (int row = r0; row < r1; ++row) {
    float ss = 0.f;
    for (int j = threadIdx.x; j < p.H; j += blockDim.x) {
      const size_t off = size_t(row) * p.H + j;
      float s;
      if (c.world > 1) {
        s = 0.f;
        for (int r = 0; r < c.world; ++r)
          s += to_f(__ldcg(reinterpret_cast<const T*>(c.data(c.rank, p.chan, par, r)) + off));
      } else {
        s = to_f(static_cast<const T*>(p.partial)[off]);
      }
      float o = round_t<T>(s);
      if (p.bias) o = round_t<T>(o + to_f(static_cast<const T*>(p.bias)[j]));
      float x = o;
      if (p.residual) x = round_t<T>(to_f(static_cast<const T*>(p.residual)[off]) + o);
      static_cast<T*>(p.out_res)[off] = from_f<T>(x);
      ss += x * x;
    }
    if (p.out_norm) {
      const float tot = block_sum(ss, red);
      const float rinv = rsqrtf(tot / float(p.H) + p.eps);
      __syncthreads();
      for (int j = threadIdx.x; j < p.H; j += blockDim.x) {
        const size_t off = size_t(row) * p.H + j;
        const float x = to_f(static_cast<const T*>(p.out_res)[off]);
        static_cast<T*>(p.out_norm)[off] = from_f<T>(__fmul_rn(__fmul_rn(x, rinv), to_f(gain[j])));
      }
    }
  }
  advance_counter(c, kCtlColl, kCtlCollDone, seq);
}

// The same operation over LL words, for messages whose LL form (8 bytes per
// kPer values) fits the communicator slot: every rank pushes its partial rows
// as LL words into channel `chan` of every rank (parity seq & 1), then each
// CTA reads its rows' words of every rank (all ranks' loads in flight
// together), sums them in rank order and finishes its rows. No fence and no
// flag: the words carry the call's sequence number.
template <typename T>
__global__ void __launch_bounds__(256) ar_norm_ll_kernel(const ArNormParams p) {
  constexpr int P = LLPack<T>::kPer;
  __shared__ float red[32];
  __shared__ int abort_s;
  pdl_launch();
  pdl_wait();
  const Comm& c = p.comm;
  const uint32_t seq = ld_volatile_u32(c.ctl() + kCtlColl) + 1u;
  const int par = seq & 1;
  const int W = p.H / P;
  const int r0 = blockIdx.x * p.rpc, r1 = min(p.rows, r0 + p.rpc);
  if (threadIdx.x == 0) abort_s = 0;
  __syncthreads();
  const T* src = static_cast<const T*>(p.partial);
  for (int i = threadIdx.x; i < (r1 - r0) * W; i += blockDim.x) {
    const size_t wi = size_t(r0) * W + i;
    float f[P];
#pragma unroll
    for (int e = 0; e < P; ++e) f[e] = to_f(src[wi * P + e]);
    const uint32_t u = LLPack<T>::pack(f);
    for (int d = 0; d < c.world; ++d) ll_put(reinterpret_cast<uint64_t*>(c.data(d, p.chan, par, c.rank)) + wi, u, seq);
  }
  const T* gain = static_cast<const T*>(p.gain);
  const T* bias = static_cast<const T*>(p.bias);
  const T* resid = static_cast<const T*>(p.residual);
  T* out_res = static_cast<T*>(p.out_res);
  bool ok = true;
  for (int row = r0; row < r1; ++row) {
    float ss = 0.f;
    for (int w = threadIdx.x; w < W; w += blockDim.x) {
      const size_t wi = size_t(row) * W + w;
      uint2 v[kMaxRanks];
      auto addr = [&](int r) { return reinterpret_cast<const uint64_t*>(c.data(c.rank, p.chan, par, r)) + wi; };
      if (ok && !ll_wait1<kMaxRanks>(c.timeout_ns, 0u, addr, c.world, seq, v, &abort_s)) {
        ok = false;
        abort_s = 1;
        atomicOr(c.status(), kStatusTimeout);
      }
      float s[P];
#pragma unroll
      for (int e = 0; e < P; ++e) s[e] = 0.f;
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        if (r < c.world) {
          float f[P];
          LLPack<T>::unpack(v[r].x, f);
#pragma unroll
          for (int e = 0; e < P; ++e) s[e] += f[e];
        }
      }
#pragma unroll
      for (int e = 0; e < P; ++e) {
        const int j = w * P + e;
        const size_t off = size_t(row) * p.H + j;
        float o = round_t<T>(s[e]);
        if (bias) o = round_t<T>(o + to_f(bias[j]));
        const float x = resid ? round_t<T>(to_f(resid[off]) + o) : o;
        out_res[off] = from_f<T>(x);
        ss += x * x;
      }
    }
    if (p.out_norm) {
      const float tot = block_sum(ss, red);
      const float rinv = rsqrtf(tot / float(p.H) + p.eps);
      __syncthreads();
      for (int j = threadIdx.x; j < p.H; j += blockDim.x) {
        const size_t off = size_t(row) * p.H + j;
        const float x = to_f(out_res[off]);
        static_cast<T*>(p.out_norm)[off] = from_f<T>(__fmul_rn(__fmul_rn(x, rinv), to_f(gain[j])));
      }
    }
  }
  advance_counter(c, kCtlColl, kCtlCollDone, seq);
}

// One-thread store of a device int (sets the decode position in-stream).
struct SetI32 {
  int* ptr;
  int value;
};
__global__ void set_i32_kernel(const SetI32 p) {
  pdl_launch();
  pdl_wait();
  *p.ptr = p.value;
}

// ---------------------------------------------------------------------------
// RMSNorm (layer.py:36-42): y = T(x * rsqrt(mean(x^2) + eps) * w), fp32 math.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const void* xv, const void* wv, void* yv, int rows,
                                                       int H, float eps) {
  __shared__ float red[32];
  pdl_launch();
  pdl_wait();
  const T* x = static_cast<const T*>(xv);
  const T* w = static_cast<const T*>(wv);
  T* y = static_cast<T*>(yv);
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    float ss = 0.f;
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
      const float v = to_f(x[size_t(row) * H + j]);
      ss += v * v;
    }
    const float tot = block_sum(ss, red);
    const float rinv = rsqrtf(tot / float(H) + eps);
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
      const float v = to_f(x[size_t(row) * H + j]);
      y[size_t(row) * H + j] = from_f<T>(__fmul_rn(__fmul_rn(v, rinv), to_f(w[j])));
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// NVLink latency floor: one LL word bounced between this rank and `peer`
// `iters` times (one thread on each of the two ranks). The lower rank sends
// ping i (sequence base + 2i) into the peer's buffer and waits for pong i
// (base + 2i + 1) in its own; the peer answers each ping. ns_out gets the
// time of the last `iters - warm` round trips on this rank. Every wait is
// bounded by the communicator timeout (kStatusTimeout, then return). The
// word sits at the start of this pair's channel-3 slot, with sequence
// numbers of 2^31 and above, which no standalone collective uses.
// ---------------------------------------------------------------------------
struct PingParams {
  Comm comm;
  int peer;
  int iters;
  int warm;
  uint32_t base;
  unsigned long long* ns_out;
};

__global__ void pingpong_kernel(const PingParams p) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const Comm& c = p.comm;
  const uint64_t* mine = reinterpret_cast<const uint64_t*>(c.data(c.rank, 3, 0, p.peer));
  uint64_t* theirs = reinterpret_cast<uint64_t*>(c.data(p.peer, 3, 0, c.rank));
  const bool lead = c.rank < p.peer;
  uint64_t t0 = global_ns();
  auto wait = [&](uint32_t seq) -> bool {
    const uint64_t s0 = global_ns();
    for (uint32_t n = 1;; ++n) {
      if (ll_ld(mine).y == seq) return true;
      if ((n & 63) == 0 && global_ns() - s0 > c.timeout_ns) return false;
    }
  };
  for (int i = 0; i < p.iters; ++i) {
    if (i == p.warm) t0 = global_ns();
    const uint32_t ping = p.base + 2u * uint32_t(i), pong = ping + 1u;
    if (lead) {
      ll_put(theirs, 0u, ping);
      if (!wait(pong)) {
        atomicOr(c.status(), kStatusTimeout);
        return;
      }
    } else {
      if (!wait(ping)) {
        atomicOr(c.status(), kStatusTimeout);
        return;
      }
      ll_put(theirs, 0u, pong);
    }
  }
  *p.ns_out = global_ns() - t0;
}

}  // namespace mtpb
