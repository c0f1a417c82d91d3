// Persistent decode megakernel: one greedy decode step of the whole TP model
// in one cooperative launch (one CTA per SM).
//
// Warp 0 is a producer: one thread streams this CTA's slice of every weight
// matrix of the step (QKV, O, gate/up and down of every layer, then the LM
// head), in execution order, into a ring of shared-memory slots with 1-D bulk
// copies (cp.async.bulk, no multicast) completing on mbarriers. It runs ahead
// of the computation by up to `nslot` slots, across stage and layer
// boundaries, so HBM keeps streaming while the consumers wait on dependencies.
//
// Warps 1..15 consume. Per layer:
//   QKV  : wait for the AllReduce site of the previous down projection (or the
//          embedding) from every CTA of every rank; reduce the partials in
//          rank order, add the residual, RMSNorm (every CTA computes the full
//          vector, so every CTA holds the residual stream in shared memory);
//          GEMV rows of the packed QKV + bias -> qkv_buf (global).
//   ATT  : attention items (row, query head, KV split) spread over all warps of
//          all CTAs; RoPE of q and of the new k, online softmax over the split,
//          partial (max, sum, o) -> att_part. The split holding the new token
//          writes its K/V into the cache slot.
//   O    : merge the splits -> attention output (T) in shared memory; GEMV
//          rows of o_proj; push the T-rounded partials to every rank.
//   GU   : AllReduce site (o_proj) + residual + RMSNorm; gate/up rows ->
//          act = T(silu(T(gate)) * T(up)) -> act_buf.
//   DOWN : act from every CTA -> shared memory; GEMV rows of down_proj; push.
// Then: AllReduce site + residual + final RMSNorm; LM-head rows -> packed
// argmax per CTA; CTA 0 exchanges the winners over NVLink, writes the token,
// advances the position and the step counter.
//
// Dependencies between CTAs use per-CTA flags (release/acquire); those across
// ranks use the communicator's flags. Every wait is bounded (status word).
#pragma once

#include "comm.cuh"
#include "tma.cuh"

namespace mtpb {

constexpr int kMkThreads = 512;
constexpr int kMkCons = 15;  // consumer warps 1..15
constexpr int kMkConsThreads = kMkCons * 32;
constexpr int kMkMaxSlots = 8;
constexpr int kMkMaxM = 8;
constexpr int kLfKinds = 4;     // local flag kinds
constexpr int kLfSlots = 4096;  // flags per kind
enum : int { kLfQkv = 0, kLfAtt = 1, kLfGu = 2, kLfLm = 3 };

struct MkLayer {
  const void* ln1;
  const void* qkv_w;
  const void* qkv_b;
  const void* o_w;
  const void* ln2;
  const void* gu_w;
  const void* down_w;
  void* k_cache;
  void* v_cache;
};

struct MkParams {
  Comm comm;
  const MkLayer* layers;
  int L, H, I, hq, hkv, hd, M;
  long long vstart, vend, vocab;
  const void* embed;
  const void* lm_head;
  const void* final_norm;
  const float* cos_tab;
  const float* sin_tab;
  int rope_len;
  float eps, scale;
  int kv_cap;
  int* pos_ptr;
  long long* tok;
  long long* out_ids;
  int ld_out;
  void* logits;
  void* qkv_buf;
  float* att_part;
  void* act_buf;
  long long* lm_best;
  uint32_t* lflags;
  int nsplit;
  int nslot;
  int slot_bytes;
  int inflight;  // max weight copies outstanding per CTA (0 = up to nslot)
  int l2_hint;   // stream weights with an L2 evict-first policy
  int xin_cols;
  uint64_t budget_ns;
  // Optional stage timeline of CTA 0 (%globaltimer ns): [0] start; layer l at
  // 1 + 12 l + e for its 12 stage events; then the final LM / selection
  // events; [512 + s] the producer's first copy of weight stage s. NULL = off.
  unsigned long long* trace;
};

// CTA 0 records at [idx], the last CTA at [2048 + idx]; for layer 1 every CTA
// records its 12 stage events at [4096 + e * 1024 + cta].
#define MK_TRACE(c, p, idx)                                                               \
  do {                                                                                    \
    if ((p).trace && (c).tid == 0) {                                                      \
      const unsigned long long t_ = global_ns();                                          \
      if (blockIdx.x == 0) (p).trace[idx] = t_;                                           \
      else if (blockIdx.x == gridDim.x - 1) (p).trace[2048 + (idx)] = t_;                 \
      if ((idx) >= 13 && (idx) < 25) (p).trace[4096 + ((idx) - 13) * 1024 + blockIdx.x] = t_; \
    }                                                                                     \
  } while (0)

struct MkLayout {
  size_t xres, xnorm, xin, attq, ring, total;
};

__host__ __device__ inline size_t mk_align(size_t x) { return (x + 127) & ~size_t(127); }

__host__ __device__ inline MkLayout mk_layout(const MkParams& p, size_t tsz) {
  MkLayout l;
  size_t off = 256;  // mbarriers + control words
  l.xres = off;
  off = mk_align(off + size_t(p.M) * p.H * tsz);
  l.xnorm = off;
  off = mk_align(off + size_t(p.M) * p.H * tsz);
  l.xin = off;
  off = mk_align(off + size_t(p.M) * p.xin_cols * tsz);
  l.attq = off;
  off = mk_align(off + size_t(kMkCons) * 3 * p.hd * sizeof(float));
  l.ring = off;
  off = mk_align(off + size_t(p.nslot) * p.slot_bytes);
  l.total = off;
  return l;
}

// weight stage s (0 .. 4L): 4l+0 QKV, 4l+1 O, 4l+2 GU, 4l+3 DOWN, 4L LM head
struct MkStage {
  const char* w;
  int K;      // row length (elements)
  int units;  // rows (UR 1) or row pairs (UR 2)
  int ur;
  int half;   // UR 2: row offset of the second row of a unit
};

__device__ __forceinline__ MkStage mk_stage(const MkParams& p, int s, size_t tsz) {
  MkStage st;
  if (s == 4 * p.L) {
    st.w = static_cast<const char*>(p.lm_head);
    st.K = p.H;
    st.units = int(p.vend - p.vstart);
    st.ur = 1;
    st.half = 0;
    return st;
  }
  const MkLayer& ly = p.layers[s >> 2];
  switch (s & 3) {
    case 0:
      st.w = static_cast<const char*>(ly.qkv_w);
      st.K = p.H;
      st.units = (p.hq + 2 * p.hkv) * p.hd;
      st.ur = 1;
      break;
    case 1:
      st.w = static_cast<const char*>(ly.o_w);
      st.K = p.hq * p.hd;
      st.units = p.H;
      st.ur = 1;
      break;
    case 2:
      st.w = static_cast<const char*>(ly.gu_w);
      st.K = p.H;
      st.units = p.I;
      st.ur = 2;
      break;
    default:
      st.w = static_cast<const char*>(ly.down_w);
      st.K = p.I;
      st.units = p.H;
      st.ur = 1;
      break;
  }
  st.half = st.ur == 2 ? p.I : 0;
  (void)tsz;
  return st;
}

__device__ __forceinline__ void mk_part(int units, int& u0, int& nu) {
  const int G = gridDim.x;
  const int base = units / G, rem = units % G;
  u0 = blockIdx.x * base + min(int(blockIdx.x), rem);
  nu = base + (int(blockIdx.x) < rem ? 1 : 0);
}

__device__ __forceinline__ int mk_upc(const MkParams& p, const MkStage& st, size_t tsz) {
  const int ub = st.ur * st.K * int(tsz);
  return max(1, p.slot_bytes / ub);
}

// ---------------------------------------------------------------------------
// consumer-side helpers (all kMkConsThreads consumer threads call them)
// ---------------------------------------------------------------------------
struct MkCtx {
  int tid;  // consumer thread index 0..479
  int cw;   // consumer warp 0..14
  int lane;
  float* red;
  volatile int* abort;
};

__device__ __forceinline__ void cons_sync() { named_sync(1, kMkConsThreads); }

__device__ __forceinline__ float cons_sum(const MkCtx& c, float v) {
  v = warp_sum(v);
  cons_sync();
  if (c.lane == 0) c.red[c.cw] = v;
  cons_sync();
  float t = 0.f;
  for (int i = 0; i < kMkCons; ++i) t += c.red[i];
  return t;
}

// Bounded wait (by all consumer threads) until flags[i] reached seq for i < n.
// (consumer warp 0 polls, the other consumer warps wait at the barrier)
__device__ __forceinline__ bool cons_wait(const MkCtx& c, const uint32_t* flags, int n, uint32_t seq,
                                          bool gpu_scope, const MkParams& p) {
  if (c.cw == 0 && !*c.abort) {
    const bool ok = warp_poll_flags(flags, n, seq, !gpu_scope, p.comm.status(), p.budget_ns, c.abort);
    if (!ok && c.lane == 0) {
      *c.abort = 1;
      atomicOr(p.comm.status(), kStatusTimeout);
    }
  }
  cons_sync();
  return *c.abort == 0;
}

// AllReduce site: wait for every producer CTA of every rank (this rank's own
// CTAs included: they run concurrently with this one).
__device__ __forceinline__ bool cons_wait_site(const MkCtx& c, const MkParams& p, uint32_t seq) {
  const Comm& cm = p.comm;
  const int par = seq & 1;
  bool ok = true;
  for (int r = 0; r < cm.world && ok; ++r) {
    ok = cons_wait(c, cm.flag(cm.rank, 0, par, r, 0), gridDim.x, seq, false, p);
  }
  return ok;
}

// x = T(sum_r recv_r) [+ residual], new residual kept in xres; xnorm = RMSNorm(x) * gain
template <typename T>
__device__ __forceinline__ void cons_reduce_norm(const MkCtx& c, const MkParams& p, uint32_t seq, bool has_res,
                                                 const T* gain, T* xres, T* xnorm) {
  const Comm& cm = p.comm;
  const int par = seq & 1;
  const int H = p.H;
  for (int m = 0; m < p.M; ++m) {
    float ss = 0.f;
    for (int j = c.tid; j < H; j += kMkConsThreads) {
      const size_t off = size_t(m) * H + j;
      float s = 0.f;
      for (int r = 0; r < cm.world; ++r) s += to_f(__ldcg(reinterpret_cast<const T*>(cm.data(cm.rank, 0, par, r)) + off));
      const float o = round_t<T>(s);
      const float x = has_res ? round_t<T>(to_f(xres[off]) + o) : o;
      xres[off] = from_f<T>(x);
      ss += x * x;
    }
    const float tot = cons_sum(c, ss);
    const float rinv = rsqrtf(tot / float(H) + p.eps);
    for (int j = c.tid; j < H; j += kMkConsThreads) {
      const size_t off = size_t(m) * H + j;
      xnorm[off] = from_f<T>(__fmul_rn(__fmul_rn(to_f(xres[off]), rinv), to_f(gain[j])));
    }
  }
  cons_sync();
}

// Raise this CTA's flag of an AllReduce site on every rank (after all consumer writes).
__device__ __forceinline__ void cons_signal_site(const MkCtx& c, const MkParams& p, uint32_t seq) {
  cons_sync();
  if (c.tid == 0) {
    fence_sys();
    const int par = seq & 1;
    for (int d = 0; d < p.comm.world; ++d) st_relaxed_sys(p.comm.flag(d, 0, par, p.comm.rank, blockIdx.x), seq);
  }
}

__device__ __forceinline__ void cons_signal_local(const MkCtx& c, uint32_t* flag, uint32_t seq) {
  cons_sync();
  if (c.tid == 0) {
    fence_gpu();
    st_release_gpu(flag, seq);
  }
}

// ---------------------------------------------------------------------------
// GEMV over one ring slot: units [0, n) of the chunk, warp-strided.
// x: [M][ldx] in shared memory. Epilogue functor ep(m, unit_local, v0, v1).
// ---------------------------------------------------------------------------
template <typename T, int MT, int UR, typename Ep>
__device__ __forceinline__ void cons_gemv_chunk(const MkCtx& c, const char* slot, int n, int K, const T* x,
                                                int ldx, int M, Ep ep) {
  constexpr int VE = VecTraits<T>::kElems;
  const int cpr = K / VE;
  const size_t rb = size_t(K) * sizeof(T);
  for (int j = c.cw; j < n; j += kMkCons) {
    float acc[MT][UR];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int r = 0; r < UR; ++r) acc[m][r] = 0.f;
    const char* row0 = slot + size_t(j) * rb;
    const char* row1 = slot + size_t(n + j) * rb;  // UR 2: second row of the unit
    for (int k = c.lane; k < cpr; k += 32) {
      float wf[UR][VE];
      unpack(*reinterpret_cast<const uint4*>(row0 + size_t(k) * 16), wf[0]);
      if constexpr (UR == 2) unpack(*reinterpret_cast<const uint4*>(row1 + size_t(k) * 16), wf[1]);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < M) {
          float xf[VE];
          unpack(*reinterpret_cast<const uint4*>(x + size_t(m) * ldx + size_t(k) * VE), xf);
#pragma unroll
          for (int r = 0; r < UR; ++r)
#pragma unroll
            for (int e = 0; e < VE; ++e) acc[m][r] = fmaf(wf[r][e], xf[e], acc[m][r]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int r = 0; r < UR; ++r) acc[m][r] = warp_sum(acc[m][r]);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m < M && c.lane == m) ep(m, j, acc[m][0], UR == 2 ? acc[m][UR - 1] : 0.f);
    }
  }
}

// ---------------------------------------------------------------------------
// attention item: (row m, query head h, split sp) by one warp
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void mk_att_item(const MkCtx& c, const MkParams& p, const MkLayer& ly, int item,
                                            int pos, float* qs) {
  const int hd = p.hd, half = hd >> 1;
  const int per_m = p.hq * p.nsplit;
  const int m = item / per_m, rem = item - m * per_m;
  const int h = rem / p.nsplit, sp = rem - h * p.nsplit;
  const int Gq = p.hq / p.hkv, kvh = h / Gq;
  const int Lc = pos + 1;
  const int chunk = (Lc + p.nsplit - 1) / p.nsplit;
  const int p0 = min(Lc, sp * chunk), p1 = min(Lc, p0 + chunk);
  const int nq = (p.hq + 2 * p.hkv) * hd;
  const bool tr = p.trace && blockIdx.x == 0 && c.cw == 0 && c.lane == 0;
  if (tr) p.trace[1000] = global_ns();
  const T* row = static_cast<const T*>(p.qkv_buf) + size_t(m) * nq;
  float* q = qs;             // rotated q
  float* kn = qs + hd;       // rotated new k
  float* vn = qs + 2 * hd;   // new v
  const float* cs = p.cos_tab + size_t(pos) * hd;
  const float* sn = p.sin_tab + size_t(pos) * hd;
  for (int i = c.lane; i < half; i += 32) {
    const float qa = to_f(__ldcg(row + h * hd + i)), qb = to_f(__ldcg(row + h * hd + i + half));
    q[i] = round_t<T>(__fadd_rn(__fmul_rn(qa, cs[i]), __fmul_rn(-qb, sn[i])));
    q[i + half] = round_t<T>(__fadd_rn(__fmul_rn(qb, cs[i + half]), __fmul_rn(qa, sn[i + half])));
    const int kb = (p.hq + kvh) * hd;
    const float ka = to_f(__ldcg(row + kb + i)), kb2 = to_f(__ldcg(row + kb + i + half));
    kn[i] = round_t<T>(__fadd_rn(__fmul_rn(ka, cs[i]), __fmul_rn(-kb2, sn[i])));
    kn[i + half] = round_t<T>(__fadd_rn(__fmul_rn(kb2, cs[i + half]), __fmul_rn(ka, sn[i + half])));
    const int vb = (p.hq + p.hkv + kvh) * hd;
    vn[i] = to_f(__ldcg(row + vb + i));
    vn[i + half] = to_f(__ldcg(row + vb + i + half));
  }
  __syncwarp();
  if (tr) p.trace[1001] = global_ns();
  T* kc = static_cast<T*>(ly.k_cache) + (size_t(m) * p.hkv + kvh) * p.kv_cap * hd;
  T* vc = static_cast<T*>(ly.v_cache) + (size_t(m) * p.hkv + kvh) * p.kv_cap * hd;
  // the split holding the new token stores its K/V for later steps
  if (h % Gq == 0 && pos >= p0 && pos < p1) {
    for (int d = c.lane; d < hd; d += 32) {
      kc[size_t(pos) * hd + d] = from_f<T>(kn[d]);
      vc[size_t(pos) * hd + d] = from_f<T>(vn[d]);
    }
  }
  float mrun = -INFINITY, lrun = 0.f;
  constexpr int VE = VecTraits<T>::kElems;
  // PV layout: lane = (position group g, 16-byte dim chunk dc); the lanes of
  // one dim chunk accumulate their positions, then a shuffle reduction sums
  // the groups (every lane ends with the sums of its dim chunk).
  const int dch = hd / VE;      // dim chunks per row (power of two <= 32)
  const int pg = 32 / dch;      // position groups
  const int dc = c.lane % dch, g = c.lane / dch;
  float o[VE];
#pragma unroll
  for (int e = 0; e < VE; ++e) o[e] = 0.f;
  for (int t0 = p0; t0 < p1; t0 += 32) {
    const int pp = t0 + c.lane;
    float s = -INFINITY;
    if (pp < p1) {
      float d = 0.f;
      if (pp == pos) {
        for (int e = 0; e < hd; ++e) d = fmaf(q[e], kn[e], d);
      } else {
        // the whole key row in flight at once (head_dim <= 128)
        const T* kr = kc + size_t(pp) * hd;
        constexpr int NV = 128 / VE;
        uint4 kv[NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) kv[v] = v * VE < hd ? ld_vec(kr + v * VE) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int v = 0; v < NV; ++v) {
          if (v * VE < hd) {
            float kf[VE];
            unpack(kv[v], kf);
#pragma unroll
            for (int e = 0; e < VE; ++e) d = fmaf(q[v * VE + e], kf[e], d);
          }
        }
      }
      s = d * p.scale;
    }
    if (tr && t0 == p0) p.trace[1002] = global_ns();
    float tmax = s;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
    const float mnew = fmaxf(mrun, tmax);
    const float corr = mrun == -INFINITY ? 0.f : expf(mrun - mnew);
    const float pl = pp < p1 ? expf(s - mnew) : 0.f;
    lrun = lrun * corr + warp_sum(pl);
    mrun = mnew;
    const int nt = min(32, p1 - t0);
    // all value loads of this lane first (at most 16 rows), then the FMAs
    constexpr int MAXIT = 16;
    uint4 vv[MAXIT];
#pragma unroll
    for (int it = 0; it < MAXIT; ++it) {
      const int j = it * pg + g;
      vv[it] = make_uint4(0, 0, 0, 0);
      if (it * pg < 32 && j < nt && t0 + j != pos) vv[it] = ld_vec(vc + size_t(t0 + j) * hd + dc * VE);
    }
    float part[VE];
#pragma unroll
    for (int e = 0; e < VE; ++e) part[e] = 0.f;
#pragma unroll
    for (int it = 0; it < MAXIT; ++it) {
      const int j = it * pg + g;
      const float pj = __shfl_sync(0xffffffffu, pl, j & 31);
      if (it * pg < 32 && j < nt) {
        float vf[VE];
        if (t0 + j == pos) {
#pragma unroll
          for (int e = 0; e < VE; ++e) vf[e] = vn[dc * VE + e];
        } else {
          unpack(vv[it], vf);
        }
#pragma unroll
        for (int e = 0; e < VE; ++e) part[e] = fmaf(pj, vf[e], part[e]);
      }
    }
    for (int off = dch; off < 32; off <<= 1) {
#pragma unroll
      for (int e = 0; e < VE; ++e) part[e] += __shfl_xor_sync(0xffffffffu, part[e], off);
    }
#pragma unroll
    for (int e = 0; e < VE; ++e) o[e] = fmaf(o[e], corr, part[e]);
  }
  if (tr) p.trace[1003] = global_ns();
  float* dst = p.att_part + size_t(item) * (hd + 2);
  if (g == 0) {
#pragma unroll
    for (int e = 0; e < VE; ++e) dst[dc * VE + e] = o[e];
  }
  if (c.lane == 0) {
    dst[hd] = p1 > p0 ? mrun : -INFINITY;
    dst[hd + 1] = lrun;
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <typename T, int MT>
__global__ void __launch_bounds__(kMkThreads, 1) decode_mk_kernel(const MkParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float red[32];
  __shared__ long long bests[kMkCons][kMkMaxM];
  __shared__ int never;  // stays 0: "no abort" for the final drain
  const size_t tsz = sizeof(T);
  const MkLayout lay = mk_layout(p, tsz);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMkMaxSlots;
  volatile int* abort = reinterpret_cast<volatile int*>(smem + 2 * kMkMaxSlots * 8);
  T* xres = reinterpret_cast<T*>(smem + lay.xres);
  T* xnorm = reinterpret_cast<T*>(smem + lay.xnorm);
  T* xin = reinterpret_cast<T*>(smem + lay.xin);
  float* attq = reinterpret_cast<float*>(smem + lay.attq);
  char* ring = reinterpret_cast<char*>(smem + lay.ring);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // step and position of this decode step (written by the previous step)
  const uint32_t step = ld_volatile_u32(p.comm.ctl() + kCtlStep) + 1u;
  const int pos = *reinterpret_cast<volatile int*>(p.pos_ptr);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nslot; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, kMkCons);
    }
    never = 0;
    *abort = 0;
    if (pos < 0 || pos >= p.kv_cap || pos >= p.rope_len) {
      *abort = 1;
      atomicOr(p.comm.status(), kStatusBadPosition);
    }
    mbar_init_fence();
  }
  __syncthreads();
  const uint32_t nsite = uint32_t(2 * p.L + 2);
  const uint32_t nloc = uint32_t(3 * p.L + 1);
  auto site_seq = [&](int site) { return step * nsite + uint32_t(site) + 1u; };
  auto loc_seq = [&](int k) { return step * nloc + uint32_t(k) + 1u; };
  const int nstages = 4 * p.L + 1;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int k = 0;
      bool stop = false;
      const uint64_t pol = l2_evict_first_policy();
      for (int s = 0; s < nstages && !stop; ++s) {
        const MkStage st = mk_stage(p, s, tsz);
        int u0, nu;
        mk_part(st.units, u0, nu);
        const int upc = mk_upc(p, st, tsz);
        const size_t rb = size_t(st.K) * tsz;
        for (int c = 0; c < nu; c += upc, ++k) {
          const int n = min(upc, nu - c);
          const int slot = k % p.nslot;
          if (k >= p.nslot && !mbar_wait(empty + slot, ((k / p.nslot) - 1) & 1, p.budget_ns, abort)) {
            *abort = 1;
            atomicOr(p.comm.status(), kStatusTimeout);
            stop = true;
            break;
          }
          // at most `inflight` copies outstanding: the ring may hold more landed
          // chunks, but deeper DRAM queues only delay the consumers' loads
          if (p.inflight > 0 && k >= p.inflight) {
            const int kk = k - p.inflight;
            mbar_wait(full + (kk % p.nslot), (kk / p.nslot) & 1, p.budget_ns, abort);
          }
          if (*abort) {
            stop = true;
            break;
          }
          char* dst = ring + size_t(slot) * p.slot_bytes;
          const uint32_t bytes = uint32_t(st.ur * n * rb);
          if (c == 0 && p.trace && blockIdx.x == 0) p.trace[512 + s] = global_ns();
          mbar_arrive_expect_tx(full + slot, bytes);
          if (p.l2_hint) {
            bulk_g2s_hint(dst, st.w + size_t(u0 + c) * rb, uint32_t(n * rb), full + slot, pol);
            if (st.ur == 2)
              bulk_g2s_hint(dst + n * rb, st.w + size_t(st.half + u0 + c) * rb, uint32_t(n * rb), full + slot, pol);
          } else {
            bulk_g2s(dst, st.w + size_t(u0 + c) * rb, uint32_t(n * rb), full + slot);
            if (st.ur == 2) bulk_g2s(dst + n * rb, st.w + size_t(st.half + u0 + c) * rb, uint32_t(n * rb), full + slot);
          }
        }
      }
      // drain: the copies in flight must land before the CTA exits
      const int issued = k;
      for (int i = max(0, issued - p.nslot); i < issued; ++i) {
        mbar_wait(full + (i % p.nslot), (i / p.nslot) & 1, p.budget_ns, &never);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    MkCtx c;
    c.tid = threadIdx.x - 32;
    c.cw = warp - 1;
    c.lane = lane;
    c.red = red;
    c.abort = abort;
    const Comm& cm = p.comm;
    const int G = gridDim.x;
    int k = 0;  // chunk counter (matches the producer)
    bool alive = true;
    const int VEx = VecTraits<T>::kElems;

    // consume all chunks of weight stage s with epilogue ep; x: [M][ldx]
    auto run_stage = [&](int s, const T* x, int ldx, auto ep) {
      const MkStage st = mk_stage(p, s, tsz);
      int u0, nu;
      mk_part(st.units, u0, nu);
      const int upc = mk_upc(p, st, tsz);
      for (int cc = 0; cc < nu; cc += upc, ++k) {
        const int n = min(upc, nu - cc);
        const int slot = k % p.nslot;
        const char* sl = ring + size_t(slot) * p.slot_bytes;
        if (!mbar_wait(full + slot, (k / p.nslot) & 1, p.budget_ns, abort)) {
          *abort = 1;
          atomicOr(cm.status(), kStatusTimeout);
        }
        if (!*abort) {
          auto epu = [&](int m, int j, float v0, float v1) { ep(m, u0 + cc + j, v0, v1); };
          if (st.ur == 2)
            cons_gemv_chunk<T, MT, 2>(c, sl, n, st.K, x, ldx, p.M, epu);
          else
            cons_gemv_chunk<T, MT, 1>(c, sl, n, st.K, x, ldx, p.M, epu);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot);
      }
    };

    MK_TRACE(c, p, 0);
    // ---- embedding -> site 0 (this CTA's column slice of every row)
    if (!*abort) {
      int j0, nj;
      mk_part(p.H, j0, nj);
      const uint32_t seq = site_seq(0);
      const int par = seq & 1;
      for (int i = c.tid; i < p.M * nj; i += kMkConsThreads) {
        const int m = i / nj, j = j0 + (i - m * nj);
        const long long id = p.tok[m];
        if ((id < 0 || id >= p.vocab) && j == j0) atomicOr(cm.status(), kStatusBadToken);
        const bool mine = id >= p.vstart && id < p.vend;
        const T v = mine ? static_cast<const T*>(p.embed)[size_t(id - p.vstart) * p.H + j] : from_f<T>(0.f);
        for (int d = 0; d < cm.world; ++d) reinterpret_cast<T*>(cm.data(d, 0, par, cm.rank))[size_t(m) * p.H + j] = v;
      }
      cons_signal_site(c, p, seq);
    }
    const int nq = (p.hq + 2 * p.hkv) * p.hd;
    const int n_items = p.M * p.hq * p.nsplit;
    float* qs = attq + size_t(c.cw) * 3 * p.hd;

    for (int l = 0; l < p.L && alive; ++l) {
      const MkLayer ly = p.layers[l];
      // ---- QKV
      alive = cons_wait_site(c, p, site_seq(2 * l));
      if (!alive) break;
      const int tb = 1 + 12 * l;
      MK_TRACE(c, p, tb + 0);
      cons_reduce_norm<T>(c, p, site_seq(2 * l), l > 0, static_cast<const T*>(ly.ln1), xres, xnorm);
      MK_TRACE(c, p, tb + 1);
      {
        const T* bias = static_cast<const T*>(ly.qkv_b);
        T* out = static_cast<T*>(p.qkv_buf);
        run_stage(4 * l, xnorm, p.H, [&](int m, int u, float v0, float) {
          float v = v0;
          if (bias) v += to_f(bias[u]);
          out[size_t(m) * nq + u] = from_f<T>(v);
        });
      }
      MK_TRACE(c, p, tb + 2);
      cons_signal_local(c, p.lflags + kLfQkv * kLfSlots + blockIdx.x, loc_seq(3 * l));
      // ---- attention items
      {
        alive = cons_wait(c, p.lflags + kLfQkv * kLfSlots, G, loc_seq(3 * l), true, p);
        if (!alive) break;
        MK_TRACE(c, p, tb + 3);
        for (int it = blockIdx.x + G * c.cw; it < n_items; it += G * kMkCons) {
          mk_att_item<T>(c, p, ly, it, pos, qs);
          __syncwarp();
          if (lane == 0) {
            fence_gpu();
            st_release_gpu(p.lflags + kLfAtt * kLfSlots + it, loc_seq(3 * l + 1));
          }
          __syncwarp();
        }
        MK_TRACE(c, p, tb + 4);
      }
      // ---- O: merge attention splits into xin, GEMV, push site 2l+1
      alive = cons_wait(c, p.lflags + kLfAtt * kLfSlots, n_items, loc_seq(3 * l + 1), true, p);
      if (!alive) break;
      MK_TRACE(c, p, tb + 5);
      {
        // merge the splits: weights w_s = exp(m_s - max) / sum_s exp(m_s - max) l_s
        // per (row, head) into shared memory (reusing the attention scratch)
        const int hd = p.hd;
        const int pairs = p.M * p.hq;
        float* wts = attq;  // [pairs][nsplit]; sized by the host (<= 15 * 3 * hd floats)
        for (int pr = c.tid; pr < pairs; pr += kMkConsThreads) {
          const float* base = p.att_part + size_t(pr) * p.nsplit * (hd + 2);
          float mx = -INFINITY;
          for (int s0 = 0; s0 < p.nsplit; s0 += 8) {
            float ms[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
              ms[u] = s0 + u < p.nsplit ? __ldcg(base + size_t(s0 + u) * (hd + 2) + hd) : -INFINITY;
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              mx = fmaxf(mx, ms[u]);
              if (s0 + u < p.nsplit) wts[size_t(pr) * p.nsplit + s0 + u] = ms[u];
            }
          }
          float den = 0.f;
          for (int s0 = 0; s0 < p.nsplit; s0 += 8) {
            float ls[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) ls[u] = s0 + u < p.nsplit ? __ldcg(base + size_t(s0 + u) * (hd + 2) + hd + 1) : 0.f;
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              if (s0 + u < p.nsplit) {
                const float ms = wts[size_t(pr) * p.nsplit + s0 + u];
                const float w = ms == -INFINITY ? 0.f : expf(ms - mx);
                wts[size_t(pr) * p.nsplit + s0 + u] = w;
                den = fmaf(w, ls[u], den);
              }
            }
          }
          const float inv = 1.0f / den;
          for (int s = 0; s < p.nsplit; ++s) wts[size_t(pr) * p.nsplit + s] *= inv;
        }
        cons_sync();
        for (int i = c.tid; i < pairs * hd; i += kMkConsThreads) {
          const int pr = i / hd, d = i - pr * hd;
          const float* base = p.att_part + size_t(pr) * p.nsplit * (hd + 2) + d;
          const float* w = wts + size_t(pr) * p.nsplit;
          float acc = 0.f;
          for (int s0 = 0; s0 < p.nsplit; s0 += 8) {
            float ov[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) ov[u] = s0 + u < p.nsplit ? __ldcg(base + size_t(s0 + u) * (hd + 2)) : 0.f;
#pragma unroll
            for (int u = 0; u < 8; ++u)
              if (s0 + u < p.nsplit) acc = fmaf(w[s0 + u], ov[u], acc);
          }
          const int m = pr / p.hq, r = (pr - m * p.hq) * hd + d;
          xin[size_t(m) * p.xin_cols + r] = from_f<T>(acc);
        }
        cons_sync();
        MK_TRACE(c, p, tb + 6);
        const uint32_t seq = site_seq(2 * l + 1);
        const int par = seq & 1;
        run_stage(4 * l + 1, xin, p.xin_cols, [&](int m, int u, float v0, float) {
          const T v = from_f<T>(v0);
          for (int d = 0; d < cm.world; ++d)
            reinterpret_cast<T*>(cm.data(d, 0, par, cm.rank))[size_t(m) * p.H + u] = v;
        });
        cons_signal_site(c, p, seq);
      }
      MK_TRACE(c, p, tb + 7);
      // ---- GU
      alive = cons_wait_site(c, p, site_seq(2 * l + 1));
      if (!alive) break;
      MK_TRACE(c, p, tb + 8);
      cons_reduce_norm<T>(c, p, site_seq(2 * l + 1), true, static_cast<const T*>(ly.ln2), xres, xnorm);
      {
        T* act = static_cast<T*>(p.act_buf);
        run_stage(4 * l + 2, xnorm, p.H, [&](int m, int u, float g, float up) {
          const float gr = round_t<T>(g), ur = round_t<T>(up);
          const float a = round_t<T>(gr / (1.0f + expf(-gr))) * ur;
          act[size_t(m) * p.I + u] = from_f<T>(a);
        });
      }
      MK_TRACE(c, p, tb + 9);
      cons_signal_local(c, p.lflags + kLfGu * kLfSlots + blockIdx.x, loc_seq(3 * l + 2));
      // ---- DOWN
      alive = cons_wait(c, p.lflags + kLfGu * kLfSlots, G, loc_seq(3 * l + 2), true, p);
      if (!alive) break;
      MK_TRACE(c, p, tb + 10);
      {
        const int vpr = p.I / VEx;
        const T* act = static_cast<const T*>(p.act_buf);
        for (int i = c.tid; i < p.M * vpr; i += kMkConsThreads) {
          const int m = i / vpr, v = i - m * vpr;
          *reinterpret_cast<uint4*>(xin + size_t(m) * p.xin_cols + size_t(v) * VEx) =
              __ldcg(reinterpret_cast<const uint4*>(act + size_t(m) * p.I) + v);
        }
        cons_sync();
        const uint32_t seq = site_seq(2 * l + 2);
        const int par = seq & 1;
        run_stage(4 * l + 3, xin, p.xin_cols, [&](int m, int u, float v0, float) {
          const T v = from_f<T>(v0);
          for (int d = 0; d < cm.world; ++d)
            reinterpret_cast<T*>(cm.data(d, 0, par, cm.rank))[size_t(m) * p.H + u] = v;
        });
        cons_signal_site(c, p, seq);
      }
      MK_TRACE(c, p, tb + 11);
    }

    // ---- final norm + LM head + packed argmax
    if (alive) alive = cons_wait_site(c, p, site_seq(2 * p.L));
    if (alive) {
      MK_TRACE(c, p, 1 + 12 * p.L);
      cons_reduce_norm<T>(c, p, site_seq(2 * p.L), true, static_cast<const T*>(p.final_norm), xres, xnorm);
      long long best[kMkMaxM];
#pragma unroll
      for (int m = 0; m < kMkMaxM; ++m) best[m] = kArgmaxEmpty;
      const bool nan_wins = cm.world == 1;
      const int vloc = int(p.vend - p.vstart);
      T* lg = static_cast<T*>(p.logits);
      run_stage(4 * p.L, xnorm, p.H, [&](int m, int u, float v0, float) {
        const float v = round_t<T>(v0);
        if (lg) lg[size_t(m) * vloc + u] = from_f<T>(v);
        const long long pk = argmax_pack(v, uint32_t(p.vstart) + uint32_t(u), nan_wins);
#pragma unroll
        for (int mm = 0; mm < kMkMaxM; ++mm)
          if (mm == m) best[mm] = pk > best[mm] ? pk : best[mm];
      });
      // lane m holds the best of row m for this warp
#pragma unroll
      for (int m = 0; m < kMkMaxM; ++m) {
        long long b = best[m];
        b = warp_max_ll(b);
        if (lane == 0) bests[c.cw][m] = b;
      }
      cons_sync();
      if (c.tid < p.M) {
        long long b = kArgmaxEmpty;
        for (int w = 0; w < kMkCons; ++w) b = bests[w][c.tid] > b ? bests[w][c.tid] : b;
        p.lm_best[size_t(blockIdx.x) * kMkMaxM + c.tid] = b;
        if (c.tid == 0 && p.trace && blockIdx.x == 0) p.trace[2 + 12 * p.L] = global_ns();
      }
      cons_signal_local(c, p.lflags + kLfLm * kLfSlots + blockIdx.x, loc_seq(3 * p.L));
      // ---- CTA 0: cross-CTA and cross-rank selection, token write, advance
      if (blockIdx.x == 0) {
        alive = cons_wait(c, p.lflags + kLfLm * kLfSlots, G, loc_seq(3 * p.L), true, p);
        if (alive) {
          const uint32_t seq = site_seq(2 * p.L + 1);
          const int par = seq & 1;
          if (c.tid < p.M) {
            long long b = kArgmaxEmpty;
            for (int g = 0; g < G; ++g) {
              const long long u = __ldcg(p.lm_best + size_t(g) * kMkMaxM + c.tid);
              b = u > b ? u : b;
            }
            for (int d = 0; d < cm.world; ++d) reinterpret_cast<long long*>(cm.data(d, 0, par, cm.rank))[c.tid] = b;
          }
          if (cm.world > 1) {
            cons_signal_site(c, p, seq);
            bool ok = true;
            for (int r = 0; r < cm.world && ok; ++r) ok = cons_wait(c, cm.flag(cm.rank, 0, par, r, 0), 1, seq, false, p);
            alive = ok;
          } else {
            cons_sync();
          }
          if (alive && c.tid < p.M) {
            long long b = kArgmaxEmpty;
            for (int r = 0; r < cm.world; ++r) {
              const long long u = __ldcg(reinterpret_cast<const long long*>(cm.data(cm.rank, 0, par, r)) + c.tid);
              b = u > b ? u : b;
            }
            const long long tk = argmax_id(b);
            p.tok[c.tid] = tk;
            if (p.out_ids) p.out_ids[size_t(c.tid) * p.ld_out + pos + 1] = tk;
          }
          cons_sync();
          if (alive && c.tid == 0) {
            *reinterpret_cast<volatile int*>(p.pos_ptr) = pos + 1;
            cm.ctl()[kCtlStep] = step;
            if (p.trace) p.trace[3 + 12 * p.L] = global_ns();
          }
        }
      }
    }
    // a consumer that stopped early still releases every slot the producer fills
    (void)alive;
  }
  __syncthreads();
}

}  // namespace mtpb
