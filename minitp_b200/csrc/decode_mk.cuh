// Persistent decode megakernel: one greedy decode step of the whole TP model
// in one cooperative launch (one CTA per SM).
//
// Warp 0 is a producer: one thread streams this CTA's slice of every weight
// matrix of the step (QKV, O, gate/up and down of every layer, then the LM
// head), in execution order, into a ring of shared-memory slots with 1-D bulk
// copies (cp.async.bulk, no multicast) completing on mbarriers. Weights do not
// depend on activations, so the stream runs ahead by up to `nslot` slots,
// across stage and layer boundaries, while the consumers wait on data.
//
// Warps 1..15 consume. Per layer:
//   QKV  : AllReduce site of the previous down projection (or the embedding):
//          partials of every CTA of every rank, summed in rank order, plus the
//          residual, RMSNorm (every CTA computes the full vector and keeps the
//          residual stream in shared memory); GEMV rows of the packed QKV.
//   ATT  : attention items (row, query head, 32-position KV split) spread
//          over the CTAs; RoPE of q and of the new k, softmax over the split,
//          partial (o, max, sum). The cached K/V rows of an item are staged
//          into shared memory by bulk copies issued a layer ahead. The split
//          holding the new token writes its K/V into the cache slot.
//   O    : merge the splits of every head; GEMV rows of o_proj; push the
//          T-rounded outputs to every rank (AllReduce site).
//   GU   : AllReduce site + residual + RMSNorm; gate/up rows ->
//          act = T(silu(T(gate)) * T(up)).
//   DOWN : gather act; GEMV rows of down_proj; push (AllReduce site).
// Then: AllReduce site + residual + final RMSNorm; LM-head rows -> packed
// argmax per CTA; CTA 0 reduces the CTAs, exchanges the winner with the other
// ranks, writes the token and advances the position.
//
// Every value that crosses CTAs or ranks travels as an LL word: 8 bytes
// {payload, sequence number} written by one aligned 64-bit store. Such a store
// is single-copy atomic, so a reader (64-bit loads) that sees the expected
// sequence number in a word also sees that word's payload; no memory fence
// and no flag is needed.
// Readers spin (bounded) on the words themselves. Sequence numbers grow with
// the step counter, which every launch advances, so no word of an earlier
// step or launch matches.
#pragma once

#include <type_traits>

#include "comm.cuh"
#include "tma.cuh"

namespace mtpb {

constexpr int kMkThreads = 512;
constexpr int kMkCons = 15;  // consumer warps 1..15
constexpr int kMkConsThreads = kMkCons * 32;
constexpr int kMkMaxSlots = 8;
constexpr int kMkMaxM = 8;
constexpr int kMkSplit = 32;      // KV positions per attention item (one per lane)
constexpr int kMkMaxSplits = 128;
constexpr int kMkMaxStage = 16;   // attention items per CTA staged in shared memory
constexpr int kMkChan = 2;        // communicator channel of the AllReduce sites
constexpr int kMkHdr = 1024;      // shared-memory header: mbarriers + control words

// ---------------------------------------------------------------------------
// LL words
// ---------------------------------------------------------------------------
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
__device__ __noinline__ LLSpin ll_spin_any(const uint64_t* src, uint32_t seq, int wide, uint64_t budget_ns,
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

// ---------------------------------------------------------------------------
// parameters
// ---------------------------------------------------------------------------
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
  uint64_t* qkv_ll;  // [M][nq / kPer] LL words
  uint64_t* att_ll;  // [items][hd + 2] LL words (fp32): o, then (max, sum)
  uint64_t* act_ll;  // [M][I / kPer]
  uint64_t* lm_ll;   // [CTA][kMkMaxM][2] packed argmax as two LL words
  int nsplit;        // KV splits of the cache capacity (upper bound)
  int att_stage;     // attention items per CTA staged in shared memory
  int nslot;
  int slot_bytes;
  int inflight;  // max weight copies outstanding per CTA (0 = up to nslot)
  int l2_hint;   // stream weights with an L2 evict-first policy
  int xin_cols;
  int wsc_floats;  // kMkCons * 3 * hd (attention items) + 2 * M * hq * nsplit (split merge)
  uint64_t budget_ns;
  uint32_t spin_ns;  // back-off between polls of a word that is not there yet
  // Optional stage timeline (%globaltimer ns): CTA 0 at [idx], the last CTA at
  // [2048 + idx], every CTA's layer-1 events at [4096 + e * 1024 + cta];
  // [0] start, [1 + 12 l + e] stage event e of layer l, then the LM head and
  // selection events, [512 + s] CTA 0's first copy of weight stage s,
  // [1000 ..] phases of CTA 0's first attention item, [1100 + 40 (s - 4) + 2 i]
  // CTA 0's chunk i of layer-1 stage s ready / consumed, [1300 + 20 (s - 4) + i]
  // its copy issued. NULL = off.
  unsigned long long* trace;
};

// Slow path of an LL read: spin (bounded) until the word / pair carries seq.
__device__ __forceinline__ bool ll_spin(const MkParams& p, const uint64_t* src, uint32_t seq, uint2& v,
                                        volatile int* abort) {
  const LLSpin r = ll_spin_any(src, seq, 0, p.budget_ns, abort, p.spin_ns);
  v = make_uint2(r.v.x, r.v.y);
  return r.ok != 0;
}
__device__ __forceinline__ bool ll_spin2(const MkParams& p, const uint64_t* src, uint32_t seq, uint4& v,
                                         volatile int* abort) {
  const LLSpin r = ll_spin_any(src, seq, 1, p.budget_ns, abort, p.spin_ns);
  v = r.v;
  return r.ok != 0;
}

#define MK_TRACE(c, p, idx)                                                                   \
  do {                                                                                        \
    if ((p).trace && (c).tid == 0) {                                                          \
      const unsigned long long t_ = global_ns();                                              \
      if (blockIdx.x == 0) (p).trace[idx] = t_;                                               \
      else if (blockIdx.x == gridDim.x - 1) (p).trace[2048 + (idx)] = t_;                     \
      if ((idx) >= 13 && (idx) < 25) (p).trace[4096 + ((idx) - 13) * 1024 + blockIdx.x] = t_; \
    }                                                                                         \
  } while (0)

struct MkLayout {
  size_t lys, xres, xnorm, xin, wsc, stg, ring, total;
};

__host__ __device__ inline size_t mk_align(size_t x) { return (x + 127) & ~size_t(127); }

__host__ __device__ inline size_t mk_stage_bytes(const MkParams& p, size_t tsz) {
  return size_t(2) * kMkSplit * p.hd * tsz;  // K and V rows of one item
}

__host__ __device__ inline MkLayout mk_layout(const MkParams& p, size_t tsz) {
  MkLayout l;
  size_t off = kMkHdr;
  l.lys = off;
  off = mk_align(off + size_t(p.L) * sizeof(MkLayer));
  l.xres = off;
  off = mk_align(off + size_t(p.M) * p.H * tsz);
  l.xnorm = off;
  off = mk_align(off + size_t(p.M) * p.H * tsz);
  l.xin = off;
  off = mk_align(off + size_t(p.M) * p.xin_cols * tsz);
  l.wsc = off;
  off = mk_align(off + size_t(p.wsc_floats) * sizeof(float));
  l.stg = off;
  off = mk_align(off + size_t(p.att_stage) * mk_stage_bytes(p, tsz));
  l.ring = off;
  off = mk_align(off + size_t(p.nslot) * p.slot_bytes);
  l.total = off;
  return l;
}

// Weight stage s (0 .. 4L): 4l+0 QKV, 4l+1 O, 4l+2 gate/up, 4l+3 down, 4L LM
// head. A GEMV unit is `rpu` consecutive rows of each of `halves` row blocks
// (gate/up: unit u takes gate rows u*rpu.. and up rows hoff + u*rpu..), so a
// unit's outputs fill whole LL words.
struct MkStage {
  const char* w;
  int K;  // row length (elements)
  int units;
  int rpu;
  int halves;
  int hoff;
};

template <typename T>
__device__ __forceinline__ MkStage mk_stage(const MkParams& p, const MkLayer* lys, int s) {
  constexpr int P = LLPack<T>::kPer;
  MkStage st;
  st.rpu = P;
  st.halves = 1;
  st.hoff = 0;
  if (s == 4 * p.L) {
    st.w = static_cast<const char*>(p.lm_head);
    st.K = p.H;
    st.units = int(p.vend - p.vstart);
    st.rpu = 1;
    return st;
  }
  const MkLayer& ly = lys[s >> 2];
  switch (s & 3) {
    case 0:
      st.w = static_cast<const char*>(ly.qkv_w);
      st.K = p.H;
      st.units = (p.hq + 2 * p.hkv) * p.hd / P;
      break;
    case 1:
      st.w = static_cast<const char*>(ly.o_w);
      st.K = p.hq * p.hd;
      st.units = p.H / P;
      break;
    case 2:
      st.w = static_cast<const char*>(ly.gu_w);
      st.K = p.H;
      st.units = p.I / P;
      st.halves = 2;
      st.hoff = p.I;
      break;
    default:
      st.w = static_cast<const char*>(ly.down_w);
      st.K = p.I;
      st.units = p.H / P;
      break;
  }
  return st;
}

__device__ __forceinline__ void mk_part(int units, int& u0, int& nu) {
  const int G = gridDim.x;
  const int base = units / G, rem = units % G;
  u0 = blockIdx.x * base + min(int(blockIdx.x), rem);
  nu = base + (int(blockIdx.x) < rem ? 1 : 0);
}

__device__ __forceinline__ int mk_upc(const MkParams& p, const MkStage& st, size_t tsz) {
  const int ub = st.halves * st.rpu * st.K * int(tsz);
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

// Barrier over the consumers that also ORs `v` over them: every consumer
// thread gets the same answer, so decisions taken on it stay uniform.
__device__ __forceinline__ bool cons_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, 1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v)), "r"(kMkConsThreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ float cons_sum(const MkCtx& c, float v) {
  v = warp_sum(v);
  cons_sync();
  if (c.lane == 0) c.red[c.cw] = v;
  cons_sync();
  float t = 0.f;
  for (int i = 0; i < kMkCons; ++i) t += c.red[i];
  return t;
}

__device__ __forceinline__ void mk_fail(const MkCtx& c, const MkParams& p) {
  *c.abort = 1;
  atomicOr(p.comm.status(), kStatusTimeout);
}

__device__ __forceinline__ uint64_t* mk_site(const MkParams& p, int dst, int site, int src) {
  return reinterpret_cast<uint64_t*>(p.comm.data(dst, kMkChan, site & 1, src));
}

// AllReduce site: x = T(sum_r partial_r) [+ residual] -> xres (new residual),
// xnorm = RMSNorm(x) * gain. Partials of rank r are read in rank order, so
// every rank computes the same bits. False on timeout.
template <typename T>
__device__ __forceinline__ bool cons_reduce_norm(const MkCtx& c, const MkParams& p, int site, uint32_t seq,
                                                 bool has_res, const T* gain, T* xres, T* xnorm) {
  constexpr int P = LLPack<T>::kPer;
  const Comm& cm = p.comm;
  const int H = p.H, W = H / P, nl = W / 2;
  bool ok = !*c.abort;
  for (int m = 0; m < p.M; ++m) {
    float ss = 0.f;
    for (int i = c.tid; i < nl && ok; i += kMkConsThreads) {
      float s[2 * P];
#pragma unroll
      for (int e = 0; e < 2 * P; ++e) s[e] = 0.f;
      // two ranks' pairs in flight at a time; summed in rank order
      for (int r0 = 0; r0 < cm.world; r0 += 2) {
        uint4 v[2];
#pragma unroll
        for (int u = 0; u < 2; ++u)
          if (r0 + u < cm.world) v[u] = ll_ld2(mk_site(p, cm.rank, site, r0 + u) + size_t(m) * W + 2 * i);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          if (r0 + u < cm.world && ok) {
            if (!ll_ok2(v[u], seq) &&
                !ll_spin2(p, mk_site(p, cm.rank, site, r0 + u) + size_t(m) * W + 2 * i, seq, v[u], c.abort))
              ok = false;
            float f[2 * P];
            LLPack<T>::unpack(v[u].x, f);
            LLPack<T>::unpack(v[u].z, f + P);
#pragma unroll
            for (int e = 0; e < 2 * P; ++e) s[e] += f[e];
          }
        }
      }
      if (!ok) break;
#pragma unroll
      for (int e = 0; e < 2 * P; ++e) {
        const size_t off = size_t(m) * H + size_t(i) * 2 * P + e;
        const float o = round_t<T>(s[e]);
        const float x = has_res ? round_t<T>(to_f(xres[off]) + o) : o;
        xres[off] = from_f<T>(x);
        ss += x * x;
      }
    }
    if (!ok && !*c.abort) mk_fail(c, p);
    const float tot = cons_sum(c, ss);
    const float rinv = rsqrtf(tot / float(H) + p.eps);
    for (int j = c.tid; j < H; j += kMkConsThreads) {
      const size_t off = size_t(m) * H + j;
      xnorm[off] = from_f<T>(__fmul_rn(__fmul_rn(to_f(xres[off]), rinv), to_f(gain[j])));
    }
  }
  return !cons_sync_or(!ok || *c.abort);
}

// Gather `n` LL words per row (n even) of M rows into T dst[m * ldd + ...].
template <typename T>
__device__ __forceinline__ bool cons_gather(const MkCtx& c, const MkParams& p, const uint64_t* src, int n,
                                            uint32_t seq, T* dst, int ldd) {
  constexpr int P = LLPack<T>::kPer;
  constexpr int NB = 4;
  const int nl = n / 2, tot = p.M * nl;
  bool ok = !*c.abort;
  for (int b0 = c.tid; b0 < tot && ok; b0 += NB * kMkConsThreads) {
    uint4 v[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const int i = b0 + b * kMkConsThreads;
      if (i < tot) {
        const int m = i / nl, w = i - m * nl;
        v[b] = ll_ld2(src + size_t(m) * n + 2 * w);
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const int i = b0 + b * kMkConsThreads;
      if (i < tot && ok) {
        const int m = i / nl, w = i - m * nl;
        if (!ll_ok2(v[b], seq) && !ll_spin2(p, src + size_t(m) * n + 2 * w, seq, v[b], c.abort))
          ok = false;
        float f[2 * P];
        LLPack<T>::unpack(v[b].x, f);
        LLPack<T>::unpack(v[b].z, f + P);
#pragma unroll
        for (int e = 0; e < 2 * P; ++e) dst[size_t(m) * ldd + size_t(w) * 2 * P + e] = from_f<T>(f[e]);
      }
    }
  }
  if (!ok && !*c.abort) mk_fail(c, p);
  return !cons_sync_or(!ok || *c.abort);
}

// ---------------------------------------------------------------------------
// GEMV over one ring slot: n units of NR rows (RPU rows of NR / RPU halves).
// x: [M][ldx] in shared memory. With fewer units than warps, K is split over
// warps and the partial sums are added in a fixed order. ep(m, unit, v[NR]).
// ---------------------------------------------------------------------------
template <typename T, int MT, int NR, int RPU, typename Ep>
__device__ __forceinline__ void cons_gemv_chunk(const MkCtx& c, const char* slot, int n, int K, const T* x,
                                                int ldx, int M, float* kred, Ep ep) {
  constexpr int VE = VecTraits<T>::kElems;
  const int cpr = K / VE;
  const size_t rb = size_t(K) * sizeof(T);
  const int kp = n >= kMkCons ? 1 : max(1, min(kMkCons / n, cpr / 32));
  const int nw = n * kp;
  for (int w = c.cw; w < nw; w += kMkCons) {
    const int j = w % n, q = w / n;
    const char* rows[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) rows[r] = slot + (size_t((r / RPU) * n + j) * RPU + (r % RPU)) * rb;
    float acc[MT][NR];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int r = 0; r < NR; ++r) acc[m][r] = 0.f;
    for (int k = q * 32 + c.lane; k < cpr; k += kp * 32) {
      float wf[NR][VE];
#pragma unroll
      for (int r = 0; r < NR; ++r) unpack(*reinterpret_cast<const uint4*>(rows[r] + size_t(k) * 16), wf[r]);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < M) {
          float xf[VE];
          unpack(*reinterpret_cast<const uint4*>(x + size_t(m) * ldx + size_t(k) * VE), xf);
#pragma unroll
          for (int r = 0; r < NR; ++r)
#pragma unroll
            for (int e = 0; e < VE; ++e) acc[m][r] = fmaf(wf[r][e], xf[e], acc[m][r]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int r = 0; r < NR; ++r) acc[m][r] = warp_sum(acc[m][r]);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m < M && c.lane == m) {
        if (kp == 1) {
          ep(m, j, acc[m]);
        } else {
#pragma unroll
          for (int r = 0; r < NR; ++r) kred[((j * kp + q) * kMkMaxM + m) * NR + r] = acc[m][r];
        }
      }
    }
  }
  if (kp > 1) {
    cons_sync();
    for (int i = c.tid; i < n * M; i += kMkConsThreads) {
      const int j = i / M, m = i - j * M;
      float v[NR];
#pragma unroll
      for (int r = 0; r < NR; ++r) v[r] = 0.f;
      for (int q = 0; q < kp; ++q)
#pragma unroll
        for (int r = 0; r < NR; ++r) v[r] += kred[((j * kp + q) * kMkMaxM + m) * NR + r];
      ep(m, j, v);
    }
    cons_sync();
  }
}

// ---------------------------------------------------------------------------
// attention items: (row m, query head h, split sp) by one warp
// ---------------------------------------------------------------------------
struct MkItem {
  int m, h, kvh, p0, p1;
};

__device__ __forceinline__ MkItem mk_item(const MkParams& p, int it, int nsp, int pos) {
  MkItem r;
  const int per_m = p.hq * nsp;
  r.m = it / per_m;
  const int rem = it - r.m * per_m;
  r.h = rem / nsp;
  const int sp = rem - r.h * nsp;
  r.kvh = r.h / (p.hq / p.hkv);
  r.p0 = sp * kMkSplit;
  r.p1 = min(r.p0 + kMkSplit, pos + 1);
  return r;
}

// Stage the cached K/V rows [p0, min(p1, pos)) of an item into shared memory
// (one lane). Completes on `bar` (zero bytes: the phase completes at once).
template <typename T>
__device__ __forceinline__ void mk_stage_kv(const MkParams& p, const MkLayer& ly, const MkItem& t, int pos, T* ks,
                                            T* vs, uint64_t* bar) {
  const int pc = min(t.p1, pos);
  const uint32_t bytes = pc > t.p0 ? uint32_t(pc - t.p0) * p.hd * sizeof(T) : 0u;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  mbar_arrive_expect_tx(bar, 2 * bytes);
  if (bytes) {
    const size_t off = ((size_t(t.m) * p.hkv + t.kvh) * p.kv_cap + t.p0) * p.hd;
    bulk_g2s(ks, static_cast<const T*>(ly.k_cache) + off, bytes, bar);
    bulk_g2s(vs, static_cast<const T*>(ly.v_cache) + off, bytes, bar);
  }
}

// One item. qs: 3 * hd floats of this warp. ks/vs: staged K/V rows of the
// item (position p0 first), or NULL to read the cache in global memory.
template <typename T>
__device__ __forceinline__ bool mk_att_item(const MkCtx& c, const MkParams& p, const MkLayer& ly, int it,
                                            const MkItem& t, int pos, float* qs, const T* ks, const T* vs,
                                            uint64_t* bar, uint32_t bar_par, uint32_t seq_in, uint32_t seq_out,
                                            bool tr) {
  constexpr int P = LLPack<T>::kPer;
  constexpr int VE = VecTraits<T>::kElems;
  const int hd = p.hd, half = hd >> 1, wph = hd / P;
  const int nq = (p.hq + 2 * p.hkv) * hd;
  const bool has_new = pos >= t.p0 && pos < t.p1;
  const uint64_t* row = p.qkv_ll + size_t(t.m) * (nq / P);
  const uint64_t* qw = row + size_t(t.h) * wph;
  const uint64_t* kw = row + size_t(p.hq + t.kvh) * wph;
  const uint64_t* vw = row + size_t(p.hq + p.hkv + t.kvh) * wph;
  float* q = qs;
  float* kn = qs + hd;
  float* vn = qs + 2 * hd;
  // q (and the new k, v) of this head: all loads first, then the spins
  bool ok = true;
  for (int w = c.lane; w < wph; w += 32) {
    uint2 a = ll_ld(qw + w), b = make_uint2(0, seq_in), d = make_uint2(0, seq_in);
    if (has_new) {
      b = ll_ld(kw + w);
      d = ll_ld(vw + w);
    }
    if (a.y != seq_in && !ll_spin(p, qw + w, seq_in, a, c.abort)) ok = false;
    if (ok && b.y != seq_in && !ll_spin(p, kw + w, seq_in, b, c.abort)) ok = false;
    if (ok && d.y != seq_in && !ll_spin(p, vw + w, seq_in, d, c.abort)) ok = false;
    if (!ok) break;
    LLPack<T>::unpack(a.x, q + w * P);
    if (has_new) {
      LLPack<T>::unpack(b.x, kn + w * P);
      LLPack<T>::unpack(d.x, vn + w * P);
    }
  }
  if (!__all_sync(0xffffffffu, ok)) return false;
  __syncwarp();
  if (tr) p.trace[1000] = global_ns();
  // RoPE (reference rotate_half form, fp32 with T-rounded result), in place
  const float* cs = p.cos_tab + size_t(pos) * hd;
  const float* sn = p.sin_tab + size_t(pos) * hd;
  for (int i = c.lane; i < half; i += 32) {
    const float qa = q[i], qb = q[i + half];
    q[i] = round_t<T>(__fadd_rn(__fmul_rn(qa, cs[i]), __fmul_rn(-qb, sn[i])));
    q[i + half] = round_t<T>(__fadd_rn(__fmul_rn(qb, cs[i + half]), __fmul_rn(qa, sn[i + half])));
    if (has_new) {
      const float ka = kn[i], kb = kn[i + half];
      kn[i] = round_t<T>(__fadd_rn(__fmul_rn(ka, cs[i]), __fmul_rn(-kb, sn[i])));
      kn[i + half] = round_t<T>(__fadd_rn(__fmul_rn(kb, cs[i + half]), __fmul_rn(ka, sn[i + half])));
    }
  }
  __syncwarp();
  const size_t cbase = (size_t(t.m) * p.hkv + t.kvh) * p.kv_cap * hd;
  T* kc = static_cast<T*>(ly.k_cache) + cbase;
  T* vc = static_cast<T*>(ly.v_cache) + cbase;
  // the first query head of the KV head stores the new K/V for later steps
  if (has_new && t.h % (p.hq / p.hkv) == 0) {
    for (int d = c.lane; d < hd; d += 32) {
      kc[size_t(pos) * hd + d] = from_f<T>(kn[d]);
      vc[size_t(pos) * hd + d] = from_f<T>(vn[d]);
    }
  }
  if (bar && !__all_sync(0xffffffffu, mbar_wait(bar, bar_par, p.budget_ns, c.abort))) return false;
  const T* kb = ks ? ks : kc + size_t(t.p0) * hd;
  const T* vb = vs ? vs : vc + size_t(t.p0) * hd;
  if (tr) p.trace[1001] = global_ns();
  // scores: lane j takes position p0 + j; 16-byte chunks visited in a
  // lane-rotated order so the lanes of a quarter warp hit distinct banks
  const int NV = hd / VE;
  const int j = c.lane, pp = t.p0 + j;
  float s = -INFINITY;
  if (pp < t.p1) {
    float d = 0.f;
    if (pp == pos) {
      for (int e = 0; e < hd; ++e) d = fmaf(q[e], kn[e], d);
    } else {
      const T* kr = kb + size_t(j) * hd;
      for (int v0 = 0; v0 < NV; v0 += 4) {
        uint4 kv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (v0 + u < NV) kv[u] = ld_vec(kr + ((v0 + u + j) & (NV - 1)) * VE);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (v0 + u < NV) {
            const float* qv = q + ((v0 + u + j) & (NV - 1)) * VE;
            float kf[VE];
            unpack(kv[u], kf);
#pragma unroll
            for (int e = 0; e < VE; ++e) d = fmaf(qv[e], kf[e], d);
          }
        }
      }
    }
    s = d * p.scale;
  }
  float mx = s;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float pl = pp < t.p1 ? expf(s - mx) : 0.f;
  const float l = warp_sum(pl);
  if (tr) p.trace[1002] = global_ns();
  // PV: lane owns dims lane, lane + 32, ...
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  const int nt = t.p1 - t.p0;
#pragma unroll 4
  for (int jj = 0; jj < nt; ++jj) {
    const float pj = __shfl_sync(0xffffffffu, pl, jj);
    const bool isnew = t.p0 + jj == pos;
    const T* vr = vb + size_t(jj) * hd;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = c.lane + 32 * i;
      if (d < hd) o[i] = fmaf(pj, isnew ? vn[d] : to_f(vr[d]), o[i]);
    }
  }
  uint64_t* dst = p.att_ll + size_t(it) * (hd + 2);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = c.lane + 32 * i;
    if (d < hd) ll_put(dst + d, __float_as_uint(o[i]), seq_out);
  }
  if (c.lane == 0) ll_put2(dst + hd, __float_as_uint(mx), __float_as_uint(l), seq_out);
  if (tr) p.trace[1003] = global_ns();
  return true;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <typename T, int MT>
__global__ void __launch_bounds__(kMkThreads, 1) decode_mk_kernel(const MkParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float red[32];
  __shared__ float kred[kMkCons * kMkMaxM * 4];
  __shared__ long long bests[kMkCons][kMkMaxM];
  __shared__ long long cta_best[kMkMaxM];
  constexpr int P = LLPack<T>::kPer;
  const size_t tsz = sizeof(T);
  const MkLayout lay = mk_layout(p, tsz);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMkMaxSlots;
  uint64_t* sbar = empty + kMkMaxSlots;  // [kMkMaxStage] attention staging
  volatile int* abort = reinterpret_cast<volatile int*>(sbar + kMkMaxStage);
  int* never = const_cast<int*>(abort) + 1;  // stays 0: "no abort" for the final drains
  MkLayer* lys = reinterpret_cast<MkLayer*>(smem + lay.lys);
  T* xres = reinterpret_cast<T*>(smem + lay.xres);
  T* xnorm = reinterpret_cast<T*>(smem + lay.xnorm);
  T* xin = reinterpret_cast<T*>(smem + lay.xin);
  float* wsc = reinterpret_cast<float*>(smem + lay.wsc);
  T* stg = reinterpret_cast<T*>(smem + lay.stg);
  char* ring = reinterpret_cast<char*>(smem + lay.ring);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // step and position of this decode step
  const uint32_t step = ld_volatile_u32(p.comm.ctl() + kCtlStep) + 1u;
  const int pos = *reinterpret_cast<volatile int*>(p.pos_ptr);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nslot; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, kMkCons);
    }
    for (int s = 0; s < p.att_stage; ++s) mbar_init(sbar + s, 1);
    *never = 0;
    *abort = 0;
    if (pos < 0 || pos >= p.kv_cap || pos >= p.rope_len) {
      *abort = 1;
      atomicOr(p.comm.status(), kStatusBadPosition);
    }
    mbar_init_fence();
  }
  {
    const uint64_t* src = reinterpret_cast<const uint64_t*>(p.layers);
    uint64_t* dst = reinterpret_cast<uint64_t*>(lys);
    for (int i = threadIdx.x; i < p.L * int(sizeof(MkLayer) / 8); i += blockDim.x) dst[i] = src[i];
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
      bool stop = *abort != 0;
      const uint64_t pol = l2_evict_first_policy();
      for (int s = 0; s < nstages && !stop; ++s) {
        const MkStage st = mk_stage<T>(p, lys, s);
        int u0, nu;
        mk_part(st.units, u0, nu);
        const int upc = mk_upc(p, st, tsz);
        const size_t rb = size_t(st.K) * tsz, ub = size_t(st.rpu) * rb;
        for (int c = 0; c < nu; c += upc, ++k) {
          const int n = min(upc, nu - c);
          const int slot = k % p.nslot;
          if (k >= p.nslot && !mbar_wait(empty + slot, ((k / p.nslot) - 1) & 1, p.budget_ns, abort)) {
            *abort = 1;
            atomicOr(p.comm.status(), kStatusTimeout);
            stop = true;
            break;
          }
          // at most `inflight` copies outstanding
          if (p.inflight > 0 && k >= p.inflight) {
            const int kk = k - p.inflight;
            mbar_wait(full + (kk % p.nslot), (kk / p.nslot) & 1, p.budget_ns, abort);
          }
          if (*abort) {
            stop = true;
            break;
          }
          char* dst = ring + size_t(slot) * p.slot_bytes;
          const uint32_t hb = uint32_t(n * ub);
          if (c == 0 && p.trace && blockIdx.x == 0) p.trace[512 + s] = global_ns();
          if (p.trace && blockIdx.x == 0 && s >= 4 && s < 8 && c / upc < 20) p.trace[1300 + (s - 4) * 20 + c / upc] = global_ns();
          mbar_arrive_expect_tx(full + slot, hb * st.halves);
          for (int h = 0; h < st.halves; ++h) {
            const char* src = st.w + (size_t(h) * st.hoff + size_t(u0 + c) * st.rpu) * rb;
            if (p.l2_hint)
              bulk_g2s_hint(dst + size_t(h) * hb, src, hb, full + slot, pol);
            else
              bulk_g2s(dst + size_t(h) * hb, src, hb, full + slot);
          }
        }
      }
      // drain: the copies in flight must land before the CTA exits
      const int issued = k;
      for (int i = max(0, issued - p.nslot); i < issued; ++i)
        mbar_wait(full + (i % p.nslot), (i / p.nslot) & 1, p.budget_ns, never);
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

    // consume every chunk of weight stage s; x: [M][ldx] in shared memory
    auto run_stage = [&](int s, const T* x, int ldx, auto nr_tag, auto rpu_tag, auto ep) {
      constexpr int NR = decltype(nr_tag)::value;
      constexpr int RPU = decltype(rpu_tag)::value;
      const MkStage st = mk_stage<T>(p, lys, s);
      int u0, nu;
      mk_part(st.units, u0, nu);
      const int upc = mk_upc(p, st, tsz);
      for (int cc = 0; cc < nu; cc += upc, ++k) {
        const int n = min(upc, nu - cc);
        const int slot = k % p.nslot;
        const char* sl = ring + size_t(slot) * p.slot_bytes;
        if (!mbar_wait(full + slot, (k / p.nslot) & 1, p.budget_ns, abort)) {
          if (!*abort) mk_fail(c, p);
        }
        const bool trc = p.trace && blockIdx.x == 0 && c.tid == 0 && s >= 4 && s < 8 && cc / upc < 20;
        if (trc) p.trace[1100 + (s - 4) * 40 + 2 * (cc / upc)] = global_ns();
        // every consumer runs the chunk (it may synchronise the consumers);
        // after an abort the outputs are dropped
        auto epu = [&](int m, int j, const float* v) {
          if (!*abort) ep(m, u0 + cc + j, v);
        };
        cons_gemv_chunk<T, MT, NR, RPU>(c, sl, n, st.K, x, ldx, p.M, kred, epu);
        if (trc) p.trace[1101 + (s - 4) * 40 + 2 * (cc / upc)] = global_ns();
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot);
      }
    };
    using I1 = std::integral_constant<int, 1>;
    using IP = std::integral_constant<int, P>;
    using I2P = std::integral_constant<int, 2 * P>;

    // attention items of this CTA: it = blockIdx.x + G * li, warp li % kMkCons;
    // the first att_stage local items have their K/V staged in shared memory
    const int nsp = min(p.nsplit, (pos + kMkSplit) / kMkSplit);
    const int n_items = p.M * p.hq * nsp;
    const int n_loc = blockIdx.x < n_items ? (n_items - 1 - int(blockIdx.x)) / G + 1 : 0;
    const size_t stg_elems = mk_stage_bytes(p, tsz) / tsz;
    float* qs = wsc + size_t(c.cw) * 3 * p.hd;
    auto stage_layer = [&](int l) {
      if (lane == 0) {
        for (int li = c.cw; li < min(n_loc, p.att_stage); li += kMkCons) {
          const int it = blockIdx.x + G * li;
          T* ks = stg + size_t(li) * stg_elems;
          mk_stage_kv<T>(p, lys[l], mk_item(p, it, nsp, pos), pos, ks, ks + stg_elems / 2, sbar + li);
        }
      }
    };
    int staged_layer = -1;  // last layer whose K/V copies this warp issued
    if (!*abort) {
      stage_layer(0);
      staged_layer = 0;
    }

    MK_TRACE(c, p, 0);
    bool alive = !cons_sync_or(*abort != 0);
    // ---- embedding -> site 0 (this CTA's word slice of every row)
    if (alive) {
      const int W = p.H / P;
      int w0, nw;
      mk_part(W, w0, nw);
      const uint32_t seq = site_seq(0);
      for (int i = c.tid; i < p.M * nw; i += kMkConsThreads) {
        const int m = i / nw, w = w0 + (i - m * nw);
        const long long id = p.tok[m];
        if ((id < 0 || id >= p.vocab) && w == w0) atomicOr(cm.status(), kStatusBadToken);
        const bool mine = id >= p.vstart && id < p.vend;
        float f[P];
#pragma unroll
        for (int e = 0; e < P; ++e)
          f[e] = mine ? to_f(static_cast<const T*>(p.embed)[size_t(id - p.vstart) * p.H + size_t(w) * P + e]) : 0.f;
        const uint32_t u = LLPack<T>::pack(f);
        for (int d = 0; d < cm.world; ++d) ll_put(mk_site(p, d, 0, cm.rank) + size_t(m) * W + w, u, seq);
      }
    }
    const int nq = (p.hq + 2 * p.hkv) * p.hd;
    const int WH = p.H / P;

    for (int l = 0; l < p.L && alive; ++l) {
      const MkLayer& ly = lys[l];
      const int tb = 1 + 12 * l;
      MK_TRACE(c, p, tb + 0);
      // ---- QKV
      alive = cons_reduce_norm<T>(c, p, 2 * l, site_seq(2 * l), l > 0, static_cast<const T*>(ly.ln1), xres, xnorm);
      if (!alive) break;
      MK_TRACE(c, p, tb + 1);
      {
        const T* bias = static_cast<const T*>(ly.qkv_b);
        uint64_t* out = p.qkv_ll;
        const uint32_t seq = loc_seq(3 * l);
        run_stage(4 * l, xnorm, p.H, IP{}, IP{}, [&](int m, int u, const float* v) {
          float r[P];
#pragma unroll
          for (int e = 0; e < P; ++e) r[e] = bias ? v[e] + to_f(bias[u * P + e]) : v[e];
          ll_put(out + size_t(m) * (nq / P) + u, LLPack<T>::pack(r), seq);
        });
      }
      MK_TRACE(c, p, tb + 2);
      // ---- attention items
      {
        bool ok = true;
        for (int li = c.cw; li < n_loc && ok; li += kMkCons) {
          const int it = blockIdx.x + G * li;
          const bool st = li < p.att_stage;
          const T* ks = st ? stg + size_t(li) * stg_elems : nullptr;
          ok = mk_att_item<T>(c, p, ly, it, mk_item(p, it, nsp, pos), pos, qs, ks, st ? ks + stg_elems / 2 : nullptr,
                              st ? sbar + li : nullptr, uint32_t(l & 1), loc_seq(3 * l), loc_seq(3 * l + 1),
                              p.trace && blockIdx.x == 0 && li == 0);
          __syncwarp();
        }
        if (!ok && lane == 0 && !*abort) mk_fail(c, p);
        // this warp's staged rows are consumed: fetch the next layer's
        if (ok && l + 1 < p.L) {
          __syncwarp();
          stage_layer(l + 1);
          staged_layer = l + 1;
        }
        MK_TRACE(c, p, tb + 4);
      }
      // ---- O: merge the splits of every (row, head) into xin
      {
        const int hd = p.hd, pairs = p.M * p.hq, npart = pairs * nsp;
        const uint32_t seq = loc_seq(3 * l + 1);
        // after the per-warp attention scratch: a warp of this CTA may still be
        // in its item while other threads already collect the partials
        float* msc = wsc + size_t(kMkCons) * 3 * hd;  // [pairs][nsp]: split max, then merge weight
        float* lsc = msc + npart;                      // [pairs][nsp]: split sum
        bool ok = !*abort;
        for (int i = c.tid; i < npart && ok; i += kMkConsThreads) {
          const uint64_t* a = p.att_ll + size_t(i) * (hd + 2) + hd;
          uint4 v = ll_ld2(a);
          if (!ll_ok2(v, seq) && !ll_spin2(p, a, seq, v, abort)) ok = false;
          msc[i] = __uint_as_float(v.x);
          lsc[i] = __uint_as_float(v.z);
        }
        if (!ok && !*abort) mk_fail(c, p);
        if (cons_sync_or(!ok || *abort)) {
          alive = false;
          break;
        }
        MK_TRACE(c, p, tb + 5);
        // weights w_s = exp(m_s - max) / sum_s exp(m_s - max) l_s
        for (int pr = c.tid; pr < pairs; pr += kMkConsThreads) {
          float* ms = msc + size_t(pr) * nsp;
          const float* ls = lsc + size_t(pr) * nsp;
          float mx = -INFINITY;
          for (int s = 0; s < nsp; ++s) mx = fmaxf(mx, ms[s]);
          float den = 0.f;
          for (int s = 0; s < nsp; ++s) {
            const float w = ms[s] == -INFINITY ? 0.f : expf(ms[s] - mx);
            ms[s] = w;
            den = fmaf(w, ls[s], den);
          }
          const float inv = 1.0f / den;
          for (int s = 0; s < nsp; ++s) ms[s] *= inv;
        }
        cons_sync();
        const int hd2 = hd / 2;
        for (int i = c.tid; i < pairs * hd2 && ok; i += kMkConsThreads) {
          const int pr = i / hd2, d = 2 * (i - pr * hd2);
          const uint64_t* base = p.att_ll + size_t(pr) * nsp * (hd + 2) + d;
          const float* w = msc + size_t(pr) * nsp;
          float a0 = 0.f, a1 = 0.f;
          for (int s0 = 0; s0 < nsp && ok; s0 += 4) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (s0 + u < nsp) v[u] = ll_ld2(base + size_t(s0 + u) * (hd + 2));
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              if (s0 + u < nsp && ok) {
                if (!ll_ok2(v[u], seq) &&
                    !ll_spin2(p, base + size_t(s0 + u) * (hd + 2), seq, v[u], abort))
                  ok = false;
                a0 = fmaf(w[s0 + u], __uint_as_float(v[u].x), a0);
                a1 = fmaf(w[s0 + u], __uint_as_float(v[u].z), a1);
              }
            }
          }
          const int m = pr / p.hq, col = (pr - m * p.hq) * hd + d;
          xin[size_t(m) * p.xin_cols + col] = from_f<T>(a0);
          xin[size_t(m) * p.xin_cols + col + 1] = from_f<T>(a1);
        }
        if (!ok && !*abort) mk_fail(c, p);
        if (cons_sync_or(!ok || *abort)) {
          alive = false;
          break;
        }
        MK_TRACE(c, p, tb + 6);
        // o_proj -> site 2l+1 of every rank
        const uint32_t sseq = site_seq(2 * l + 1);
        run_stage(4 * l + 1, xin, p.xin_cols, IP{}, IP{}, [&](int m, int u, const float* v) {
          float r[P];
#pragma unroll
          for (int e = 0; e < P; ++e) r[e] = round_t<T>(v[e]);
          const uint32_t wd = LLPack<T>::pack(r);
          for (int d = 0; d < cm.world; ++d) ll_put(mk_site(p, d, 2 * l + 1, cm.rank) + size_t(m) * WH + u, wd, sseq);
        });
      }
      MK_TRACE(c, p, tb + 7);
      // ---- GU
      alive = cons_reduce_norm<T>(c, p, 2 * l + 1, site_seq(2 * l + 1), true, static_cast<const T*>(ly.ln2), xres,
                                  xnorm);
      if (!alive) break;
      MK_TRACE(c, p, tb + 8);
      {
        uint64_t* act = p.act_ll;
        const uint32_t seq = loc_seq(3 * l + 2);
        run_stage(4 * l + 2, xnorm, p.H, I2P{}, IP{}, [&](int m, int u, const float* v) {
          float a[P];
#pragma unroll
          for (int e = 0; e < P; ++e) {
            const float gr = round_t<T>(v[e]), ur = round_t<T>(v[P + e]);
            a[e] = round_t<T>(gr / (1.0f + expf(-gr))) * ur;
          }
          ll_put(act + size_t(m) * (p.I / P) + u, LLPack<T>::pack(a), seq);
        });
      }
      MK_TRACE(c, p, tb + 9);
      // ---- DOWN
      alive = cons_gather<T>(c, p, p.act_ll, p.I / P, loc_seq(3 * l + 2), xin, p.xin_cols);
      if (!alive) break;
      MK_TRACE(c, p, tb + 10);
      {
        const uint32_t sseq = site_seq(2 * l + 2);
        run_stage(4 * l + 3, xin, p.xin_cols, IP{}, IP{}, [&](int m, int u, const float* v) {
          float r[P];
#pragma unroll
          for (int e = 0; e < P; ++e) r[e] = round_t<T>(v[e]);
          const uint32_t wd = LLPack<T>::pack(r);
          for (int d = 0; d < cm.world; ++d) ll_put(mk_site(p, d, 2 * l + 2, cm.rank) + size_t(m) * WH + u, wd, sseq);
        });
      }
      MK_TRACE(c, p, tb + 11);
    }

    // ---- final norm + LM head + packed argmax
    if (alive)
      alive = cons_reduce_norm<T>(c, p, 2 * p.L, site_seq(2 * p.L), true, static_cast<const T*>(p.final_norm), xres,
                                  xnorm);
    if (alive) {
      MK_TRACE(c, p, 1 + 12 * p.L);
      long long best[kMkMaxM];
#pragma unroll
      for (int m = 0; m < kMkMaxM; ++m) best[m] = kArgmaxEmpty;
      const bool nan_wins = cm.world == 1;
      const int vloc = int(p.vend - p.vstart);
      T* lg = static_cast<T*>(p.logits);
      run_stage(4 * p.L, xnorm, p.H, I1{}, I1{}, [&](int m, int u, const float* v) {
        const float x = round_t<T>(v[0]);
        if (lg) lg[size_t(m) * vloc + u] = from_f<T>(x);
        const long long pk = argmax_pack(x, uint32_t(p.vstart) + uint32_t(u), nan_wins);
#pragma unroll
        for (int mm = 0; mm < kMkMaxM; ++mm)
          if (mm == m) best[mm] = pk > best[mm] ? pk : best[mm];
      });
#pragma unroll
      for (int m = 0; m < kMkMaxM; ++m) {
        const long long b = warp_max_ll(best[m]);
        if (lane == 0) bests[c.cw][m] = b;
      }
      cons_sync();
      const uint32_t lseq = loc_seq(3 * p.L);
      if (c.tid < p.M) {
        long long b = kArgmaxEmpty;
        for (int w = 0; w < kMkCons; ++w) b = bests[w][c.tid] > b ? bests[w][c.tid] : b;
        const unsigned long long ub = static_cast<unsigned long long>(b);
        ll_put2(p.lm_ll + (size_t(blockIdx.x) * kMkMaxM + c.tid) * 2, uint32_t(ub), uint32_t(ub >> 32), lseq);
        cta_best[c.tid] = kArgmaxEmpty;
        if (c.tid == 0 && p.trace && blockIdx.x == 0) p.trace[2 + 12 * p.L] = global_ns();
      }
      // ---- CTA 0: best over CTAs, then over ranks; token write, advance
      if (blockIdx.x == 0) {
        cons_sync();
        bool ok = !*abort;
        for (int i = c.tid; i < G * p.M && ok; i += kMkConsThreads) {
          const int g = i / p.M, m = i - g * p.M;
          const uint64_t* a = p.lm_ll + (size_t(g) * kMkMaxM + m) * 2;
          uint4 v = ll_ld2(a);
          if (!ll_ok2(v, lseq) && !ll_spin2(p, a, lseq, v, abort)) {
            ok = false;
            break;
          }
          atomicMax(reinterpret_cast<long long*>(&cta_best[m]),
                    static_cast<long long>((static_cast<unsigned long long>(v.z) << 32) | v.x));
        }
        if (!ok && !*abort) mk_fail(c, p);
        alive = !cons_sync_or(!ok || *abort);
        if (alive) {
          const int site = 2 * p.L + 1;
          const uint32_t sseq = site_seq(site);
          if (c.tid < p.M) {
            const unsigned long long ub = static_cast<unsigned long long>(cta_best[c.tid]);
            for (int d = 0; d < cm.world; ++d)
              ll_put2(mk_site(p, d, site, cm.rank) + 2 * c.tid, uint32_t(ub), uint32_t(ub >> 32), sseq);
          }
          cons_sync();
          if (c.tid < p.M) cta_best[c.tid] = kArgmaxEmpty;
          cons_sync();
          ok = true;
          if (c.tid < cm.world * p.M) {
            const int r = c.tid / p.M, m = c.tid - r * p.M;
            const uint64_t* a = mk_site(p, cm.rank, site, r) + 2 * m;
            uint4 v = ll_ld2(a);
            if (!ll_ok2(v, sseq) && !ll_spin2(p, a, sseq, v, abort)) ok = false;
            if (ok)
              atomicMax(reinterpret_cast<long long*>(&cta_best[m]),
                        static_cast<long long>((static_cast<unsigned long long>(v.z) << 32) | v.x));
          }
          if (!ok && !*abort) mk_fail(c, p);
          alive = !cons_sync_or(!ok || *abort);
          if (alive && c.tid < p.M) {
            const long long tk = argmax_id(cta_best[c.tid]);
            p.tok[c.tid] = tk;
            if (p.out_ids) p.out_ids[size_t(c.tid) * p.ld_out + pos + 1] = tk;
          }
          cons_sync();
          if (alive && c.tid == 0) {
            *reinterpret_cast<volatile int*>(p.pos_ptr) = pos + 1;
            if (p.trace) p.trace[3 + 12 * p.L] = global_ns();
          }
        }
      }
    }
    // bulk copies into this warp's staging buffers must land before exit
    if (lane == 0 && staged_layer >= 0) {
      for (int li = c.cw; li < min(n_loc, p.att_stage); li += kMkCons)
        mbar_wait(sbar + li, uint32_t(staged_layer & 1), p.budget_ns, never);
    }
  }
  __syncthreads();
  // every launch advances the step counter (also one that gave up), so the
  // next launch's sequence numbers match no word written by this one
  if (blockIdx.x == 0 && threadIdx.x == 0) p.comm.ctl()[kCtlStep] = step;
}

}  // namespace mtpb
