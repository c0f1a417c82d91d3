// Persistent decode megakernel: one greedy decode step of the whole TP model
// in one cooperative launch (one CTA per SM).
//
// Warp 0 is a producer: one thread streams this CTA's slice of every weight
// matrix of the step (QKV, O, gate/up and down of every layer, then the LM
// head), in execution order, into a circular byte ring in shared memory with
// 1-D bulk copies (cp.async.bulk, no multicast) completing on mbarriers. Each
// chunk is contiguous in the ring; the RMSNorm gains and the QKV bias travel
// in front of the rows that follow them. Weights do not depend on
// activations, so the stream runs ahead by the whole ring, across stage and
// layer boundaries, while the consumers wait on data.
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
// and no flag is needed. Readers spin (bounded) on the words themselves.
// Sequence numbers grow with the step counter, which every launch advances,
// so no word of an earlier step or launch matches.
#pragma once

#include <type_traits>

#include "comm.cuh"
#include "ll.cuh"
#include "tma.cuh"

namespace mtpb {

constexpr int kMkThreads = 512;
constexpr int kMkCons = 15;  // consumer warps 1..15
constexpr int kMkConsThreads = kMkCons * 32;
constexpr int kMkRingSlots = 8;   // chunks in the ring at once (mbarrier pairs)
constexpr int kMkMaxM = 8;
constexpr int kMkSplit = 32;      // KV positions per attention item (one per lane)
constexpr int kMkMaxSplits = 64;  // the split merge holds two splits per lane
constexpr int kMkMaxStage = 16;   // attention items per CTA (all staged in shared memory)
constexpr int kMkChan = 2;        // communicator channel of the AllReduce sites
// LM-head rows a warp streams at once: a unit is rows {u, u + V/4, u + V/2,
// u + 3V/4} of the shard when its vocabulary divides by 4 (else one row)
constexpr int kMkLmRows = 4;
constexpr int kMkHdr = 1024;      // shared-memory header: mbarriers + control words
// Copies of the words that every CTA reads (merged attention output, act):
// CTA b reads copy b % kMkRep, so fewer CTAs poll any one line.
constexpr int kMkRep = 4;
constexpr int kMkMergeLoads = 4;  // split outputs a merge lane loads per round
constexpr int kMkBiasMax = 256;   // QKV bias values of one CTA's units

// GEMV stage kinds
enum : int { kMkQkv = 0, kMkO = 1, kMkGu = 2, kMkDown = 3, kMkLm = 4, kMkKinds = 5 };

// shared-memory loads by 32-bit shared address
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ float4 lds128f(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
template <typename T> __device__ __forceinline__ float lds_t(uint32_t a);
template <> __device__ __forceinline__ float lds_t<float>(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
template <> __device__ __forceinline__ float lds_t<bf16>(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return __uint_as_float(uint32_t(v) << 16);
}

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

// One GEMV stage kind, planned on the host. A unit is `rpu` consecutive rows
// of each of `halves` row blocks (gate/up: unit u also takes rows
// hoff + u * rpu ..), so a unit's outputs fill whole LL words. CTA b owns
// units [b * base + min(b, rem), +base + (b < rem)); a chunk holds up to `upc`
// units and, in front of the first chunk, `pre` bytes of vectors (gains, bias).
struct MkKind {
  int K;  // row length (elements)
  int rpu;
  int halves;
  int hoff;
  int base;
  int rem;
  int upc;
  int pre;
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
  uint64_t* head_ll;  // [kMkRep][M][hq * hd / kPer] merged attention output
  uint64_t* act_ll;   // [kMkRep][M][I / kPer]
  uint64_t* lm_ll;   // [CTA][kMkMaxM][2] packed argmax as two LL words
  MkKind kinds[kMkKinds];
  int nsplit;     // KV splits of the cache capacity (upper bound)
  int att_stage;  // attention items per CTA (all staged in shared memory)
  int ring_bytes;
  int l2_hint;    // stream weights with an L2 evict-first policy
  int l2_ahead;   // prefetch the next layer's weight rows into L2
  int xin_cols;
  int wsc_floats;  // kMkCons * 3 * hd: q, new k and new v of each warp's attention item
  uint64_t budget_ns;
  uint32_t spin_ns;  // back-off between polls of a word that is not there yet
  // Optional stage timeline (%globaltimer ns): CTA 0 at [idx], the last CTA at
  // [2048 + idx], every CTA's layer-1 events at [4096 + e * 1024 + cta];
  // [0] start, [1 + 12 l + e] stage event e of layer l, then the LM head and
  // selection events, [512 + s] CTA 0's first copy of stage s, [1000 ..]
  // phases of CTA 0's first attention item, [1100], [1101] CTA 0's SM clock
  // (clock64) at its start and end, [1102] the time at its end. NULL = off.
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
  size_t lys, xres, xnorm, xin, wsc, bias, stg, ring, total;
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
  l.bias = off;
  off = mk_align(off + size_t(kMkBiasMax) * sizeof(float));
  l.stg = off;
  off = mk_align(off + size_t(p.att_stage) * mk_stage_bytes(p, tsz));
  l.ring = off;
  off = mk_align(off + size_t(p.ring_bytes));
  l.total = off;
  return l;
}

__device__ __forceinline__ void mk_units(const MkKind& kd, int& u0, int& nu) {
  const int b = blockIdx.x;
  u0 = b * kd.base + min(b, kd.rem);
  nu = kd.base + (b < kd.rem ? 1 : 0);
}

// floor(kMkCons / n) for n = 0 .. 15
__constant__ int kMkDivCons[16] = {1, 15, 7, 5, 3, 3, 2, 2, 1, 1, 1, 1, 1, 1, 1, 1};

// ---------------------------------------------------------------------------
// consumer-side helpers (all kMkConsThreads consumer threads call them)
// ---------------------------------------------------------------------------
struct MkCtx {
  int tid;  // consumer thread index 0..479
  int cw;   // consumer warp 0..14
  int lane;
  float* red;
  float* kred;  // split-K partial sums of the GEMV chunks
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
#pragma unroll
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
      // the line of four ranks in flight together; summed in rank order
      float s[2 * P];
#pragma unroll
      for (int e = 0; e < 2 * P; ++e) s[e] = 0.f;
      for (int r0 = 0; r0 < cm.world; r0 += 4) {
        uint4 v[4];
        auto addr = [&](int r) { return mk_site(p, cm.rank, site, r0 + r) + size_t(m) * W + 2 * i; };
        if (!ll_wait2<4>(p.budget_ns, p.spin_ns, addr, min(4, cm.world - r0), seq, v, c.abort)) ok = false;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          if (r0 + r < cm.world) {
            float f[2 * P];
            LLPack<T>::unpack(v[r].x, f);
            LLPack<T>::unpack(v[r].z, f + P);
#pragma unroll
            for (int e = 0; e < 2 * P; ++e) s[e] += f[e];
          }
        }
      }
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
  constexpr int NB = 3;
  const int nl = n / 2, tot = p.M * nl;
  bool ok = !*c.abort;
  for (int b0 = c.tid; b0 < tot && ok; b0 += NB * kMkConsThreads) {
    uint4 v[NB];
    const int nb = min(NB, (tot - b0 + kMkConsThreads - 1) / kMkConsThreads);
    auto addr = [&](int b) {
      const int i = b0 + b * kMkConsThreads, m = i / nl, w = i - m * nl;
      return src + size_t(m) * n + 2 * w;
    };
    if (!ll_wait2<NB>(p.budget_ns, p.spin_ns, addr, nb, seq, v, c.abort)) ok = false;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const int i = b0 + b * kMkConsThreads;
      if (b < nb) {
        const int m = i / nl, w = i - m * nl;
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
// GEMV over one chunk: n units of NR rows (RPU rows of NR / RPU halves), the
// row blocks starting at shared address `rows`, row length K. x: [M] rows of
// `xstride` bytes at shared address `xs`. With fewer units than warps, K is
// split over warps and the partial sums are added in a fixed order.
// ep(m, unit, v[NR]).
// ---------------------------------------------------------------------------
template <typename T, int MT, int NR, int RPU, typename Ep>
__device__ __forceinline__ void cons_gemv_chunk(const MkCtx& c, const char* rows, int n, int K, const char* xs,
                                                int xstride, int M, float* kred, Ep ep) {
  constexpr int VE = VecTraits<T>::kElems;
  const int cpr = K / VE;
  const uint32_t rb = uint32_t(K) * sizeof(T);
  // plain loads through pointers into the shared-memory array: the compiler
  // sees their address space and schedules them freely
  auto ld16 = [](const char* a) { return *reinterpret_cast<const uint4*>(a); };
  // fewer units than warps: split K over the idle warps, at least one
  // 16-byte vector per lane each (short stages such as O and QKV then use
  // most warps instead of one warp per unit)
  const int kp = n >= kMkCons ? 1 : max(1, min(kMkDivCons[n], (cpr + 31) >> 5));
  const int nw = n * kp;
  for (int w = c.cw; w < nw; w += kMkCons) {
    int j = w, q = 0;
    if (kp > 1) {
      while (j >= n) {
        j -= n;
        ++q;
      }
    }
    const char* ra[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) ra[r] = rows + size_t((r / RPU) * n * RPU + j * RPU + (r % RPU)) * rb;
    float acc[MT][NR];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int r = 0; r < NR; ++r) acc[m][r] = 0.f;
    // UN vectors per row in flight, then a remainder loop
    constexpr int UN = NR >= 4 ? 2 : 4;
    const int step = kp * 32;
    int k = q * 32 + c.lane;
    for (; k + (UN - 1) * step < cpr; k += UN * step) {
      uint4 wv[UN][NR];
#pragma unroll
      for (int u = 0; u < UN; ++u)
#pragma unroll
        for (int r = 0; r < NR; ++r) wv[u][r] = ld16(ra[r] + size_t(k + u * step) * 16);
#pragma unroll
      for (int u = 0; u < UN; ++u) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < M) {
            float xf[VE];
            unpack(ld16(xs + size_t(m) * xstride + size_t(k + u * step) * 16), xf);
#pragma unroll
            for (int r = 0; r < NR; ++r) {
              float wf[VE];
              unpack(wv[u][r], wf);
#pragma unroll
              for (int e = 0; e < VE; ++e) acc[m][r] = fmaf(wf[e], xf[e], acc[m][r]);
            }
          }
        }
      }
    }
    for (; k < cpr; k += step) {
      uint4 wv[NR];
#pragma unroll
      for (int r = 0; r < NR; ++r) wv[r] = ld16(ra[r] + size_t(k) * 16);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < M) {
          float xf[VE];
          unpack(ld16(xs + size_t(m) * xstride + size_t(k) * 16), xf);
#pragma unroll
          for (int r = 0; r < NR; ++r) {
            float wf[VE];
            unpack(wv[r], wf);
#pragma unroll
            for (int e = 0; e < VE; ++e) acc[m][r] = fmaf(wf[e], xf[e], acc[m][r]);
          }
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
    if (c.tid < n) {
      const int j = c.tid;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < M) {
          float v[NR];
#pragma unroll
          for (int r = 0; r < NR; ++r) v[r] = 0.f;
          for (int q = 0; q < kp; ++q)
#pragma unroll
            for (int r = 0; r < NR; ++r) v[r] += kred[((j * kp + q) * kMkMaxM + m) * NR + r];
          ep(m, j, v);
        }
      }
    }
    cons_sync();
  }
}

// Epilogue of a layer's GEMV stage: what happens to the outputs of unit u.
struct MkEpi {
  int kind;           // kMkQkv, kMkO, kMkGu or kMkDown
  uint32_t seq;       // sequence number of the words it writes
  int site;           // AllReduce site (O, down)
  const float* bias;  // QKV bias of this CTA's units (shared memory) or null
  int bias_u0;        // first unit of that slice
};

// One chunk of a layer's GEMV stage with its epilogue (QKV, O and down share
// the NR = kPer code, gate/up has its own).
template <typename T, int MT, int NR, int RPU>
__device__ __forceinline__ void mk_stage_chunk(MkCtx c, const MkParams& p, MkEpi e, const char* rows, int n, int K,
                                            const char* xs, int xstride, int u_base) {
  constexpr int P = LLPack<T>::kPer;
  const Comm& cm = p.comm;
  auto ep = [&](int m, int j, const float* v) {
    if (*c.abort) return;
    const int u = u_base + j;
    float r[P];
    if (e.kind == kMkGu) {
#pragma unroll
      for (int k = 0; k < P; ++k) {
        const float gr = round_t<T>(v[k]), ur = round_t<T>(v[(P + k) % NR]);
        r[k] = round_t<T>(gr / (1.0f + expf(-gr))) * ur;
      }
      const uint32_t wd = LLPack<T>::pack(r);
      const size_t act_n = size_t(p.M) * (p.I / P);
#pragma unroll
      for (int q = 0; q < kMkRep; ++q) ll_put(p.act_ll + q * act_n + size_t(m) * (p.I / P) + u, wd, e.seq);
    } else if (e.kind == kMkQkv) {
#pragma unroll
      for (int k = 0; k < P; ++k) r[k] = e.bias ? v[k] + e.bias[(u - e.bias_u0) * P + k] : v[k];
      const int nq = (p.hq + 2 * p.hkv) * p.hd;
      ll_put(p.qkv_ll + size_t(m) * (nq / P) + u, LLPack<T>::pack(r), e.seq);
    } else {
#pragma unroll
      for (int k = 0; k < P; ++k) r[k] = round_t<T>(v[k]);
      const uint32_t wd = LLPack<T>::pack(r);
      const int WH = p.H / P;
      for (int d = 0; d < cm.world; ++d) ll_put(mk_site(p, d, e.site, cm.rank) + size_t(m) * WH + u, wd, e.seq);
    }
  };
  cons_gemv_chunk<T, MT, NR, RPU>(c, rows, n, K, xs, xstride, p.M, c.kred, ep);
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

// One item, head_dim HD. qs: 3 * HD floats of this warp. ks/vs: the item's
// staged K/V rows (position p0 first); the new position's row is filled in
// here. Loops have compile-time trip counts and no branches inside, so the
// shared-memory loads and shuffles of all positions are in flight together.
template <typename T, int HD>
__device__ __forceinline__ bool mk_att_item(const MkCtx& c, const MkParams& p, const MkLayer& ly, int it,
                                            const MkItem& t, int pos, float* qs, T* ks, T* vs, uint64_t* bar,
                                            uint32_t bar_par, uint32_t seq_in, uint32_t seq_out, bool tr) {
  constexpr int P = LLPack<T>::kPer;
  constexpr int VE = VecTraits<T>::kElems;
  constexpr int HALF = HD / 2, WPH = HD / P;     // LL words of one head
  constexpr int NV = HD / VE;                    // 16-byte chunks of one K row
  constexpr int ND = HD >= 32 ? HD / 32 : 1;     // PV dims per lane
  const int nq = (p.hq + 2 * p.hkv) * HD;
  const bool has_new = pos >= t.p0 && pos < t.p1;
  const uint64_t* row = p.qkv_ll + size_t(t.m) * (nq / P);
  const uint64_t* qw = row + size_t(t.h) * WPH;
  const uint64_t* kw = row + size_t(p.hq + t.kvh) * WPH;
  const uint64_t* vw = row + size_t(p.hq + p.hkv + t.kvh) * WPH;
  float* q = qs;
  float* kn = qs + HD;
  float* vn = qs + 2 * HD;
  // q (and the new k, v) of this head: all loads first, then the spins
  bool ok = true;
  for (int w = c.lane; w < WPH && ok; w += 32) {
    uint2 v[3];
    const uint64_t* src[3] = {qw + w, kw + w, vw + w};
    auto addr = [&](int b) { return src[b]; };
    if (!ll_wait1<3>(p.budget_ns, p.spin_ns, addr, has_new ? 3 : 1, seq_in, v, c.abort)) ok = false;
    LLPack<T>::unpack(v[0].x, q + w * P);
    if (has_new) {
      LLPack<T>::unpack(v[1].x, kn + w * P);
      LLPack<T>::unpack(v[2].x, vn + w * P);
    }
  }
  if (!__all_sync(0xffffffffu, ok)) return false;
  __syncwarp();
  if (tr) p.trace[1000] = global_ns();
  // RoPE (reference rotate_half form, fp32 with T-rounded result), in place
  const float* cs = p.cos_tab + size_t(pos) * HD;
  const float* sn = p.sin_tab + size_t(pos) * HD;
  for (int i = c.lane; i < HALF; i += 32) {
    const float qa = q[i], qb = q[i + HALF];
    q[i] = round_t<T>(__fadd_rn(__fmul_rn(qa, cs[i]), __fmul_rn(-qb, sn[i])));
    q[i + HALF] = round_t<T>(__fadd_rn(__fmul_rn(qb, cs[i + HALF]), __fmul_rn(qa, sn[i + HALF])));
    if (has_new) {
      const float ka = kn[i], kb = kn[i + HALF];
      kn[i] = round_t<T>(__fadd_rn(__fmul_rn(ka, cs[i]), __fmul_rn(-kb, sn[i])));
      kn[i + HALF] = round_t<T>(__fadd_rn(__fmul_rn(kb, cs[i + HALF]), __fmul_rn(ka, sn[i + HALF])));
    }
  }
  __syncwarp();
  if (has_new) {
    // the new token's row joins the staged rows; the first query head of the
    // KV head also stores it in the cache for later steps
    const int jn = pos - t.p0;
    const bool store = t.h % (p.hq / p.hkv) == 0;
    T* kc = static_cast<T*>(ly.k_cache) + ((size_t(t.m) * p.hkv + t.kvh) * p.kv_cap + pos) * HD;
    T* vc = static_cast<T*>(ly.v_cache) + ((size_t(t.m) * p.hkv + t.kvh) * p.kv_cap + pos) * HD;
    for (int d = c.lane; d < HD; d += 32) {
      const T kv = from_f<T>(kn[d]), vv = from_f<T>(vn[d]);
      ks[size_t(jn) * HD + d] = kv;
      vs[size_t(jn) * HD + d] = vv;
      if (store) {
        kc[d] = kv;
        vc[d] = vv;
      }
    }
  }
  if (!__all_sync(0xffffffffu, mbar_wait(bar, bar_par, p.budget_ns, c.abort))) return false;
  __syncwarp();
  if (tr) p.trace[1001] = global_ns();
  // scores: lane j takes position p0 + j (lanes past the split read row 0 and
  // are masked afterwards); 16-byte chunks visited in a lane-rotated order so
  // the lanes of a quarter warp hit distinct banks
  const int nt = t.p1 - t.p0;
  const int j = c.lane;
  const int jr = j < nt ? j : 0;
  const uint32_t ks_s = smem_u32(ks), vs_s = smem_u32(vs), q_s = smem_u32(q);
  float d4[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const uint32_t kr = ks_s + uint32_t(jr * HD) * sizeof(T);
    uint4 kv[NV];
#pragma unroll
    for (int u = 0; u < NV; ++u) kv[u] = lds128(kr + uint32_t((u + j) & (NV - 1)) * 16);
#pragma unroll
    for (int u = 0; u < NV; ++u) {
      const uint32_t qa = q_s + uint32_t(((u + j) & (NV - 1)) * VE) * 4;
      float qf[VE], kf[VE];
#pragma unroll
      for (int e = 0; e < VE; e += 4) {
        const float4 f = lds128f(qa + e * 4);
        qf[e] = f.x;
        qf[e + 1] = f.y;
        qf[e + 2] = f.z;
        qf[e + 3] = f.w;
      }
      unpack(kv[u], kf);
#pragma unroll
      for (int e = 0; e < VE; ++e) d4[e & 3] = fmaf(qf[e], kf[e], d4[e & 3]);
    }
  }
  const float s = j < nt ? ((d4[0] + d4[1]) + (d4[2] + d4[3])) * p.scale : -INFINITY;
  float mx = s;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float pl = j < nt ? expf(s - mx) : 0.f;
  const float l = warp_sum(pl);
  if (tr) p.trace[1002] = global_ns();
  // PV: lane owns dims lane + 32 i; positions past the split have weight 0
  // and read row 0, so the loop runs without branches
  float o[ND];
#pragma unroll
  for (int i = 0; i < ND; ++i) o[i] = 0.f;
  const int dl = HD >= 32 ? c.lane : (c.lane & (HD - 1));
#pragma unroll
  for (int jj = 0; jj < kMkSplit; ++jj) {
    const float pj = __shfl_sync(0xffffffffu, pl, jj);
    const uint32_t vr = vs_s + uint32_t((jj < nt ? jj : 0) * HD) * sizeof(T);
#pragma unroll
    for (int i = 0; i < ND; ++i) o[i] = fmaf(pj, lds_t<T>(vr + uint32_t(dl + 32 * i) * sizeof(T)), o[i]);
  }
  uint64_t* dst = p.att_ll + size_t(it) * (HD + 2);
  if (HD >= 32 || c.lane < HD) {
#pragma unroll
    for (int i = 0; i < ND; ++i) ll_put(dst + dl + 32 * i, __float_as_uint(o[i]), seq_out);
  }
  if (c.lane == 0) ll_put2(dst + HD, __float_as_uint(mx), __float_as_uint(l), seq_out);
  if (tr) p.trace[1003] = global_ns();
  return true;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <typename T, int MT, int HD>
__global__ void __launch_bounds__(kMkThreads, 1) decode_mk_kernel(const __grid_constant__ MkParams pk) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(16) MkParams p_s;
  __shared__ float red[32];
  __shared__ float kred[kMkCons * kMkMaxM * 4];
  __shared__ long long bests[kMkCons][kMkMaxM];
  __shared__ long long cta_best[kMkMaxM];
  __shared__ int ring_lo[kMkRingSlots], ring_hi[kMkRingSlots];  // ring range of a chunk in flight
  constexpr int P = LLPack<T>::kPer;
  for (int i = threadIdx.x; i < int(sizeof(MkParams) / 4); i += blockDim.x)
    reinterpret_cast<uint32_t*>(&p_s)[i] = reinterpret_cast<const uint32_t*>(&pk)[i];
  __syncthreads();
  const MkParams& p = p_s;
  const size_t tsz = sizeof(T);
  const MkLayout lay = mk_layout(p, tsz);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMkRingSlots;
  uint64_t* sbar = empty + kMkRingSlots;  // [kMkMaxStage] attention staging
  volatile int* abort = reinterpret_cast<volatile int*>(sbar + kMkMaxStage);
  int* never = const_cast<int*>(abort) + 1;  // stays 0: "no abort" for the final drains
  MkLayer* lys = reinterpret_cast<MkLayer*>(smem + lay.lys);
  T* xres = reinterpret_cast<T*>(smem + lay.xres);
  T* xnorm = reinterpret_cast<T*>(smem + lay.xnorm);
  T* xin = reinterpret_cast<T*>(smem + lay.xin);
  float* wsc = reinterpret_cast<float*>(smem + lay.wsc);
  float* qkv_bias_s = reinterpret_cast<float*>(smem + lay.bias);  // this CTA's QKV bias values
  T* stg = reinterpret_cast<T*>(smem + lay.stg);
  char* ring = reinterpret_cast<char*>(smem + lay.ring);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // step and position of this decode step
  const uint32_t step = ld_volatile_u32(p.comm.ctl() + kCtlStep) + 1u;
  const int pos = *reinterpret_cast<volatile int*>(p.pos_ptr);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMkRingSlots; ++s) {
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
  // local sequence numbers: 4l qkv, 4l+1 attention partials, 4l+2 merged
  // attention output, 4l+3 act; 4L the LM winners
  const uint32_t nloc = uint32_t(4 * p.L + 1);
  auto site_seq = [&](int site) { return step * nsite + uint32_t(site) + 1u; };
  auto loc_seq = [&](int k) { return step * nloc + uint32_t(k) + 1u; };
  const int H = p.H;
  const int nq = (p.hq + 2 * p.hkv) * p.hd;
  const uint32_t hvec = uint32_t(mk_align(size_t(H) * tsz));  // a gain vector in front of a chunk

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int k = 0, k_old = 0, head = 0;
      bool stop = *abort != 0;
      const uint64_t pol = l2_evict_first_policy();
      for (int s = 0; s < 4 * p.L + 1 && !stop; ++s) {
        const int kind = s == 4 * p.L ? int(kMkLm) : (s & 3);
        const MkKind& kd = p.kinds[kind];
        const MkLayer* ly = kind == kMkLm ? nullptr : lys + (s >> 2);
        const void* wv = kind == kMkQkv ? ly->qkv_w
                         : kind == kMkO ? ly->o_w
                         : kind == kMkGu ? ly->gu_w
                         : kind == kMkDown ? ly->down_w
                                           : p.lm_head;
        const char* w = static_cast<const char*>(wv);
        int u0, nu;
        mk_units(kd, u0, nu);
        const uint32_t rb = uint32_t(kd.K) * uint32_t(tsz), hb1 = uint32_t(kd.rpu) * rb;
        int pf_upto = 0;  // units of this stage already prefetched into L2 while the ring was full
        // a stage with vectors in front has at least one chunk, even without units
        for (int cc = 0; (cc < nu || (cc == 0 && kd.pre)) && !stop; cc += kd.upc) {
          const int n = max(0, min(kd.upc, nu - cc));
          const uint32_t pre = cc == 0 ? uint32_t(kd.pre) : 0u;
          const uint32_t B = pre + uint32_t(kd.halves * n) * hb1;
          const int at = head + int(B) <= p.ring_bytes ? head : 0;
          // room: fewer than kMkRingSlots chunks in flight, none overlapping [at, at + B)
          for (bool first = true;; first = false) {
            bool fit = k - k_old < kMkRingSlots;
            for (int i = k_old; i < k && fit; ++i)
              fit = at + int(B) <= ring_lo[i & (kMkRingSlots - 1)] || at >= ring_hi[i & (kMkRingSlots - 1)];
            if (fit) break;
            if (first) {
              // the ring is full: start this chunk's rows and the next chunk's on
              // their way into L2, so the copies are L2 hits once room frees
              const int u_end = min(nu, cc + 2 * kd.upc);
              if (pf_upto < u_end) {
                const int ub = max(pf_upto, cc);
                for (int h = 0; h < kd.halves; ++h)
                  bulk_prefetch_l2(w + (size_t(h) * kd.hoff + size_t(u0 + ub) * kd.rpu) * rb, uint32_t(u_end - ub) * hb1);
                pf_upto = u_end;
              }
            }
            if (!mbar_wait(empty + (k_old & (kMkRingSlots - 1)), uint32_t(k_old / kMkRingSlots) & 1u, p.budget_ns,
                           abort)) {
              *abort = 1;
              atomicOr(p.comm.status(), kStatusTimeout);
              stop = true;
              break;
            }
            ++k_old;
          }
          if (stop || *abort) {
            stop = true;
            break;
          }
          const int slot = k & (kMkRingSlots - 1);
          ring_lo[slot] = at;
          ring_hi[slot] = at + int(B);
          char* dst = ring + at;
          // exact transaction bytes: the vectors in front, then the rows
          uint32_t tx = uint32_t(kd.halves * n) * hb1;
          const void* v0 = nullptr;
          const void* v1 = nullptr;
          if (pre) {
            v0 = kind == kMkQkv ? ly->ln1 : kind == kMkGu ? ly->ln2 : p.final_norm;
            v1 = kind == kMkQkv ? ly->qkv_b : nullptr;
            tx += uint32_t(H) * uint32_t(tsz) + (v1 ? uint32_t(nq) * uint32_t(tsz) : 0u);
          }
          if (p.trace && blockIdx.x == 0 && cc == 0) p.trace[512 + s] = global_ns();
          mbar_arrive_expect_tx(full + slot, tx);
          if (v0) bulk_g2s(dst, v0, uint32_t(H) * uint32_t(tsz), full + slot);
          if (v1) bulk_g2s(dst + hvec, v1, uint32_t(nq) * uint32_t(tsz), full + slot);
          for (int h = 0; h < kd.halves; ++h) {
            const char* src = w + (size_t(h) * kd.hoff + size_t(u0 + cc) * kd.rpu) * rb;
            char* d = dst + pre + uint32_t(h * n) * hb1;
            if (p.l2_hint)
              bulk_g2s_hint(d, src, uint32_t(n) * hb1, full + slot, pol);
            else
              bulk_g2s(d, src, uint32_t(n) * hb1, full + slot);
            // the same rows of the next layer start moving into L2 now, so its
            // ring copies are L2 hits
            if (p.l2_ahead && n > 0 && s + 4 < 4 * p.L) {
              const MkLayer* ln = lys + (s >> 2) + 1;
              const void* wn = kind == kMkQkv ? ln->qkv_w
                               : kind == kMkO ? ln->o_w
                               : kind == kMkGu ? ln->gu_w
                                               : ln->down_w;
              bulk_prefetch_l2(static_cast<const char*>(wn) + (size_t(h) * kd.hoff + size_t(u0 + cc) * kd.rpu) * rb,
                               uint32_t(n) * hb1);
            }
          }
          head = at + int(B);
          ++k;
        }
      }
      // drain: the copies in flight must land before the CTA exits
      for (int i = max(0, k - kMkRingSlots); i < k; ++i)
        mbar_wait(full + (i & (kMkRingSlots - 1)), uint32_t(i / kMkRingSlots) & 1u, p.budget_ns, never);
    }
  } else {
    // ------------------------------------------------------------ consumers
    MkCtx c;
    c.tid = threadIdx.x - 32;
    c.cw = warp - 1;
    c.lane = lane;
    c.red = red;
    c.kred = kred;
    c.abort = abort;
    const Comm& cm = p.comm;
    const int G = gridDim.x;
    int kc = 0;  // chunk counter (matches the producer)

    // wait for the next chunk; its offset in the ring
    auto chunk_wait = [&]() -> uint32_t {
      const int slot = kc & (kMkRingSlots - 1);
      if (!mbar_wait(full + slot, uint32_t(kc / kMkRingSlots) & 1u, p.budget_ns, abort) && !*abort) mk_fail(c, p);
      return uint32_t(ring_lo[slot]);
    };
    auto chunk_release = [&]() {
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + (kc & (kMkRingSlots - 1)));
      ++kc;
    };
    // GEMV of every chunk of a stage kind; the first chunk may already be
    // waited for (first >= 0: its ring offset). x: [M][ldx] T in shared memory
    auto run_stage = [&](int kind, int first, const T* x, int ldx, MkEpi e) {
      const MkKind& kd = p.kinds[kind];
      int u0, nu;
      mk_units(kd, u0, nu);
      for (int cc = 0; cc < nu || (cc == 0 && kd.pre); cc += kd.upc) {
        const int n = max(0, min(kd.upc, nu - cc));
        const uint32_t off = (cc == 0 && first >= 0) ? uint32_t(first) : chunk_wait();
        const uint32_t pre = cc == 0 ? uint32_t(kd.pre) : 0u;
        const char* xr = reinterpret_cast<const char*>(x);
        if (kind == kMkGu)
          mk_stage_chunk<T, MT, 2 * P, P>(c, p, e, ring + off + pre, n, kd.K, xr, ldx * int(tsz), u0 + cc);
        else
          mk_stage_chunk<T, MT, P, P>(c, p, e, ring + off + pre, n, kd.K, xr, ldx * int(tsz), u0 + cc);
        chunk_release();
      }
    };
    auto run_kind = [&](int kind, int first, const T* x, int ldx, auto nr_tag, auto rpu_tag, auto ep) {
      constexpr int NR = decltype(nr_tag)::value;
      constexpr int RPU = decltype(rpu_tag)::value;
      const MkKind& kd = p.kinds[kind];
      int u0, nu;
      mk_units(kd, u0, nu);
      for (int cc = 0; cc < nu || (cc == 0 && kd.pre); cc += kd.upc) {
        const int n = max(0, min(kd.upc, nu - cc));
        const uint32_t off = (cc == 0 && first >= 0) ? uint32_t(first) : chunk_wait();
        const uint32_t pre = cc == 0 ? uint32_t(kd.pre) : 0u;
        // every consumer runs the chunk (it may synchronise the consumers);
        // after an abort the outputs are dropped
        auto epu = [&](int m, int j, const float* v) {
          if (!*abort) ep(m, u0 + cc + j, v);
        };
        cons_gemv_chunk<T, MT, NR, RPU>(c, ring + off + pre, n, kd.K, reinterpret_cast<const char*>(x),
                                        ldx * int(tsz), p.M, kred, epu);
        chunk_release();
      }
    };
    using I1 = std::integral_constant<int, 1>;
    using IP = std::integral_constant<int, P>;
    using I2P = std::integral_constant<int, 2 * P>;

    // attention items of this CTA: it = blockIdx.x + G * li, warp li % kMkCons,
    // K/V staged in shared memory slot li
    const int nsp = min(p.nsplit, (pos + kMkSplit) / kMkSplit);
    const int n_items = p.M * p.hq * nsp;
    const int n_loc = min(p.att_stage, int(blockIdx.x) < n_items ? (n_items - 1 - int(blockIdx.x)) / G + 1 : 0);
    const size_t stg_elems = mk_stage_bytes(p, tsz) / tsz;
    float* qs = wsc + size_t(c.cw) * 3 * p.hd;
    auto stage_layer = [&](int l) {
      if (lane == 0) {
        for (int li = c.cw; li < n_loc; li += kMkCons) {
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
    if (p.trace && blockIdx.x == 0 && c.tid == 0) p.trace[1100] = clock64();
    bool alive = !cons_sync_or(*abort != 0);
    // ---- embedding -> site 0 (this CTA's word slice of every row)
    const int WH = H / P;
    if (alive) {
      const int base = WH / G, rem = WH % G;
      const int w0 = blockIdx.x * base + min(int(blockIdx.x), rem), nw = base + (int(blockIdx.x) < rem ? 1 : 0);
      const uint32_t seq = site_seq(0);
      for (int i = c.tid; i < p.M * nw; i += kMkConsThreads) {
        const int m = i / nw, w = w0 + (i - m * nw);
        const long long id = p.tok[m];
        if ((id < 0 || id >= p.vocab) && w == w0) atomicOr(cm.status(), kStatusBadToken);
        const bool mine = id >= p.vstart && id < p.vend;
        float f[P];
#pragma unroll
        for (int e = 0; e < P; ++e)
          f[e] = mine ? to_f(static_cast<const T*>(p.embed)[size_t(id - p.vstart) * H + size_t(w) * P + e]) : 0.f;
        const uint32_t u = LLPack<T>::pack(f);
        for (int d = 0; d < cm.world; ++d) ll_put(mk_site(p, d, 0, cm.rank) + size_t(m) * WH + w, u, seq);
      }
    }

    // The layers as a sequence of phases; each kind of phase (reduce + norm,
    // GEMV stage, gather, attention, merge) appears once in the code and
    // serves every place of a layer that needs it, which keeps the code a
    // layer executes small. Phases k of layer l:
    //   0 reduce (site 2l) + ln1    1 QKV     2 attention   3 merge
    //   4 gather head outputs       5 O       6 reduce (site 2l+1) + ln2
    //   7 gate/up                   8 gather act             9 down
    uint32_t first_off = 0;   // ring offset of the chunk that carries the gain
    const float* qkv_bias = nullptr;
    int qkv_u0 = 0;
    for (int ph = 0; ph < 10 * p.L && alive; ++ph) {
      const int l = ph / 10, k = ph - 10 * l;
      const MkLayer& ly = lys[l];
      const int tb = 1 + 12 * l;
      if (k == 0 || k == 6) {
        if (k == 0) MK_TRACE(c, p, tb + 0);
        first_off = chunk_wait();
        if (k == 6) MK_TRACE(c, p, tb + 3);  // the gate/up chunk (with ln2) has landed
        const T* gain = reinterpret_cast<const T*>(ring + first_off);
        if (k == 0 && ly.qkv_b) {
          // this CTA's slice of the QKV bias leaves the ring now: the chunk
          // that carries it is released after the stage's first chunk, while
          // the epilogue of later chunks still needs it (the barrier that ends
          // the reduce below orders these stores before the QKV stage)
          const T* rb = reinterpret_cast<const T*>(ring + first_off + hvec);
          int nu;
          mk_units(p.kinds[kMkQkv], qkv_u0, nu);
          for (int i = c.tid; i < nu * P; i += kMkConsThreads) qkv_bias_s[i] = to_f(rb[size_t(qkv_u0) * P + i]);
          qkv_bias = qkv_bias_s;
        } else if (k == 0) {
          qkv_bias = nullptr;
        }
        const int site = 2 * l + (k == 6 ? 1 : 0);
        alive = cons_reduce_norm<T>(c, p, site, site_seq(site), k == 6 || l > 0, gain, xres, xnorm);
        MK_TRACE(c, p, tb + (k == 0 ? 1 : 8));
      } else if (k == 1 || k == 5 || k == 7 || k == 9) {
        const int kind = k == 1 ? int(kMkQkv) : k == 5 ? int(kMkO) : k == 7 ? int(kMkGu) : int(kMkDown);
        const bool from_norm = kind == kMkQkv || kind == kMkGu;
        MkEpi e;
        e.kind = kind;
        e.site = kind == kMkO ? 2 * l + 1 : 2 * l + 2;
        e.seq = kind == kMkQkv ? loc_seq(4 * l) : kind == kMkGu ? loc_seq(4 * l + 3) : site_seq(e.site);
        e.bias = kind == kMkQkv ? qkv_bias : nullptr;
        e.bias_u0 = qkv_u0;
        run_stage(kind, from_norm ? int(first_off) : -1, from_norm ? xnorm : xin, from_norm ? H : p.xin_cols, e);
        MK_TRACE(c, p, tb + (k == 1 ? 2 : k == 5 ? 7 : k == 7 ? 9 : 11));
      } else if (k == 4 || k == 8) {
        const size_t hn = size_t(p.M) * (p.hq * p.hd / P), an = size_t(p.M) * (p.I / P);
        const uint64_t* src = k == 4 ? p.head_ll + (blockIdx.x % kMkRep) * hn : p.act_ll + (blockIdx.x % kMkRep) * an;
        const int nw = k == 4 ? p.hq * p.hd / P : p.I / P;
        alive = cons_gather<T>(c, p, src, nw, loc_seq(4 * l + (k == 4 ? 2 : 3)), xin, p.xin_cols);
        MK_TRACE(c, p, tb + (k == 4 ? 6 : 10));
      } else if (k == 2) {
        {
          bool ok = true;
          for (int li = c.cw; li < n_loc && ok; li += kMkCons) {
            const int it = blockIdx.x + G * li;
            T* ks = stg + size_t(li) * stg_elems;
            const MkItem t = mk_item(p, it, nsp, pos);
            const bool tr = p.trace && blockIdx.x == 0 && li == 0;
            const uint32_t sp = uint32_t(l & 1), si = loc_seq(4 * l), so = loc_seq(4 * l + 1);
            T* vs = ks + stg_elems / 2;
            ok = mk_att_item<T, HD>(c, p, ly, it, t, pos, qs, ks, vs, sbar + li, sp, si, so, tr);
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
      } else {
      {
          // one warp per (row, head, block of 32 dim pairs): head dims above
          // 64 take several warps, each its own dims of every split
          const int hd = p.hd, hd2 = hd / 2, ndb = (hd2 + 31) / 32, items = p.M * p.hq * ndb;
          const uint32_t seq = loc_seq(4 * l + 1), hseq = loc_seq(4 * l + 2);
          const size_t head_n = size_t(p.M) * (p.hq * hd / P);
          bool ok = !*abort;
          for (int wi = blockIdx.x + G * c.cw; wi < items && ok; wi += G * kMkCons) {
            const int pr = wi / ndb, db = wi - pr * ndb;
            const uint64_t* part = p.att_ll + size_t(pr) * nsp * (hd + 2);
            uint4 a[2];
            a[0] = make_uint4(__float_as_uint(-INFINITY), seq, 0u, seq);
            a[1] = a[0];
            {
              const int na = lane + 32 < nsp ? 2 : lane < nsp ? 1 : 0;
              auto addr = [&](int b) { return part + size_t(lane + 32 * b) * (hd + 2) + hd; };
              if (!ll_wait2<2>(p.budget_ns, p.spin_ns, addr, na, seq, a, abort)) ok = false;
            }
            if (!__all_sync(0xffffffffu, ok)) {
              ok = false;
              break;
            }
            const uint4 a0 = a[0], a1 = a[1];
            const float m0 = __uint_as_float(a0.x), m1 = __uint_as_float(a1.x);
            float mx = fmaxf(m0, m1);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            float w0 = m0 == -INFINITY ? 0.f : expf(m0 - mx), w1 = m1 == -INFINITY ? 0.f : expf(m1 - mx);
            const float den = warp_sum(fmaf(w0, __uint_as_float(a0.z), w1 * __uint_as_float(a1.z)));
            const float inv = 1.0f / den;
            w0 *= inv;
            w1 *= inv;
            const int m = pr / p.hq, hh = pr - m * p.hq;
            // every lane runs every iteration (the shuffles need the whole warp);
            // lanes past the head's dim pairs load and store nothing
            {
              const int dp = db * 32 + lane;
              const bool act = dp < hd2;
              float o[2] = {0.f, 0.f};
              // every split's (max, sum) has arrived, so its outputs have too:
              // kMkMergeLoads loads per round
              for (int s0 = 0; s0 < nsp; s0 += kMkMergeLoads) {
                uint4 v[kMkMergeLoads];
                auto addr = [&](int u) { return part + size_t(s0 + u) * (hd + 2) + 2 * dp; };
                if (act && ok &&
                    !ll_wait2<kMkMergeLoads>(p.budget_ns, p.spin_ns, addr, min(kMkMergeLoads, nsp - s0), seq, v, abort))
                  ok = false;
#pragma unroll
                for (int u = 0; u < kMkMergeLoads; ++u) {
                  const int sidx = s0 + u;
                  if (sidx < nsp) {
                    const float ws = __shfl_sync(0xffffffffu, sidx < 32 ? w0 : w1, sidx & 31);
                    if (act) {
                      o[0] = fmaf(ws, __uint_as_float(v[u].x), o[0]);
                      o[1] = fmaf(ws, __uint_as_float(v[u].z), o[1]);
                    }
                  }
                }
              }
              if (act && !*abort) {
                // dims (2 dp, 2 dp + 1) of head hh: word (hh * hd + 2 dp) / P
                const size_t w = size_t(m) * (p.hq * hd / P) + (size_t(hh) * hd + 2 * dp) / P;
#pragma unroll
                for (int r = 0; r < kMkRep; ++r) {
                  uint64_t* dst = p.head_ll + r * head_n + w;
                  if constexpr (P == 2) {
                    ll_put(dst, LLPack<T>::pack(o), hseq);
                  } else {
                    ll_put2(dst, __float_as_uint(o[0]), __float_as_uint(o[1]), hseq);
                  }
                }
              }
            }
          }
          if (!ok && !*abort) mk_fail(c, p);
          alive = !cons_sync_or(!ok || *abort);
        }
        MK_TRACE(c, p, tb + 5);
      }
    }

    // ---- final norm + LM head + packed argmax (the first LM chunk carries the gain)
    if (alive) {
      const uint32_t off = chunk_wait();
      const T* gain = reinterpret_cast<const T*>(ring + off);
      alive = cons_reduce_norm<T>(c, p, 2 * p.L, site_seq(2 * p.L), true, gain, xres, xnorm);
      MK_TRACE(c, p, 1 + 12 * p.L);
      long long best[kMkMaxM];
#pragma unroll
      for (int m = 0; m < kMkMaxM; ++m) best[m] = kArgmaxEmpty;
      const bool nan_wins = cm.world == 1;
      const int vloc = int(p.vend - p.vstart);
      T* lg = static_cast<T*>(p.logits);
      auto lm_row = [&](int m, int u, float v) {
        const float x = round_t<T>(v);
        if (lg) lg[size_t(m) * vloc + u] = from_f<T>(x);
        const long long pk = argmax_pack(x, uint32_t(p.vstart) + uint32_t(u), nan_wins);
#pragma unroll
        for (int mm = 0; mm < kMkMaxM; ++mm)
          if (mm == m) best[mm] = pk > best[mm] ? pk : best[mm];
      };
      if (p.kinds[kMkLm].halves == kMkLmRows) {
        const int q = p.kinds[kMkLm].hoff;
        run_kind(kMkLm, int(off), xnorm, H, std::integral_constant<int, kMkLmRows>{}, I1{},
                 [&](int m, int u, const float* v) {
#pragma unroll
                   for (int r = 0; r < kMkLmRows; ++r) lm_row(m, r * q + u, v[r]);
                 });
      } else {
        run_kind(kMkLm, int(off), xnorm, H, I1{}, I1{}, [&](int m, int u, const float* v) { lm_row(m, u, v[0]); });
      }
#pragma unroll
      for (int m = 0; m < kMkMaxM; ++m) {
        const long long b = warp_max_ll(best[m]);
        if (lane == 0) bests[c.cw][m] = b;
      }
      cons_sync();
      const uint32_t lseq = loc_seq(4 * p.L);
      if (alive && c.tid < p.M) {
        long long b = kArgmaxEmpty;
        for (int w = 0; w < kMkCons; ++w) b = bests[w][c.tid] > b ? bests[w][c.tid] : b;
        const unsigned long long ub = static_cast<unsigned long long>(b);
        ll_put2(p.lm_ll + (size_t(blockIdx.x) * kMkMaxM + c.tid) * 2, uint32_t(ub), uint32_t(ub >> 32), lseq);
        cta_best[c.tid] = kArgmaxEmpty;
        if (c.tid == 0 && p.trace && blockIdx.x == 0) p.trace[2 + 12 * p.L] = global_ns();
      }
      // ---- CTA 0: best over CTAs, then over ranks; token write, advance
      if (alive && blockIdx.x == 0) {
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
      for (int li = c.cw; li < n_loc; li += kMkCons)
        mbar_wait(sbar + li, uint32_t(staged_layer & 1), p.budget_ns, never);
    }
  }
  __syncthreads();
  if (p.trace && blockIdx.x == 0 && threadIdx.x == 32) {
    p.trace[1101] = clock64();
    p.trace[1102] = global_ns();
  }
  // every launch advances the step counter (also one that gave up), so the
  // next launch's sequence numbers match no word written by this one
  if (blockIdx.x == 0 && threadIdx.x == 0) p.comm.ctl()[kCtlStep] = step;
}

}  // namespace mtpb
