// Tensor-core GEMM for the bf16 projections of many rows (prefill chunks of
// >= 64 rows, kernel-chain decode steps of >= 8 rows): y = x · Wᵀ with the
// GEMV path's epilogues (store, SwiGLU, RoPE + KV append, AllReduce push).
//
// Persistent kernel, one CTA per SM, each CTA walking output tiles of
// 128 rows of x by BN (128 or 256) rows of W:
//   warp 0      TMA producer: 128 x 64 tiles of x and BN x 64 tiles of W into
//               a multi-stage shared-memory ring (2-D TMA, 128-byte swizzle,
//               no multicast);
//   warp 1      MMA issuer: tcgen05.mma (M 128, N BN, K 16, bf16 inputs, fp32
//               accumulation) into one of two tensor-memory accumulators;
//   warps 2-9   epilogue: tcgen05.ld of the finished accumulator, a transpose
//               through shared memory so that the lanes of a warp hold
//               consecutive output columns of one row (coalesced stores), then
//               the GEMV epilogue per element.
// The two accumulators let the epilogue of one tile run under the MMAs of the
// next. Every wait is bounded; on expiry the CTA records a status bit, lets
// its copies and MMAs land, frees its tensor memory and returns.
//
// Split K (single-CTA kernel, BN 128): when there are too few output tiles
// to occupy the SMs, each tile's K blocks are cut into `splits` consecutive
// ranges, one work item each. An item's epilogue writes its fp32 partial
// accumulator to a workspace, publishes it (fence + a per-tile arrival
// counter) and the CTA that completes the count sums the tile's partials in
// split order 0, 1, ... (the same order whichever CTA arrives last, so the
// result does not depend on timing) and runs the epilogue on the sum; it
// also returns the counter to zero for the next launch.
//
// Output units follow the GEMV epilogue: SwiGLU pairs gate row u with up row
// I + u, so its W tile is loaded as two BN/2-row halves (gate rows, then the
// matching up rows); RoPE pairs rows i and i + hd/2 of a head, which a tile of
// whole heads holds in columns c and c + hd/2.
#pragma once

#include <cuda.h>

#include "gemv.cuh"
#include "tma.cuh"

namespace mtpb {

constexpr int kTcBM = 128, kTcBK = 64;
constexpr int kTcEpiWarps = 8;
constexpr int kTcThreads = 64 + 32 * kTcEpiWarps;
constexpr int kTcXs = 33;                               // transpose row stride (floats): conflict-free
constexpr uint32_t kTcXposeBytes = 2 * 32 * kTcXs * 4;  // per epilogue warp: two 32 x 32 fp32 buffers
constexpr uint32_t kTcABytes = kTcBM * kTcBK * 2;       // one 128 x 64 bf16 tile: 16 KB

template <int BN>
struct TcCfg {
  static constexpr int kStages = BN == 256 ? 3 : 4;
  static constexpr uint32_t kBBytes = uint32_t(BN) * kTcBK * 2;
  static constexpr uint32_t kStageBytes = kTcABytes + kBBytes;
  static constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators
  static constexpr size_t kSmem = size_t(kStages) * kStageBytes + size_t(kTcEpiWarps) * kTcXposeBytes + 1024;
  // instruction descriptor: bf16 x bf16 -> fp32, both K-major, M 128, N BN
  static constexpr uint32_t kIdesc =
      (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(kTcBM >> 4) << 24);
};

struct TcParams {
  GemvParams g;  // shapes, inputs and epilogue fields (GEMV conventions)
  int tiles_m, tiles_n;
  int splits;    // K ranges per output tile (1: no split; > 1 only with BN 128)
  float* ws;     // split partials: [tile][split][BN / 4][128 rows][4] fp32
  int* cnt;      // per-tile arrival counters, zero between launches
  uint64_t budget_ns;
};

// Offset (floats) of accumulator column c (multiple of 4) of tile row r in
// one split partial: four consecutive columns of 128 rows are 2 KB, so the 32
// lanes (rows) of a warp store and load 512 consecutive bytes.
__device__ __forceinline__ size_t tc_ws_off(int c, int r) { return (size_t(c >> 2) * kTcBM + r) * 4; }

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor: K-major tile, 128-byte rows, 128-byte
// swizzle, 8-row groups 1024 bytes apart (tile base 1024-byte aligned).
__device__ __forceinline__ uint64_t tc_smem_desc(uint32_t addr) {
  return uint64_t((addr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's tensor-memory lane (no wait)
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Accumulator column of tile-local unit q (first of its pair) and of its
// partner (SwiGLU up row, RoPE second half of the head).
template <int EPI, int BN>
__device__ __forceinline__ int tc_col_a(int q, int hd) {
  if constexpr (EPI == kEpiRope) return (q / (hd >> 1)) * hd + q % (hd >> 1);
  return q;
}
template <int EPI, int BN>
__device__ __forceinline__ int tc_col_b(int q, int hd) {
  if constexpr (EPI == kEpiRope) return tc_col_a<EPI, BN>(q, hd) + (hd >> 1);
  return BN / 2 + q;
}

// Epilogue of one output unit (this lane's column) over `rows` rows of a
// tile: a[r * kTcXs] and b[r * kTcXs] hold row r's accumulator values (the
// unit's two operands for SwiGLU / RoPE). Store and SwiGLU keep the GEMV
// epilogue's arithmetic with the per-unit bias loaded once for all rows (so
// the row iterations are independent and interleave); the other epilogues
// call the GEMV epilogue per element.
template <typename T, int EPI>
__device__ __forceinline__ void tc_epi_rows(const GemvParams& p, int row0, int rows, int unit, const float* a,
                                            const float* b, uint32_t out_seq) {
  if constexpr (EPI == kEpiStore) {
    T* y = static_cast<T*>(p.y) + unit;
    if (p.bias) {
      const float bias = to_f(static_cast<const T*>(p.bias)[unit]);
#pragma unroll 4
      for (int r = 0; r < rows; ++r) y[size_t(out_row(p, row0 + r)) * p.ldy] = from_f<T>(a[r * kTcXs] + bias);
    } else {
#pragma unroll 4
      for (int r = 0; r < rows; ++r) y[size_t(out_row(p, row0 + r)) * p.ldy] = from_f<T>(a[r * kTcXs]);
    }
  } else if constexpr (EPI == kEpiSwiglu) {
    const int half = p.N >> 1;
    const bool has_bias = p.bias != nullptr;
    const float bg = has_bias ? to_f(static_cast<const T*>(p.bias)[unit]) : 0.f;
    const float bu = has_bias ? to_f(static_cast<const T*>(p.bias)[unit + half]) : 0.f;
    T* y = static_cast<T*>(p.y) + unit;
#pragma unroll 4
    for (int r = 0; r < rows; ++r) {
      float g = a[r * kTcXs], up = b[r * kTcXs];
      if (has_bias) {
        g += bg;
        up += bu;
      }
      g = round_t<T>(g);
      up = round_t<T>(up);
      y[size_t(row0 + r) * p.ldy] = from_f<T>(round_t<T>(silu_f(g)) * up);
    }
  } else {
#pragma unroll 2
    for (int r = 0; r < rows; ++r) gemv_epilogue<T, EPI>(p, row0 + r, unit, a[r * kTcXs], b[r * kTcXs], out_seq, nullptr);
  }
}

// One epilogue warp's share of a finished accumulator: tile-local units
// [part * U/2, (part + 1) * U/2) of rows row0 .. row0 + 31, where trow is the
// tensor-memory address of the warp's lane quarter in the accumulator, U the
// units per tile and u_tile the first unit of the tile.
// ld16(col, r) fetches 16 consecutive accumulator columns of this lane's row
// (tensor memory, or the sum of the split partials).
template <typename T, int EPI, int BN, typename Ld>
__device__ __forceinline__ void tc_epilogue_tile(const GemvParams& p, const Ld& ld16, int row0, int u_tile, int part,
                                                 float* bufa, float* bufb, int lane, uint32_t out_seq) {
  constexpr bool kPair = EPI == kEpiSwiglu || EPI == kEpiRope;
  constexpr int kUnitsPerTile = kPair ? BN / 2 : BN;
  const int hd = p.hd;
  const int bound = EPI == kEpiSwiglu ? (p.N >> 1) : EPI == kEpiRope ? (p.hq + 2 * p.hkv) * (hd >> 1) : p.N;
  for (int q0 = part * (kUnitsPerTile / 2); q0 < (part + 1) * (kUnitsPerTile / 2); q0 += 32) {
    uint32_t ra[32], rb[32];
    ld16(tc_col_a<EPI, BN>(q0, hd), ra);
    ld16(tc_col_a<EPI, BN>(q0 + 16, hd), ra + 16);
    if constexpr (kPair) {
      ld16(tc_col_b<EPI, BN>(q0, hd), rb);
      ld16(tc_col_b<EPI, BN>(q0 + 16, hd), rb + 16);
    }
    tc_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      bufa[lane * kTcXs + j] = __uint_as_float(ra[j]);
      if constexpr (kPair) bufb[lane * kTcXs + j] = __uint_as_float(rb[j]);
    }
    __syncwarp();
    const int unit = u_tile + q0 + lane;
    const int rows = min(32, p.M - row0);
    if (unit < bound && rows > 0) tc_epi_rows<T, EPI>(p, row0, rows, unit, bufa + lane, bufb + lane, out_seq);
    __syncwarp();
  }
}

template <typename T, int EPI, int BN>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const TcParams tp, const __grid_constant__ CUtensorMap map_x,
                   const __grid_constant__ CUtensorMap map_w) {
  using C = TcCfg<BN>;
  constexpr int S = C::kStages;
  constexpr bool kPair = EPI == kEpiSwiglu || EPI == kEpiRope;
  constexpr int kUnitsPerTile = kPair ? BN / 2 : BN;
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t full[S], empty[S], acc_full[2], acc_empty[2], drain;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_sh;
  volatile int* abort = &abort_sh;
  const GemvParams& p = tp.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  float* xpose = reinterpret_cast<float*>(smem_raw + (base - smem_u32(smem_raw)) + size_t(S) * C::kStageBytes);
  const int nk = (p.K + kTcBK - 1) / kTcBK;
  const int tiles = tp.tiles_m * tp.tiles_n;
  const int splits = tp.splits;
  const int items = tiles * splits;  // item i: tile i / splits, K range i % splits
  __shared__ int last_sh;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, kTcEpiWarps);
    }
    mbar_init(&drain, 1);
    *abort = 0;
    mbar_init_fence();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  pdl_launch();
  pdl_wait();

  uint32_t out_seq = 0;
  if constexpr (EPI == kEpiPush) out_seq = resolve_seq(p.comm, p.out_seq);
  int issued = 0;  // producer: k-blocks issued over all tiles (for the drain)

  if (warp == 0) {
    // ---- TMA producer
    if (lane == 0) {
      int g = 0;
      for (int it = blockIdx.x; it < items && !*abort; it += gridDim.x) {
        const int t = it / splits, sp = it - t * splits;
        const int tm = t % tp.tiles_m, tn = t / tp.tiles_m;
        for (int kb = sp * nk / splits; kb < (sp + 1) * nk / splits; ++kb, ++g) {
          const int s = g % S;
          if (g >= S && !mbar_wait(empty + s, uint32_t((g / S) & 1) ^ 1u, tp.budget_ns, abort)) {
            *abort = 1;
            break;
          }
          if (*abort) break;
          const uint32_t sa = base + uint32_t(s) * C::kStageBytes, sb = sa + kTcABytes;
          mbar_arrive_expect_tx(full + s, C::kStageBytes);
          tma_load_2d(sa, &map_x, kb * kTcBK, tm * kTcBM, full + s);
          if constexpr (EPI == kEpiSwiglu) {
            const int u0 = tn * (BN / 2), half = p.N >> 1;
            tma_load_2d(sb, &map_w, kb * kTcBK, u0, full + s);
            tma_load_2d(sb + C::kBBytes / 2, &map_w, kb * kTcBK, half + u0, full + s);
          } else {
            tma_load_2d(sb, &map_w, kb * kTcBK, tn * BN, full + s);
          }
          issued = g + 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      int g = 0, i = 0;
      for (int it = blockIdx.x; it < items && !*abort; it += gridDim.x, ++i) {
        const int sp = it % splits;
        const int kb0 = sp * nk / splits;
        const int b = i & 1, use = i >> 1;
        if (use > 0 && !mbar_wait(acc_empty + b, uint32_t((use - 1) & 1), tp.budget_ns, abort)) {
          *abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + uint32_t(b * BN);
        bool ok = true;
        for (int kb = kb0; kb < (sp + 1) * nk / splits; ++kb, ++g) {
          const int s = g % S;
          if (!mbar_wait(full + s, uint32_t((g / S) & 1), tp.budget_ns, abort)) {
            *abort = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + uint32_t(s) * C::kStageBytes, sb = sa + kTcABytes;
#pragma unroll
          for (int k = 0; k < kTcBK / 16; ++k)
            tc_mma(acc, tc_smem_desc(sa + k * 32), tc_smem_desc(sb + k * 32), C::kIdesc, (kb > kb0 || k > 0) ? 1u : 0u);
          tc_commit(empty + s);  // the stage is free once these MMAs have read it
        }
        if (!ok) break;
        tc_commit(acc_full + b);  // the accumulator is complete once every MMA above has
      }
    }
  } else {
    // ---- epilogue: warp w reads tensor-memory lanes 32 (w % 4) .. + 31 (rows of
    // the tile); warps 2-5 take the first half of the tile's units, 6-9 the second
    const int ew = warp - 2, quarter = warp & 3, part = ew >> 2;
    float* bufa = xpose + size_t(ew) * (2 * 32 * kTcXs);
    float* bufb = bufa + 32 * kTcXs;
    int i = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x, ++i) {
      const int t = it / splits;
      const int b = i & 1, use = i >> 1;
      const int tm = t % tp.tiles_m, tn = t / tp.tiles_m;
      const int row0 = tm * kTcBM + quarter * 32;
      const bool ok = mbar_wait(acc_full + b, uint32_t(use & 1), tp.budget_ns, abort);
      // split items meet at CTA barriers below: there all epilogue warps leave together
      if (splits > 1 ? !named_sync_and(2, 32 * kTcEpiWarps, __all_sync(0xffffffffu, ok))
                     : !__all_sync(0xffffffffu, ok)) {
        if (lane == 0) *abort = 1;
        break;
      }
      tc_fence_after();
      const uint32_t trow = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(b * BN);
      if (splits == 1) {
        auto ld_tmem = [&](int col, uint32_t* r) { tc_ld16(trow + uint32_t(col), r); };
        tc_epilogue_tile<T, EPI, BN>(p, ld_tmem, row0, tn * kUnitsPerTile, part, bufa, bufb, lane, out_seq);
        // the accumulator may be overwritten once every epilogue warp has read it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + b);
        continue;
      }
      if constexpr (BN == 128) {
        // this item's partial: the warp's 32 rows x BN / 2 columns, rows of x only
        const int r = quarter * 32 + lane;
        const bool row_ok = tm * kTcBM + r < p.M;
        if (row0 < p.M) {
          float* dst = tp.ws + size_t(it) * (kTcBM * BN);
#pragma unroll
          for (int c0 = part * (BN / 2); c0 < (part + 1) * (BN / 2); c0 += 16) {
            uint32_t v[16];
            tc_ld16(trow + uint32_t(c0), v);
            tc_wait_ld();
            if (row_ok) {
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<float4*>(dst + tc_ws_off(c0 + j, r)) =
                    make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                                __uint_as_float(v[j + 3]));
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + b);
        // publish: every writer's stores ordered before the count
        __threadfence();
        named_sync(1, 32 * kTcEpiWarps);
        if (warp == 2 && lane == 0) {
          const int prev = atomicAdd(tp.cnt + t, 1);
          const int last = prev == splits - 1;
          if (last) tp.cnt[t] = 0;
          last_sh = last;
        }
        named_sync(1, 32 * kTcEpiWarps);
        if (!last_sh) continue;
        __threadfence();
        // the tile's sum, by all epilogue threads (one float4 of a row each,
        // consecutive threads on consecutive rows), into split 0's partial
        float* sum = tp.ws + size_t(t) * splits * (kTcBM * BN);
        const int rows_t = min(kTcBM, p.M - tm * kTcBM), n4 = rows_t * (BN / 4);
        for (int e4 = int(threadIdx.x) - 64; e4 < n4; e4 += 32 * kTcEpiWarps) {
          const int rr = e4 % rows_t, c4 = e4 / rows_t;
          float4* a0 = reinterpret_cast<float4*>(sum + tc_ws_off(4 * c4, rr));
          float4 acc = __ldcg(a0);
#pragma unroll 8
          for (int q = 1; q < splits; ++q) {
            const float4 f =
                __ldcg(reinterpret_cast<const float4*>(sum + size_t(q) * (kTcBM * BN) + tc_ws_off(4 * c4, rr)));
            acc.x += f.x;
            acc.y += f.y;
            acc.z += f.z;
            acc.w += f.w;
          }
          __stcg(a0, acc);
        }
        named_sync(1, 32 * kTcEpiWarps);
        if (row0 >= p.M) continue;
        auto ld_sum = [&](int col, uint32_t* out) {
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            const float4 f = row_ok ? __ldcg(reinterpret_cast<const float4*>(sum + tc_ws_off(col + j, r)))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
            out[j] = __float_as_uint(f.x);
            out[j + 1] = __float_as_uint(f.y);
            out[j + 2] = __float_as_uint(f.z);
            out[j + 3] = __float_as_uint(f.w);
          }
        };
        tc_epilogue_tile<T, EPI, BN>(p, ld_sum, row0, tn * kUnitsPerTile, part, bufa, bufb, lane, out_seq);
      }
    }
  }
  __syncwarp();
  if constexpr (EPI == kEpiPush) signal_peers(p.comm, p.out_chan, out_seq);

  // ---- teardown: copies and MMAs in flight land before the memory goes away
  if (warp == 0 && lane == 0) {
    int never = 0;
    for (int g = max(0, issued - S); g < issued; ++g)
      mbar_wait(full + (g % S), uint32_t((g / S) & 1), tp.budget_ns, &never);
  }
  if (warp == 1 && lane == 0) {
    int never = 0;
    tc_commit(&drain);  // completes once every MMA this thread issued has
    mbar_wait(&drain, 0u, tp.budget_ns, &never);
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort) atomicOr(p.comm.status(), kStatusTimeout);
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (cta_group::2): a cluster of two CTAs on two SMs computes
// a 256 x 256 output tile. Each CTA loads its own 128 rows of x and half of
// the tile's W rows (128) per K block, so an SM takes in 32 KB per 128 x 256 x
// 64 block of MMAs instead of 48 KB; the leader CTA (cluster rank 0) issues
// tcgen05.mma.cta_group::2 (M 256, N 256), which reads A and B from both
// CTAs' shared memory and accumulates rows 0-127 in the leader's tensor
// memory and rows 128-255 in the peer's. Both CTAs' TMA loads (no multicast)
// complete on the leader's stage barrier; the leader's commits arrive on the
// barriers of both CTAs; the peer's epilogue warps release an accumulator on
// the leader's barrier. Before either CTA frees its tensor memory or exits,
// every stage it loaded has been consumed by the MMAs and a cluster barrier
// has been passed, so no copy, MMA or remote arrive targets a finished CTA.
// ---------------------------------------------------------------------------
constexpr int kTc2Stages = 4;
constexpr uint32_t kTc2StageBytes = 2 * kTcABytes;  // own x tile + own half of the W tile
constexpr size_t kTc2Smem = size_t(kTc2Stages) * kTc2StageBytes + size_t(kTcEpiWarps) * kTcXposeBytes + 1024;
constexpr uint32_t kTc2Idesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(256 >> 3) << 17) | (uint32_t(256 >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t mapa_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2-D TMA load into this CTA's shared memory completing on a barrier of either
// CTA of the pair (no multicast)
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc2_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(da), "l"(db), "r"(kTc2Idesc), "r"(accumulate)
      : "memory");
}
// arrive on the barrier at this offset in both CTAs once the MMAs issued so far complete
__device__ __forceinline__ void tc2_commit_both(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc2_commit_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

template <typename T, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    gemm_tc2_kernel(const TcParams tp, const __grid_constant__ CUtensorMap map_x,
                    const __grid_constant__ CUtensorMap map_w) {
  constexpr int BN = 256;
  constexpr int S = kTc2Stages;
  constexpr bool kPair = EPI == kEpiSwiglu || EPI == kEpiRope;
  constexpr int kUnitsPerTile = kPair ? BN / 2 : BN;
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t full[S], empty[S], acc_full[2], acc_empty[2], drain;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_sh;
  volatile int* abort = &abort_sh;
  const GemvParams& p = tp.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  float* xpose = reinterpret_cast<float*>(smem_raw + (base - smem_u32(smem_raw)) + size_t(S) * kTc2StageBytes);
  const int nk = (p.K + kTcBK - 1) / kTcBK;
  const int tiles = tp.tiles_m * tp.tiles_n;  // 256 x 256 tiles

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);   // the leader's expect-tx arrive (+ both CTAs' bytes)
      mbar_init(empty + s, 1);  // the leader's MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 2 * kTcEpiWarps);  // epilogue warps of both CTAs
    }
    mbar_init(&drain, 1);
    *abort = 0;
    mbar_init_fence();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(2 * BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers and tensor memory exist before any copy or MMA
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  pdl_launch();
  pdl_wait();

  uint32_t out_seq = 0;
  if constexpr (EPI == kEpiPush) out_seq = resolve_seq(p.comm, p.out_seq);
  int issued = 0;

  if (warp == 0) {
    // ---- TMA producer (both CTAs): own x rows and own half of the W rows
    if (lane == 0) {
      const uint32_t full_leader = mapa_rank(smem_u32(full), 0);
      int g = 0;
      for (int t = cid; t < tiles && !*abort; t += ncl) {
        const int tm = t % tp.tiles_m, tn = t / tp.tiles_m;
        int wrow;
        if constexpr (EPI == kEpiSwiglu) {
          wrow = tn * (BN / 2) + (crank ? (p.N >> 1) : 0);  // gate rows in the leader, up rows in the peer
        } else {
          wrow = tn * BN + int(crank) * (BN / 2);
        }
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % S;
          if (g >= S && !mbar_wait(empty + s, uint32_t((g / S) & 1) ^ 1u, tp.budget_ns, abort)) {
            *abort = 1;
            break;
          }
          if (*abort) break;
          const uint32_t sa = base + uint32_t(s) * kTc2StageBytes, sb = sa + kTcABytes;
          if (leader) mbar_arrive_expect_tx(full + s, 2 * kTc2StageBytes);
          tma_load_2d_pair(sa, &map_x, kb * kTcBK, tm * 256 + int(crank) * kTcBM, full_leader + 8u * uint32_t(s));
          tma_load_2d_pair(sb, &map_w, kb * kTcBK, wrow, full_leader + 8u * uint32_t(s));
          issued = g + 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer (leader only)
    if (lane == 0 && leader) {
      int g = 0, i = 0;
      for (int t = cid; t < tiles && !*abort; t += ncl, ++i) {
        const int b = i & 1, use = i >> 1;
        if (use > 0 && !mbar_wait(acc_empty + b, uint32_t((use - 1) & 1), tp.budget_ns, abort)) {
          *abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + uint32_t(b * BN);
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % S;
          if (!mbar_wait(full + s, uint32_t((g / S) & 1), tp.budget_ns, abort)) {
            *abort = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + uint32_t(s) * kTc2StageBytes, sb = sa + kTcABytes;
#pragma unroll
          for (int k = 0; k < kTcBK / 16; ++k)
            tc2_mma(acc, tc_smem_desc(sa + k * 32), tc_smem_desc(sb + k * 32), (kb > 0 || k > 0) ? 1u : 0u);
          tc2_commit_both(empty + s);  // both CTAs' stage s is free once these MMAs have read it
        }
        if (!ok) break;
        tc2_commit_both(acc_full + b);
      }
    }
  } else {
    // ---- epilogue (both CTAs): this CTA's 128 rows of the tile
    const int ew = warp - 2, quarter = warp & 3, part = ew >> 2;
    float* bufa = xpose + size_t(ew) * (2 * 32 * kTcXs);
    float* bufb = bufa + 32 * kTcXs;
    const uint32_t acc_empty_leader = mapa_rank(smem_u32(acc_empty), 0);
    int i = 0;
    for (int t = cid; t < tiles; t += ncl, ++i) {
      const int b = i & 1, use = i >> 1;
      const int tm = t % tp.tiles_m, tn = t / tp.tiles_m;
      const bool ok = mbar_wait(acc_full + b, uint32_t(use & 1), tp.budget_ns, abort);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) *abort = 1;
        break;
      }
      tc_fence_after();
      const uint32_t trow = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(b * BN);
      auto ld_tmem = [&](int col, uint32_t* r) { tc_ld16(trow + uint32_t(col), r); };
      tc_epilogue_tile<T, EPI, BN>(p, ld_tmem, tm * 256 + int(crank) * kTcBM + quarter * 32, tn * kUnitsPerTile, part,
                                   bufa, bufb, lane, out_seq);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader + 8u * uint32_t(b));
    }
  }
  __syncwarp();
  if constexpr (EPI == kEpiPush) signal_peers(p.comm, p.out_chan, out_seq);

  // ---- teardown
  if (warp == 0 && lane == 0) {
    // every stage this CTA loaded has been read by the MMAs (so its copies landed)
    int never = 0;
    for (int g = max(0, issued - S); g < issued; ++g)
      mbar_wait(empty + (g % S), uint32_t((g / S) & 1), tp.budget_ns, &never);
  }
  if (warp == 1 && lane == 0 && leader) {
    int never = 0;
    tc2_commit_local(&drain);  // completes once every MMA this thread issued has
    mbar_wait(&drain, 0u, tp.budget_ns, &never);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer is done with this CTA's memory
  if (threadIdx.x == 0 && *abort) atomicOr(p.comm.status(), kStatusTimeout);
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN) : "memory");
  }
}

}  // namespace mtpb
