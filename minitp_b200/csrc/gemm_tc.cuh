// Tensor-core GEMM for the prefill projections (bf16): y = x · Wᵀ with the
// GEMV path's epilogues (store, SwiGLU, RoPE + KV append, AllReduce push).
//
// One CTA computes a 128 x 128 output tile (rows of x by rows of W) with
// 5th-generation tensor cores: warp 0 streams 128 x 64 tiles of x and W into
// a 4-stage shared-memory pipeline with 2-D TMA loads (128-byte swizzle, no
// multicast), warp 1 issues tcgen05.mma (M 128, N 128, K 16, bf16 inputs, fp32
// accumulator in tensor memory), warp 2 owns the tensor-memory allocation, and
// all four warps run the epilogue from tensor memory (tcgen05.ld). Every wait
// is bounded; on expiry the CTA records a status bit, lets its copies and
// MMAs land, frees its tensor memory and returns.
//
// Output units follow the GEMV epilogue: SwiGLU pairs gate row u with up row
// I + u, so its W tile is loaded as two 64-row halves (gate rows, then the
// matching up rows); RoPE pairs rows i and i + hd/2 of a head, which a tile of
// whole heads holds in columns c and c + hd/2.
#pragma once

#include <cuda.h>

#include "gemv.cuh"
#include "tma.cuh"

namespace mtpb {

constexpr int kTcBM = 128, kTcBN = 128, kTcBK = 64, kTcStages = 4;
constexpr int kTcThreads = 128;
constexpr uint32_t kTcHalfStage = kTcBM * kTcBK * 2;  // one 128 x 64 bf16 tile: 16 KB
constexpr uint32_t kTcStageBytes = 2 * kTcHalfStage;  // x tile + W tile
constexpr size_t kTcSmem = size_t(kTcStages) * kTcStageBytes + 1024;

struct TcParams {
  GemvParams g;  // shapes, inputs and epilogue fields (GEMV conventions)
  int tiles_n;   // output tiles along N
  uint64_t budget_ns;
};

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

// Instruction descriptor: bf16 x bf16 -> fp32, both K-major, M 128, N 128.
constexpr uint32_t kTcIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kTcBN >> 3) << 17) |
                              (uint32_t(kTcBM >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(da), "l"(db), "r"(kTcIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's tensor-memory lane
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <typename T, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const TcParams tp, const __grid_constant__ CUtensorMap map_x,
                   const __grid_constant__ CUtensorMap map_w) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint64_t full[kTcStages], empty[kTcStages], accb;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_sh;
  volatile int* abort = &abort_sh;
  const GemvParams& p = tp.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tn = blockIdx.x % tp.tiles_n, tm = blockIdx.x / tp.tiles_n;
  const int m0 = tm * kTcBM;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int nk = (p.K + kTcBK - 1) / kTcBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(&accb, 1);
    *abort = 0;
    mbar_init_fence();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(kTcBN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  pdl_launch();
  pdl_wait();

  int issued = 0;  // producer: stages issued (for the drain)
  if (warp == 0 && lane == 0) {
    // ---- TMA producer
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kTcStages;
      if (kb >= kTcStages && !mbar_wait(empty + s, uint32_t((kb / kTcStages) & 1) ^ 1u, tp.budget_ns, abort)) {
        *abort = 1;
        break;
      }
      if (*abort) break;
      const uint32_t sa = base + uint32_t(s) * kTcStageBytes, sb = sa + kTcHalfStage;
      mbar_arrive_expect_tx(full + s, kTcStageBytes);
      tma_load_2d(sa, &map_x, kb * kTcBK, m0, full + s);
      if constexpr (EPI == kEpiSwiglu) {
        const int u0 = tn * (kTcBN / 2), half = p.N >> 1;
        tma_load_2d(sb, &map_w, kb * kTcBK, u0, full + s);
        tma_load_2d(sb + kTcHalfStage / 2, &map_w, kb * kTcBK, half + u0, full + s);
      } else {
        tma_load_2d(sb, &map_w, kb * kTcBK, tn * kTcBN, full + s);
      }
      ++issued;
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kTcStages;
      if (!mbar_wait(full + s, uint32_t((kb / kTcStages) & 1), tp.budget_ns, abort)) {
        *abort = 1;
        break;
      }
      tc_fence_after();
      const uint32_t sa = base + uint32_t(s) * kTcStageBytes, sb = sa + kTcHalfStage;
#pragma unroll
      for (int k = 0; k < kTcBK / 16; ++k)
        tc_mma(tmem, tc_smem_desc(sa + k * 32), tc_smem_desc(sb + k * 32), (kb > 0 || k > 0) ? 1u : 0u);
      tc_commit(empty + s);  // the stage is free once these MMAs have read it
    }
    tc_commit(&accb);  // the accumulator is complete once every MMA above has
  }
  __syncwarp();

  // ---- epilogue: warp w owns tensor-memory lanes (rows) 32 w .. 32 w + 31
  const bool acc_ok = mbar_wait(&accb, 0u, tp.budget_ns, abort);
  tc_fence_after();
  const bool good = __all_sync(0xffffffffu, acc_ok && !*abort);
  const int m = m0 + warp * 32 + lane;
  const uint32_t trow = tmem + (uint32_t(warp * 32) << 16);
  uint32_t out_seq = 0;
  if constexpr (EPI == kEpiPush) out_seq = resolve_seq(p.comm, p.out_seq);
  if (good) {
    if constexpr (EPI == kEpiSwiglu) {
      const int half = p.N >> 1;
      for (int c0 = 0; c0 < kTcBN / 2; c0 += 16) {
        float g[16], u[16];
        tc_ld16(trow + c0, g);
        tc_ld16(trow + kTcBN / 2 + c0, u);
        if (m < p.M) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int unit = tn * (kTcBN / 2) + c0 + j;
            if (unit < half) gemv_epilogue<T, EPI>(p, m, unit, g[j], u[j], out_seq, nullptr);
          }
        }
      }
    } else if constexpr (EPI == kEpiRope) {
      // the tile holds whole heads: columns c and c + hd/2 of a head pair up
      const int hd = p.hd, half = hd >> 1;
      for (int h0 = 0; h0 < kTcBN; h0 += hd) {
        for (int c0 = 0; c0 < half; c0 += 16) {
          float a[16], b[16];
          tc_ld16(trow + h0 + c0, a);
          tc_ld16(trow + h0 + half + c0, b);
          if (m < p.M) {
            const int head = (tn * kTcBN + h0) / hd;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int unit = head * half + c0 + j;
              if (head < p.hq + 2 * p.hkv) gemv_epilogue<T, EPI>(p, m, unit, a[j], b[j], out_seq, nullptr);
            }
          }
        }
      }
    } else {
      for (int c0 = 0; c0 < kTcBN; c0 += 16) {
        float v[16];
        tc_ld16(trow + c0, v);
        if (m < p.M) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int unit = tn * kTcBN + c0 + j;
            if (unit < p.N) gemv_epilogue<T, EPI>(p, m, unit, v[j], 0.f, out_seq, nullptr);
          }
        }
      }
    }
  } else if (threadIdx.x == 0) {
    atomicOr(p.comm.status(), kStatusTimeout);
  }
  if constexpr (EPI == kEpiPush) signal_peers(p.comm, p.out_chan, out_seq);

  // ---- teardown: copies and MMAs in flight land before the memory goes away
  if (warp == 0 && lane == 0) {
    int never = 0;
    for (int kb = max(0, issued - kTcStages); kb < issued; ++kb)
      mbar_wait(full + (kb % kTcStages), uint32_t((kb / kTcStages) & 1), tp.budget_ns, &never);
  }
  if (warp == 1 && lane == 0 && !acc_ok) {
    int never = 0;
    mbar_wait(&accb, 0u, tp.budget_ns, &never);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcBN) : "memory");
  }
}

}  // namespace mtpb
