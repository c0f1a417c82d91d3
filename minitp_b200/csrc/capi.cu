// C ABI of libminitp_b200.so (declared in include/minitp_b200.h): launch
// configuration, the NVLink communicator, standalone operators and the model
// sequencer that chains the kernels of one forward / one decode step.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "attention.cuh"
#include "gemv.cuh"
#include "minitp_b200.h"
#include "misc.cuh"
#include "ar_rows.cuh"
#include "decode_mk_launch.cuh"
#include "gemm_tc.cuh"

#include <cudaTypedefs.h>

using namespace mtpb;

namespace {

thread_local std::string g_err;
bool g_pdl = true;
uint32_t g_prefetch_cap = 4u << 20;
int g_gemv_ctas_per_sm = 2;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
int fail_cuda(cudaError_t e, const char* what) {
  return fail(MTPB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
#define MTPB_CUDA(call)                                 \
  do {                                                  \
    cudaError_t e_ = (call);                            \
    if (e_ != cudaSuccess) return fail_cuda(e_, #call); \
  } while (0)
#define MTPB_TRY(call)         \
  do {                         \
    int r_ = (call);           \
    if (r_ != MTPB_OK) return r_; \
  } while (0)

size_t dsize(int dtype) { return dtype == MTPB_BF16 ? 2 : 4; }
int vec_elems(int dtype) { return dtype == MTPB_BF16 ? 8 : 4; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <typename Kern, typename Param>
int launch(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, const Param& prm) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl ? 1 : 0;
  if (smem > 48 * 1024) {
    MTPB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  }
  MTPB_CUDA(cudaLaunchKernelEx(&cfg, kern, prm));
  return MTPB_OK;
}

// ------------------------------------------------------------------ comm
struct CommHost {
  Comm dev;
  void* local = nullptr;
  void* mapped[kMaxRanks] = {};
  int device = 0;
  bool open = false;
  uint32_t ping_calls = 0;  // mtpb_comm_pingpong calls (their sequence numbers)
};

// A communicator-less call still needs control words and a local slot: a
// lazily created world-1 communicator per device serves those.
CommHost* default_comm() {
  static std::mutex mu;
  static CommHost* per_dev[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!per_dev[dev]) {
    void* c = nullptr;
    if (mtpb_comm_create(0, 1, 1u << 20, &c) != MTPB_OK) return nullptr;
    per_dev[dev] = static_cast<CommHost*>(c);
  }
  return per_dev[dev];
}

CommHost* as_comm(void* c) { return c ? static_cast<CommHost*>(c) : default_comm(); }

// ------------------------------------------------------------------ GEMV launch
constexpr size_t kXsStageMax = 64 * 1024;  // x staged in smem up to this size

template <typename T, int EPI>
int gemv_launch(GemvParams p, cudaStream_t st) {
  constexpr int UR = EpiTraits<EPI>::kUR;
  constexpr int RPW = kRowsPerWarp / UR;
  constexpr int VE = VecTraits<T>::kElems;
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return fail(MTPB_ERR_INVALID, "gemv: empty shape");
  if (p.K % VE != 0 || !aligned16(p.w)) {
    return fail(MTPB_ERR_INVALID, "gemv: K * sizeof(dtype) must be a multiple of 16 bytes and w 16-byte aligned");
  }
  if (p.x_mode == 0 && (!aligned16(p.x) || (size_t(p.ldx) * sizeof(T)) % 16 != 0)) {
    return fail(MTPB_ERR_INVALID, "gemv: x must be 16-byte aligned with a 16-byte row stride");
  }
  if (EPI == kEpiArgmax && p.M > 64) return fail(MTPB_ERR_INVALID, "gemv argmax: M > 64");
  const int sms = sm_count();
  const int G = std::max(1, std::min(p.units, std::min(sms * g_gemv_ctas_per_sm, kMaxCtas)));
  const int per = (p.units + G - 1) / G;
  const int groups = (per + RPW - 1) / RPW;
  const int CPR = p.K / VE;
  int ks = 1;
  while (ks < kGemvWarps && groups * ks * 2 <= kGemvWarps && CPR / (ks * 2) >= 16) ks *= 2;
  p.ks = ks;
  const size_t xbytes = size_t(p.M) * p.K * sizeof(T);
  if (p.x_mode == 1) {
    if (xbytes > 200 * 1024) return fail(MTPB_ERR_INVALID, "gemv consume: x does not fit in shared memory");
    p.x_smem = 1;
  } else {
    p.x_smem = xbytes <= kXsStageMax ? 1 : 0;
  }
  p.prefetch_cap = g_prefetch_cap;
  const size_t smem = (p.x_smem ? xbytes : 0) + size_t(kGemvWarps) * 32 * 2 * sizeof(float);
  const int MT = p.M >= 8 ? 8 : p.M >= 4 ? 4 : p.M >= 2 ? 2 : 1;
  switch (MT) {
    case 1: return launch(gemv_kernel<T, EPI, 1>, dim3(G), dim3(kGemvThreads), smem, st, p);
    case 2: return launch(gemv_kernel<T, EPI, 2>, dim3(G), dim3(kGemvThreads), smem, st, p);
    case 4: return launch(gemv_kernel<T, EPI, 4>, dim3(G), dim3(kGemvThreads), smem, st, p);
    default: return launch(gemv_kernel<T, EPI, 8>, dim3(G), dim3(kGemvThreads), smem, st, p);
  }
}

// ------------------------------------------------------------------ tensor-core GEMM (prefill)
bool capturing(cudaStream_t st);
int g_tc_min_rows = 64;  // bf16 projections of at least this many rows use tcgen05
// the same for the projections of a decode step (one row per batch row): the
// CUDA-core GEMV turns compute-bound at a few tens of rows
int g_tc_min_rows_decode = 8;

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// 2-D bf16 tensor map over rows x cols (row stride ld elements), box
// box_rows x 64 columns, 128-byte swizzle; out-of-range boxes read zeros.
// Encoded maps are kept in a small cache keyed on all of those fields (a map
// holds nothing else), so a prefill chain re-encodes only new buffers.
int make_map_bf16(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
  struct Entry {
    const void* ptr;
    uint64_t rows, cols, ld;
    uint32_t box;
    CUtensorMap map;
  };
  static Entry cache[64];
  static int used = 0, next = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i) {
    const Entry& e = cache[i];
    if (e.ptr == ptr && e.rows == rows && e.cols == cols && e.ld == ld && e.box == box_rows) {
      *map = e.map;
      return MTPB_OK;
    }
  }
  auto enc = tensor_map_encoder();
  if (!enc) return fail(MTPB_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {uint32_t(kTcBK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MTPB_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  Entry& e = cache[next];
  e = Entry{ptr, rows, cols, ld, box_rows, *map};
  next = (next + 1) % 64;
  used = std::max(used, next == 0 ? 64 : next);
  return MTPB_OK;
}

template <int EPI>
bool tc_eligible(int dtype, const GemvParams& p) {
  if (dtype != MTPB_BF16 || p.M < (p.decode ? g_tc_min_rows_decode : g_tc_min_rows) || p.x_mode != 0 || !p.x)
    return false;
  if (EPI != kEpiStore && EPI != kEpiSwiglu && EPI != kEpiRope && EPI != kEpiPush) return false;
  if (p.K % 8 || p.ldx % 8 || p.K < kTcBK || !aligned16(p.x) || !aligned16(p.w)) return false;
  if (EPI == kEpiRope && (p.hd < 32 || p.hd > 128 || 128 % p.hd)) return false;
  if (EPI == kEpiSwiglu && (p.N % 2)) return false;
  return true;
}

// output tiles along N for a tile width of BN accumulator columns
template <int EPI>
int tc_tiles_n(const GemvParams& p, int bn) {
  if (EPI == kEpiSwiglu) return ((p.N >> 1) + bn / 2 - 1) / (bn / 2);
  return (p.N + bn - 1) / bn;
}

// Launch plan of a tensor-core GEMM: CTA pairs with 256 x 256 tiles when
// there are at least as many tiles as co-resident pairs, else single CTAs
// with 128-row tiles 256 columns wide when those alone give every SM a tile,
// else 128 wide (more CTAs on the small-M, HBM-bound shapes). Persistent
// grids: one CTA per SM at most.
struct TcPlan {
  int pair;    // 1: gemm_tc2_kernel (cta_group::2)
  int bn;      // single-CTA tile width
  int tiles_m, tiles_n;
  int splits;  // K ranges per tile (single CTAs, BN 128)
  int grid;
};

int g_tc_pair = 1;       // CTA-pair kernel allowed
int g_tc_split_max = 32;  // most K ranges per output tile (1: no split K)

// Split-K workspace of a device: fp32 partial tiles for at most one item per
// SM (a split plan never has more items than SMs) and one arrival counter per
// tile (zero between launches; the kernel returns each to zero). One set per
// device, so split GEMMs on one device run one at a time (one stream).
struct TcSplitWs {
  float* ws = nullptr;
  int* cnt = nullptr;
};

int tc_split_ws(cudaStream_t st, TcSplitWs* out) {
  static std::mutex mu;
  static TcSplitWs per_dev[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  TcSplitWs& w = per_dev[dev];
  if (!w.ws) {
    if (capturing(st)) return fail(MTPB_ERR_INVALID, "tensor-core GEMM: run one call eagerly before graph capture");
    const size_t items = size_t(sm_count());
    MTPB_CUDA(cudaMalloc(&w.ws, items * kTcBM * 128 * sizeof(float)));
    MTPB_CUDA(cudaMalloc(&w.cnt, items * sizeof(int)));
    MTPB_CUDA(cudaMemset(w.cnt, 0, items * sizeof(int)));
  }
  *out = w;
  return MTPB_OK;
}

// Per-epilogue one-time setup: shared-memory limits of the three kernels and
// the number of co-resident CTA pairs (their shared memory allows one CTA per
// SM). Done on the first eligible call, which must not be under graph capture.
struct TcState {
  bool ready = false;
  int pairs = 0;
};

template <int EPI>
TcState& tc_state() {
  static TcState s;
  return s;
}

template <int EPI>
int tc_prepare(cudaStream_t st) {
  TcState& s = tc_state<EPI>();
  if (s.ready) return MTPB_OK;
  if (capturing(st)) return fail(MTPB_ERR_INVALID, "tensor-core GEMM: run one call eagerly before graph capture");
  MTPB_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<bf16, EPI, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(TcCfg<128>::kSmem)));
  MTPB_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<bf16, EPI, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(TcCfg<256>::kSmem)));
  MTPB_CUDA(cudaFuncSetAttribute(gemm_tc2_kernel<bf16, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(kTc2Smem)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * sm_count());
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = kTc2Smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_tc2_kernel<bf16, EPI>, &cfg) != cudaSuccess || n < 0) {
    cudaGetLastError();
    n = 0;
  }
  s.pairs = std::min(n, sm_count() / 2);
  s.ready = true;
  return MTPB_OK;
}

template <int EPI>
TcPlan tc_plan(const GemvParams& p) {
  TcPlan pl{};
  const int pairs = (g_tc_pair && p.M >= 256) ? tc_state<EPI>().pairs : 0;
  const int tm2 = (p.M + 255) / 256, tn2 = tc_tiles_n<EPI>(p, 256);
  if (pairs > 0 && tm2 * tn2 >= pairs) {
    pl.pair = 1;
    pl.tiles_m = tm2;
    pl.tiles_n = tn2;
    pl.grid = 2 * std::min(tm2 * tn2, pairs);
    return pl;
  }
  const int sms = sm_count();
  pl.tiles_m = (p.M + kTcBM - 1) / kTcBM;
  pl.bn = pl.tiles_m * tc_tiles_n<EPI>(p, 256) >= sms ? 256 : 128;
  pl.tiles_n = tc_tiles_n<EPI>(p, pl.bn);
  // split K for projections of at most 64 rows (decode steps of many rows)
  // whose tiles fill at most half of the SMs: as many ranges as keep every
  // item within one per SM, each of at least two K blocks. (On full 128-row
  // tiles the last CTA's sum of the partials cost more than the split saved:
  // a 128-token prefill of the 0.5B shape took 4.7 ms with it, 3.1 without.)
  const int tiles = pl.tiles_m * pl.tiles_n, nk = (p.K + kTcBK - 1) / kTcBK;
  pl.splits = 1;
  if (pl.bn == 128 && g_tc_split_max > 1 && p.M <= 64 && 2 * tiles <= sms)
    pl.splits = std::max(1, std::min(std::min(sms / tiles, nk / 2), g_tc_split_max));
  pl.grid = std::min(tiles * pl.splits, sms);
  return pl;
}

template <int EPI>
int tc_grid(const GemvParams& p) {
  return tc_plan<EPI>(p).grid;
}

template <typename K>
int tc_launch_kernel(K kern, const TcPlan& pl, size_t smem, const TcParams& tp, const CUtensorMap& mx,
                     const CUtensorMap& mw, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl ? 1 : 0;
  MTPB_CUDA(cudaLaunchKernelEx(&cfg, kern, tp, mx, mw));
  return MTPB_OK;
}

template <int EPI>
int gemm_tc_launch(const GemvParams& g, cudaStream_t st) {
  MTPB_TRY(tc_prepare<EPI>(st));
  const TcPlan pl = tc_plan<EPI>(g);
  TcParams tp;
  tp.g = g;
  tp.tiles_m = pl.tiles_m;
  tp.tiles_n = pl.tiles_n;
  tp.splits = pl.pair ? 1 : pl.splits;
  tp.ws = nullptr;
  tp.cnt = nullptr;
  if (tp.splits > 1) {
    TcSplitWs w;
    MTPB_TRY(tc_split_ws(st, &w));
    tp.ws = w.ws;
    tp.cnt = w.cnt;
  }
  tp.budget_ns = 2000000000ull;
  // W boxes: a CTA of a pair loads 128 rows; a single CTA BN rows (SwiGLU: two halves)
  const uint32_t wbox = pl.pair ? 128u : uint32_t(EPI == kEpiSwiglu ? pl.bn / 2 : pl.bn);
  CUtensorMap mx, mw;
  MTPB_TRY(make_map_bf16(&mx, g.x, uint64_t(g.M), uint64_t(g.K), uint64_t(g.ldx), kTcBM));
  MTPB_TRY(make_map_bf16(&mw, g.w, uint64_t(g.N), uint64_t(g.K), uint64_t(g.K), wbox));
  if (pl.pair) return tc_launch_kernel(gemm_tc2_kernel<bf16, EPI>, pl, kTc2Smem, tp, mx, mw, st);
  if (pl.bn == 256) return tc_launch_kernel(gemm_tc_kernel<bf16, EPI, 256>, pl, TcCfg<256>::kSmem, tp, mx, mw, st);
  return tc_launch_kernel(gemm_tc_kernel<bf16, EPI, 128>, pl, TcCfg<128>::kSmem, tp, mx, mw, st);
}

template <int EPI>
int gemv_dispatch(int dtype, const GemvParams& p, cudaStream_t st) {
  if (tc_eligible<EPI>(dtype, p)) return gemm_tc_launch<EPI>(p, st);
  if (dtype == MTPB_BF16) return gemv_launch<bf16, EPI>(p, st);
  if (dtype == MTPB_F32) return gemv_launch<float, EPI>(p, st);
  return fail(MTPB_ERR_INVALID, "unsupported dtype");
}

// grid size a GEMV launch will use (producer CTA count of a push site)
int gemv_grid(int units) {
  return std::max(1, std::min(units, std::min(sm_count() * g_gemv_ctas_per_sm, kMaxCtas)));
}

// producer CTA count of a push-epilogue dispatch (GEMV or tensor-core GEMM)
int push_grid(int dtype, const GemvParams& p) {
  return tc_eligible<kEpiPush>(dtype, p) ? tc_grid<kEpiPush>(p) : gemv_grid(p.units);
}

GemvParams gemv_base(const void* w, const void* bias, int M, int N, int K, int units) {
  GemvParams p;
  std::memset(&p, 0, sizeof(p));
  p.w = w;
  p.bias = bias;
  p.M = M;
  p.N = N;
  p.K = K;
  p.units = units;
  p.tpr = 1;
  return p;
}

// ------------------------------------------------------------------ attention launch
constexpr size_t kAttnSmemMax = 160 * 1024;

struct AttnScratch {
  float* part_o = nullptr;
  float* part_ml = nullptr;
  uint32_t* counters = nullptr;
  size_t o_elems = 0, ml_elems = 0, ctr_elems = 0;
};

int attn_choose_splits(int M, int hkv, int G, int cap, int hd, int* chunk_cap) {
  const int sms = sm_count();
  int ns = 1;
  // fill the GPU: (rows x kv heads x splits) >= SMs, but keep >= 64 keys per split
  while (M * hkv * ns < sms && (cap + ns * 2 - 1) / (ns * 2) >= 64) ns *= 2;
  // bound the score buffer in shared memory
  auto smem_of = [&](int s) {
    const int cc = (cap + s - 1) / s;
    return size_t(G) * hd * 4 + size_t(G) * cc * 4 + size_t(G) * 8 + 16 * 1024 + 64;
  };
  while (smem_of(ns) > kAttnSmemMax) ns *= 2;
  *chunk_cap = (cap + ns - 1) / ns;
  return ns;
}

template <typename T>
int attn_launch_t(AttnParams p, int hd, cudaStream_t st) {
  const int G = p.hq / p.hkv;
  const size_t smem = size_t(G) * hd * 4 + size_t(G) * p.chunk_cap * 4 + size_t(G) * 8 + 16 * 1024 + 64;
  dim3 grid(p.nsplit, p.hkv, p.M);
  switch (hd) {
    case 16: return launch(attn_kernel<T, 16>, grid, dim3(kAttnThreads), smem, st, p);
    case 32: return launch(attn_kernel<T, 32>, grid, dim3(kAttnThreads), smem, st, p);
    case 64: return launch(attn_kernel<T, 64>, grid, dim3(kAttnThreads), smem, st, p);
    case 128: return launch(attn_kernel<T, 128>, grid, dim3(kAttnThreads), smem, st, p);
    default: return fail(MTPB_ERR_INVALID, "attention: head_dim must be 16, 32, 64 or 128");
  }
}

template <typename T>
int attn_pf_launch(const AttnParams& p, int hd, int G, int rpt, cudaStream_t st) {
  const int qt = 16 * rpt / G;
  dim3 grid((p.tpr + qt - 1) / qt, p.hkv, p.M / p.tpr);
  if (hd == 64 && rpt == 8)
    return launch(attn_prefill_kernel<T, 64, 8>, grid, dim3(kAttnPfThreads), attn_pf_smem<64, 8>(), st, p);
  if (hd == 64) return launch(attn_prefill_kernel<T, 64, 4>, grid, dim3(kAttnPfThreads), attn_pf_smem<64, 4>(), st, p);
  if (rpt == 8)
    return launch(attn_prefill_kernel<T, 128, 8>, grid, dim3(kAttnPfThreads), attn_pf_smem<128, 8>(), st, p);
  return launch(attn_prefill_kernel<T, 128, 4>, grid, dim3(kAttnPfThreads), attn_pf_smem<128, 4>(), st, p);
}

int attn_run(int dtype, const void* q, const void* kc, const void* vc, void* out, int B, int T, int hq,
             int hkv, int hd, int cap, const int* pos_ptr, int pos_base, AttnScratch& scr,
             uint32_t* status, cudaStream_t st) {
  if (hq % hkv != 0) return fail(MTPB_ERR_INVALID, "attention: hq must be a multiple of hkv");
  const int G = hq / hkv;
  if (G > 64) return fail(MTPB_ERR_INVALID, "attention: more than 64 query heads per KV head");
  if (B * T > 65535 || hkv > 65535) return fail(MTPB_ERR_INVALID, "attention: more than 65535 rows per launch");
  if (dtype == MTPB_F32 && hd < 16) return fail(MTPB_ERR_INVALID, "attention: head_dim too small");
  const int M = B * T;
  AttnParams p;
  std::memset(&p, 0, sizeof(p));
  p.q = q;
  p.k_cache = kc;
  p.v_cache = vc;
  p.out = out;
  p.M = M;
  p.tpr = T;
  p.hq = hq;
  p.hkv = hkv;
  p.cap = cap;
  p.pos_ptr = pos_ptr;
  p.pos_base = pos_base;
  p.scale = 1.0f / std::sqrt(float(hd));
  // prefill: query tiles with K/V streamed through shared memory (no scratch)
  if (T >= kAttnPfMinT && (hd == 64 || hd == 128)) {
    p.nsplit = 1;
    // 128 (query, head) rows per CTA when that still gives every SM a tile, else 64
    const bool big = (T + 128 / G - 1) / (128 / G) * hkv * B >= sm_count();
    if (dtype == MTPB_BF16) return attn_pf_launch<bf16>(p, hd, G, big ? 8 : 4, st);
    if (dtype == MTPB_F32) return attn_pf_launch<float>(p, hd, G, big ? 8 : 4, st);
    return fail(MTPB_ERR_INVALID, "unsupported dtype");
  }
  p.nsplit = attn_choose_splits(M, hkv, G, cap, hd, &p.chunk_cap);
  p.status = status;
  if (p.nsplit > 1) {
    const size_t need_o = size_t(M) * hq * p.nsplit * hd, need_ml = size_t(M) * hq * p.nsplit * 2,
                 need_c = size_t(M) * hkv;
    if (need_o > scr.o_elems || need_ml > scr.ml_elems || need_c > scr.ctr_elems) {
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      cudaStreamIsCapturing(st, &cs);
      if (cs != cudaStreamCaptureStatusNone)
        return fail(MTPB_ERR_INVALID, "attention scratch must be reserved before graph capture");
      cudaFree(scr.part_o);
      cudaFree(scr.part_ml);
      cudaFree(scr.counters);
      MTPB_CUDA(cudaMalloc(&scr.part_o, need_o * 4));
      MTPB_CUDA(cudaMalloc(&scr.part_ml, need_ml * 4));
      MTPB_CUDA(cudaMalloc(&scr.counters, need_c * 4));
      MTPB_CUDA(cudaMemsetAsync(scr.counters, 0, need_c * 4, st));
      scr.o_elems = need_o;
      scr.ml_elems = need_ml;
      scr.ctr_elems = need_c;
    }
    p.part_o = scr.part_o;
    p.part_ml = scr.part_ml;
    p.counters = scr.counters;
  }
  if (dtype == MTPB_BF16) return attn_launch_t<bf16>(p, hd, st);
  if (dtype == MTPB_F32) return attn_launch_t<float>(p, hd, st);
  return fail(MTPB_ERR_INVALID, "unsupported dtype");
}

AttnScratch& standalone_attn_scratch() {
  static AttnScratch s[64];
  int dev = 0;
  cudaGetDevice(&dev);
  return s[dev];
}

// ------------------------------------------------------------------ small launches
template <typename T>
int embed_launch(const EmbedParams& p, int grid, cudaStream_t st) {
  return launch(embed_kernel<T>, dim3(grid), dim3(128), 0, st, p);
}
int embed_run(int dtype, const EmbedParams& p, int grid, cudaStream_t st) {
  if (dtype == MTPB_BF16) return embed_launch<bf16>(p, grid, st);
  if (dtype == MTPB_F32) return embed_launch<float>(p, grid, st);
  return fail(MTPB_ERR_INVALID, "unsupported dtype");
}

// Two-shot AllReduce sites of the model (reduce-scatter + all-gather,
// comm.cuh) for messages of at least g_ts_min_bytes on at least
// g_ts_min_world ranks: each rank then sends 2 (tp - 1) / tp of the message
// instead of (tp - 1) copies, for one more flag round trip. Off by default:
// on the 7B shape at TP=4 a 1024-token prefill took 7.05 ms with every such
// site two-shot and 6.87 ms one-shot (8 layers; 46.3 vs 45.4 ms at batch 8).
long long g_ts_min_bytes = -1;
int g_ts_min_world = 4;

// Column slice width of a two-shot site of rows of H values (0: one-shot).
int ts_cols_for(size_t bytes, int H, int world, int dtype) {
  if (g_ts_min_bytes < 0 || world < std::max(2, g_ts_min_world) || bytes < size_t(g_ts_min_bytes)) return 0;
  if (!(dtype == MTPB_BF16 ? ar_rows_vec_ok<bf16>(H) : ar_rows_vec_ok<float>(H))) return 0;
  // producer and consumer grids stay below the all-gather flag indices
  if (sm_count() * std::max(2, g_gemv_ctas_per_sm) > kAgCta) return 0;
  const int VE = vec_elems(dtype);
  const int per = (H + world - 1) / world;
  return (per + VE - 1) / VE * VE;
}

int ar_norm_run(int dtype, ArNormParams p, cudaStream_t st) {
  if (size_t(p.rows) * p.H * dsize(dtype) > p.comm.slot_bytes && p.comm.world > 1)
    return fail(MTPB_ERR_INVALID, "allreduce: message larger than the communicator slot");
  // LL words (8 bytes per 2 bf16 / 1 fp32 value) when they fit the slot
  const int P = dtype == MTPB_BF16 ? 2 : 1;
  const bool ll = p.comm.world > 1 && p.H % P == 0 && size_t(p.rows) * (p.H / P) * 8 <= p.comm.slot_bytes;
  // rows per CTA: spread rows over the SMs, at most kMaxCtas CTAs
  const int sms = sm_count();
  int ctas = std::min(p.rows, std::min(sms * 2, kMaxCtas));
  ctas = std::max(ctas, 1);
  p.rpc = (p.rows + ctas - 1) / ctas;
  ctas = (p.rows + p.rpc - 1) / p.rpc;
  if (ll) p.chan = 3;  // LL words never share a slot with raw data
  if (dtype == MTPB_BF16)
    return ll ? launch(ar_norm_ll_kernel<bf16>, dim3(ctas), dim3(256), 0, st, p)
              : launch(ar_norm_kernel<bf16>, dim3(ctas), dim3(256), 0, st, p);
  if (dtype == MTPB_F32)
    return ll ? launch(ar_norm_ll_kernel<float>, dim3(ctas), dim3(256), 0, st, p)
              : launch(ar_norm_kernel<float>, dim3(ctas), dim3(256), 0, st, p);
  return fail(MTPB_ERR_INVALID, "unsupported dtype");
}

int argmax_splits(int V) { return std::max(1, std::min(64, (V + 4095) / 4096)); }

int argmax_rows_run(int dtype, const ArgmaxRowsParams& p, cudaStream_t st) {
  dim3 grid(argmax_splits(p.V), p.M);
  if (dtype == MTPB_BF16) return launch(argmax_rows_kernel<bf16>, grid, dim3(256), 0, st, p);
  if (dtype == MTPB_F32) return launch(argmax_rows_kernel<float>, grid, dim3(256), 0, st, p);
  return fail(MTPB_ERR_INVALID, "unsupported dtype");
}

// a consumer-only pass for the model channel when x does not fit in shared
// memory: it reduces a collective site into res_out and the normalised xn.
struct ConsumeRowsParams {
  GemvParams g;  // x_mode-1 fields (comm, seq, res_in, res_out, gain, eps, M, K = H)
  void* xn;      // [M][H]
  int ts_cols;   // > 0: a two-shot site (slices of ts_cols columns, see comm.cuh)
};

// Vector form (H a multiple of the 16-byte vector, at most kArRowVecs
// vectors per thread): row m on CTA m % grid, the same on every rank, which
// the two-shot all-gather relies on (CTA b waits only for CTA b of each rank).
template <typename T>
__global__ void __launch_bounds__(kArRowThreads) consume_rows_vec_kernel(const ConsumeRowsParams cp) {
  __shared__ float red[32];
  pdl_launch();
  pdl_wait();
  const GemvParams& p = cp.g;
  const Comm& c = p.comm;
  const uint32_t seq = resolve_seq(c, p.in_seq);
  if (!wait_peers(c, p.in_chan, seq, p.in_nprod)) return;
  const int par = seq & 1;
  const int H = p.K;
  const int ts = c.world > 1 ? cp.ts_cols : 0;
  if (ts > 0) {
    for (int m = blockIdx.x; m < p.M; m += gridDim.x) ar_reduce_slice<T>(c, p.in_chan, par, ts, m, H);
    signal_peers_at(c, p.in_chan, seq, kAgCta + blockIdx.x);
    if (!wait_peers_cta(c, p.in_chan, seq, kAgCta + blockIdx.x)) return;
  }
  for (int m = blockIdx.x; m < p.M; m += gridDim.x)
    ar_finish_row<T>(c, p.in_chan, par, ts, nullptr, m, H, static_cast<const T*>(p.ar_bias),
                     p.has_res ? static_cast<const T*>(p.res_in) : nullptr, static_cast<T*>(p.res_out),
                     static_cast<const T*>(p.gain), p.eps, static_cast<T*>(cp.xn), red);
}

// Scalar form (any H; one-shot sites only).
template <typename T>
__global__ void __launch_bounds__(256) consume_rows_kernel(const ConsumeRowsParams cp) {
  __shared__ float red[32];
  pdl_launch();
  pdl_wait();
  const GemvParams& p = cp.g;
  const Comm& c = p.comm;
  const uint32_t seq = resolve_seq(c, p.in_seq);
  if (!wait_peers(c, p.in_chan, seq, p.in_nprod)) return;
  const int par = seq & 1;
  const int H = p.K;
  const T* gain = static_cast<const T*>(p.gain);
  T* xn = static_cast<T*>(cp.xn);
  for (int m = blockIdx.x; m < p.M; m += gridDim.x) {
    float ss = 0.f;
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
      const size_t off = size_t(m) * H + j;
      float s = 0.f;
      for (int r = 0; r < c.world; ++r) s += to_f(__ldcg(reinterpret_cast<const T*>(c.data(c.rank, p.in_chan, par, r)) + off));
      float o = round_t<T>(s);
      if (p.ar_bias) o = round_t<T>(o + to_f(static_cast<const T*>(p.ar_bias)[j]));
      float x = o;
      if (p.has_res) x = round_t<T>(to_f(static_cast<const T*>(p.res_in)[off]) + o);
      static_cast<T*>(p.res_out)[off] = from_f<T>(x);
      ss += x * x;
    }
    const float tot = block_sum(ss, red);
    const float rinv = rsqrtf(tot / float(H) + p.eps);
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
      const size_t off = size_t(m) * H + j;
      const float x = to_f(static_cast<const T*>(p.res_out)[off]);
      xn[off] = from_f<T>(__fmul_rn(__fmul_rn(x, rinv), to_f(gain[j])));
    }
    __syncthreads();
  }
}

int consume_rows_run(int dtype, const ConsumeRowsParams& cp, cudaStream_t st) {
  const int grid = std::max(1, std::min(cp.g.M, sm_count() * 2));
  const bool vec = dtype == MTPB_BF16 ? ar_rows_vec_ok<bf16>(cp.g.K) : ar_rows_vec_ok<float>(cp.g.K);
  if (cp.ts_cols > 0 && (!vec || grid > kAgCta)) return fail(MTPB_ERR_INVALID, "two-shot site: unsupported row shape");
  if (dtype == MTPB_BF16)
    return vec ? launch(consume_rows_vec_kernel<bf16>, dim3(grid), dim3(kArRowThreads), 0, st, cp)
               : launch(consume_rows_kernel<bf16>, dim3(grid), dim3(256), 0, st, cp);
  if (dtype == MTPB_F32)
    return vec ? launch(consume_rows_vec_kernel<float>, dim3(grid), dim3(kArRowThreads), 0, st, cp)
               : launch(consume_rows_kernel<float>, dim3(grid), dim3(256), 0, st, cp);
  return fail(MTPB_ERR_INVALID, "unsupported dtype");
}

// ------------------------------------------------------------------ model
struct ModelHost {
  mtpb_model_desc d;
  std::vector<mtpb_layer_desc> layers;
  CommHost* comm = nullptr;
  int reserved_rows = 0;
  char* scratch = nullptr;
  size_t scratch_bytes = 0;
  void* q = nullptr;
  void* attn = nullptr;
  void* act = nullptr;
  void* res[2] = {nullptr, nullptr};
  void* xn = nullptr;
  void* logits = nullptr;  // [64][V_local] scratch for decode steps without a logits output
  long long* best = nullptr;
  AttnScratch ascr;
  // decode megakernel state
  MkLayer* mk_layers = nullptr;  // device copy of the per-layer pointers (+ KV caches)
  std::vector<MkLayer> mk_host;  // what mk_layers currently holds
  char* mk_scratch = nullptr;
  size_t mk_bytes = 0;
};

int g_decode_impl = 0;  // 0: megakernel when the shape allows it, 1: kernel chain
unsigned long long* g_mk_trace = nullptr;  // stage timeline buffer of the megakernel (device)
int g_mk_slot_kb = 0, g_mk_lm_kb = 0, g_mk_l2hint = 1, g_mk_l2ahead = 1;  // chunk caps 0: automatic
uint32_t g_mk_spin_ns = 0;

bool capturing(cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cs);
  return cs != cudaStreamCaptureStatusNone;
}

int model_reserve(ModelHost& mh, int rows, cudaStream_t st) {
  if (rows <= mh.reserved_rows) return MTPB_OK;
  if (capturing(st)) return fail(MTPB_ERR_INVALID, "model scratch must be reserved before graph capture");
  const mtpb_model_desc& d = mh.d;
  const size_t es = dsize(d.dtype);
  const size_t qb = size_t(rows) * d.hq_local * d.head_dim * es;
  const size_t ab = size_t(rows) * d.inter_local * es;
  const size_t hb = size_t(rows) * d.hidden * es;
  const size_t lb = size_t(64) * size_t(d.vocab_end - d.vocab_start) * es;
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t total = up(qb) * 2 + up(ab) + up(hb) * 3 + up(lb) + 64 * 8;
  cudaFree(mh.scratch);
  mh.scratch = nullptr;
  MTPB_CUDA(cudaMalloc(&mh.scratch, total));
  char* p = mh.scratch;
  mh.q = p; p += up(qb);
  mh.attn = p; p += up(qb);
  mh.act = p; p += up(ab);
  mh.res[0] = p; p += up(hb);
  mh.res[1] = p; p += up(hb);
  mh.xn = p; p += up(hb);
  mh.logits = p; p += up(lb);
  mh.best = reinterpret_cast<long long*>(p);
  std::vector<long long> init(64, kArgmaxEmpty);
  MTPB_CUDA(cudaMemcpy(mh.best, init.data(), 64 * 8, cudaMemcpyHostToDevice));
  mh.scratch_bytes = total;
  mh.reserved_rows = rows;
  return MTPB_OK;
}

struct FwdArgs {
  const long long* ids;  // embedding input [M]
  int B, T;
  const long long* rope_pos;
  int cache_len;        // slot of token 0 (when pos_ptr is null)
  int* pos_ptr;         // device slot of token 0 (decode step)
  void* const* kc;
  void* const* vc;
  int cap;
  void* logits;
  int last_only;
  bool decode;          // distributed argmax + token write + position advance
  long long* tok_out;
  long long* out_ids;
  int ld_out;
};

// One forward over tokens [t0, t0 + tc) of every batch row (a chunk of the
// caller's T tokens). Every collective payload is B * tc * H elements, which
// the caller sized to fit one communicator slot.
template <typename T>
int model_chunk_t(ModelHost& mh, const FwdArgs& a, int t0, int tc, bool last_chunk, cudaStream_t st) {
  const mtpb_model_desc& d = mh.d;
  const Comm& comm = mh.comm->dev;
  const int L = d.n_layers, H = d.hidden, hd = d.head_dim;
  const int hq = d.hq_local, hkv = d.hkv_local;
  const int M = a.B * tc;
  const int qrows = (hq + 2 * hkv) * hd;
  const int vloc = int(d.vocab_end - d.vocab_start);
  const uint32_t nsite = uint32_t(2 * L + 2);
  const bool chunked = tc != a.T;
  // decode steps of many rows take the tensor cores, which read x from global
  // memory: no fused consume prologue for them
  const bool tc_decode = a.decode && d.dtype == MTPB_BF16 && M >= g_tc_min_rows_decode;
  const bool fused_x = size_t(M) * H * sizeof(T) <= kXsStageMax && tc == 1 && !tc_decode;
  // sites consumed by the separate pass may take the two-shot form
  const int ts = fused_x ? 0 : ts_cols_for(size_t(M) * H * sizeof(T), H, comm.world, d.dtype);
  const int chan = 0;
  const int pos_base = a.cache_len + t0;
  const long long* rope_pos = a.rope_pos ? a.rope_pos + t0 : nullptr;

  // embedding -> site 0 (opens a new step of channel 0)
  const int egrid = std::max(1, std::min(M, 64));
  {
    EmbedParams e;
    std::memset(&e, 0, sizeof(e));
    e.ids = a.ids;
    if (chunked) {
      e.ids_tpr = tc;
      e.ids_T = a.T;
      e.ids_t0 = t0;
    }
    e.table = d.embed;
    e.M = M;
    e.H = H;
    e.vstart = d.vocab_start;
    e.vend = d.vocab_end;
    e.vtotal = d.vocab_size;
    e.comm = comm;
    e.chan = chan;
    e.seq = SeqRef{0u, nsite, 0u};
    e.advance_step = 1;
    MTPB_TRY(embed_run(d.dtype, e, egrid, st));
  }
  int nprod = egrid;
  int cur = 0;  // residual ping-pong index holding the current residual
  bool has_res = false;

  auto consume_into = [&](GemvParams& g, uint32_t site, const void* gain) {
    g.comm = comm;
    g.in_seq = SeqRef{site, nsite, 0u};
    g.in_chan = chan;
    g.in_nprod = nprod;
    g.res_in = has_res ? mh.res[cur] : nullptr;
    g.res_out = mh.res[has_res ? 1 - cur : cur];
    g.gain = gain;
    g.eps = d.eps;
    g.has_res = has_res ? 1 : 0;
  };
  auto after_consume = [&]() {
    if (has_res) cur = 1 - cur;
    has_res = true;
  };
  // consume site `site` + RMSNorm, either fused into the GEMV `g` (x in
  // shared memory) or as a separate pass that writes mh.xn
  auto prepare_input = [&](GemvParams& g, uint32_t site, const void* gain, bool allow_fused) -> int {
    consume_into(g, site, gain);
    if (fused_x && allow_fused) {
      g.x_mode = 1;
    } else {
      ConsumeRowsParams cp;
      cp.g = g;
      cp.g.M = M;
      cp.g.K = H;
      cp.xn = mh.xn;
      cp.ts_cols = ts;
      MTPB_TRY(consume_rows_run(d.dtype, cp, st));
      g.x_mode = 0;
      g.x = mh.xn;
      g.ldx = H;
    }
    after_consume();
    return MTPB_OK;
  };

  for (int l = 0; l < L; ++l) {
    const mtpb_layer_desc& ly = mh.layers[l];
    // fused QKV + RoPE + KV append, consuming site 2l (embedding or previous down)
    {
      GemvParams g = gemv_base(ly.qkv_w, ly.qkv_b, M, qrows, H, qrows / 2);
      g.decode = a.decode ? 1 : 0;
      MTPB_TRY(prepare_input(g, uint32_t(2 * l), ly.ln1, true));
      g.y = mh.q;
      g.ldy = hq * hd;
      g.cos_tab = d.cos_tab;
      g.sin_tab = d.sin_tab;
      g.rope_len = d.rope_len;
      g.hd = hd;
      g.hq = hq;
      g.hkv = hkv;
      g.k_cache = a.kc[l];
      g.v_cache = a.vc[l];
      g.kv_cap = a.cap;
      g.tpr = tc;
      g.pos_ptr = a.pos_ptr;
      g.pos_base = pos_base;
      g.rope_pos = rope_pos;
      MTPB_TRY(gemv_dispatch<kEpiRope>(d.dtype, g, st));
    }
    // attention over the cache
    MTPB_TRY(attn_run(d.dtype, mh.q, a.kc[l], a.vc[l], mh.attn, a.B, tc, hq, hkv, hd, a.cap, a.pos_ptr,
                      pos_base, mh.ascr, comm.status(), st));
    // o_proj partial -> push site 2l+1
    {
      GemvParams g = gemv_base(ly.o_w, nullptr, M, H, hq * hd, H);
      g.decode = a.decode ? 1 : 0;
      g.x = mh.attn;
      g.ldx = hq * hd;
      g.comm = comm;
      g.out_seq = SeqRef{uint32_t(2 * l + 1), nsite, 0u};
      g.out_chan = chan;
      g.ts_cols = ts;
      MTPB_TRY(gemv_dispatch<kEpiPush>(d.dtype, g, st));
      nprod = push_grid(d.dtype, g);
    }
    // gate/up + SwiGLU, consuming site 2l+1
    {
      GemvParams g = gemv_base(ly.gu_w, nullptr, M, 2 * d.inter_local, H, d.inter_local);
      g.decode = a.decode ? 1 : 0;
      MTPB_TRY(prepare_input(g, uint32_t(2 * l + 1), ly.ln2, true));
      g.y = mh.act;
      g.ldy = d.inter_local;
      MTPB_TRY(gemv_dispatch<kEpiSwiglu>(d.dtype, g, st));
    }
    // down partial -> push site 2l+2
    {
      GemvParams g = gemv_base(ly.down_w, nullptr, M, H, d.inter_local, H);
      g.decode = a.decode ? 1 : 0;
      g.x = mh.act;
      g.ldx = d.inter_local;
      g.comm = comm;
      g.out_seq = SeqRef{uint32_t(2 * l + 2), nsite, 0u};
      g.out_chan = chan;
      g.ts_cols = ts;
      MTPB_TRY(gemv_dispatch<kEpiPush>(d.dtype, g, st));
      nprod = push_grid(d.dtype, g);
    }
  }

  // final norm + LM head, consuming site 2L. With last_only, only the last
  // chunk computes logits, and only for the last token of each batch row.
  if (a.last_only && !last_chunk) return MTPB_OK;
  {
    const int rows = a.last_only ? a.B : M;
    GemvParams g = gemv_base(d.lm_head, nullptr, rows, vloc, H, vloc);
    g.decode = a.decode ? 1 : 0;
    const bool direct = fused_x && rows == M;
    MTPB_TRY(prepare_input(g, uint32_t(2 * L), d.final_norm, direct));
    if (!direct && a.last_only) {
      g.x = static_cast<const char*>(mh.xn) + size_t(tc - 1) * H * sizeof(T);
      g.ldx = tc * H;
    }
    g.y = a.logits ? a.logits : mh.logits;
    g.ldy = vloc;
    if (!a.last_only && chunked) {
      g.tpr = tc;
      g.out_T = a.T;
      g.out_t0 = t0;
    }
    if (a.decode) {
      g.best = mh.best;
      g.vocab_start = uint32_t(d.vocab_start);
      g.nan_wins = comm.world == 1 ? 1 : 0;
      MTPB_TRY(gemv_dispatch<kEpiArgmax>(d.dtype, g, st));
    } else {
      if (!a.logits) return fail(MTPB_ERR_INVALID, "forward: logits output required");
      MTPB_TRY(gemv_dispatch<kEpiStore>(d.dtype, g, st));
    }
  }

  if (a.decode) {
    ArgmaxFinishParams f;
    std::memset(&f, 0, sizeof(f));
    f.best = mh.best;
    f.M = a.B;
    f.comm = comm;
    f.chan = chan;
    f.seq = SeqRef{uint32_t(2 * L + 1), nsite, 0u};
    f.tok_out = a.tok_out;
    f.out_ids = a.out_ids;
    f.ld_out = a.ld_out;
    f.pos_ptr = a.pos_ptr;
    MTPB_TRY(launch(argmax_finish_kernel, dim3(1), dim3(64), 0, st, f));
  }
  return MTPB_OK;
}

template <typename T>
int model_forward_t(ModelHost& mh, const FwdArgs& a, cudaStream_t st) {
  const mtpb_model_desc& d = mh.d;
  const Comm& comm = mh.comm->dev;
  if (a.cap > 0 && !a.pos_ptr && a.cache_len + a.T > a.cap) return fail(MTPB_ERR_INVALID, "KV cache overflow");
  const size_t row_bytes = size_t(a.B) * d.hidden * sizeof(T);
  if (row_bytes > comm.slot_bytes)
    return fail(MTPB_ERR_INVALID, "forward: batch x hidden exceeds the communicator slot");
  if (a.decode && (a.T != 1 || a.B > 64)) return fail(MTPB_ERR_INVALID, "decode step: T == 1 and B <= 64");
  const int tc = int(std::min<size_t>(size_t(a.T), comm.slot_bytes / row_bytes));
  MTPB_TRY(model_reserve(mh, a.B * tc, st));
  for (int t0 = 0; t0 < a.T; t0 += tc) {
    const int n = std::min(tc, a.T - t0);
    MTPB_TRY(model_chunk_t<T>(mh, a, t0, n, t0 + n == a.T, st));
  }
  return MTPB_OK;
}

// ------------------------------------------------------------------ decode megakernel
constexpr int kNotEligible = 1;

// Row tile of the megakernel instantiation that serves M batch rows.
int mk_row_tile(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

int smem_optin() {
  int dev = 0, v = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return v > 0 ? v : 227 * 1024;
}

// Device scratch of the megakernel (LL words), sized for the largest batch.
struct MkScratch {
  size_t qkv, att, head, act, lm, total;
};

MkScratch mk_scratch_layout(const mtpb_model_desc& d) {
  const int P = d.dtype == MTPB_BF16 ? 2 : 1;
  const size_t nq = size_t(d.hq_local + 2 * d.hkv_local) * d.head_dim;
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  MkScratch s;
  s.qkv = up(size_t(kMkMaxM) * (nq / P) * 8);
  s.att = up(size_t(kMkMaxM) * d.hq_local * kMkMaxSplits * (d.head_dim + 2) * 8);
  s.head = up(size_t(kMkRep) * kMkMaxM * (size_t(d.hq_local) * d.head_dim / P) * 8);
  s.act = up(size_t(kMkRep) * kMkMaxM * (d.inter_local / P) * 8);
  s.lm = up(size_t(kMaxCtas) * kMkMaxM * 16);
  s.total = s.qkv + s.att + s.head + s.act + s.lm;
  return s;
}

// Fill the shape / scratch part of the megakernel parameters; returns
// kNotEligible when this model or batch does not fit the megakernel.
int mk_plan(ModelHost& mh, int M, int cap, MkParams& p, size_t* smem_out) {
  const mtpb_model_desc& d = mh.d;
  const size_t tsz = dsize(d.dtype);
  const int VE = vec_elems(d.dtype);
  const int P = d.dtype == MTPB_BF16 ? 2 : 1;
  const int hd = d.head_dim;
  if (M < 1 || M > kMkMaxM) return kNotEligible;
  if (!mk_has_variant(d.dtype == MTPB_BF16, mk_row_tile(M), d.head_dim)) return kNotEligible;
  // head_dim: a power of two in [16, 128] (lane-rotated 16-byte chunks)
  if (hd < 16 || hd > 128 || (hd & (hd - 1)) || d.hq_local % d.hkv_local) return kNotEligible;
  // 16-byte weight rows, and rows of whole LL pairs
  if (d.hidden % VE || d.inter_local % VE || (d.hq_local * hd) % VE) return kNotEligible;
  if (d.hidden % (2 * P) || d.inter_local % (2 * P)) return kNotEligible;
  const int G = sm_count();
  if (G > kMaxCtas) return kNotEligible;
  const int ns = (cap + kMkSplit - 1) / kMkSplit;
  if (ns < 1 || ns > kMkMaxSplits) return kNotEligible;
  // AllReduce-site words of one batch must fit a communicator slot
  if (size_t(M) * (d.hidden / P) * 8 > mh.comm->dev.slot_bytes) return kNotEligible;
  std::memset(&p, 0, sizeof(p));
  p.L = d.n_layers;
  p.H = d.hidden;
  p.I = d.inter_local;
  p.hq = d.hq_local;
  p.hkv = d.hkv_local;
  p.hd = hd;
  p.M = M;
  p.kv_cap = cap;
  p.nsplit = ns;
  p.xin_cols = std::max(d.hq_local * hd, d.inter_local);
  p.wsc_floats = kMkCons * 3 * hd;
  // the QKV bias of a CTA's units is kept in shared memory
  if (((d.hq_local + 2 * d.hkv_local) * hd / P + G - 1) / G * P > kMkBiasMax) return kNotEligible;
  // every attention item of a CTA is staged in shared memory
  const int per_cta = (M * d.hq_local * ns + G - 1) / G;
  if (per_cta > kMkMaxStage) return kNotEligible;
  p.att_stage = per_cta;
  // stage kinds: units, their split over the CTAs, chunking
  const size_t nq = size_t(d.hq_local + 2 * d.hkv_local) * hd;
  const size_t hvec = mk_align(size_t(d.hidden) * tsz);
  struct KindShape {
    int K, units, rpu, halves, hoff;
    size_t pre;
  };
  // LM head: kMkLmRows rows a quarter of the shard apart per unit when they divide it
  const int vloc = int(d.vocab_end - d.vocab_start);
  const int lmq = vloc % kMkLmRows == 0 ? kMkLmRows : 1;
  const KindShape ks[kMkKinds] = {
      {d.hidden, int(nq) / P, P, 1, 0, hvec + mk_align(nq * tsz)},  // QKV (+ ln1, bias)
      {d.hq_local * hd, d.hidden / P, P, 1, 0, 0},                  // O
      {d.hidden, d.inter_local / P, P, 2, d.inter_local, hvec},     // gate/up (+ ln2)
      {d.inter_local, d.hidden / P, P, 1, 0, 0},                    // down
      {d.hidden, vloc / lmq, 1, lmq, vloc / lmq, hvec},            // LM head (+ final norm)
  };
  // the ring takes the rest of shared memory and must hold the biggest
  // chunk: the layer chunk cap shrinks (16 KiB steps) until it does
  const int budget = smem_optin() - 4096;  // static shared memory of the kernel
  p.ring_bytes = 0;
  const size_t fixed = mk_layout(p, tsz).ring;
  // Chunk caps. The ring is what is left of shared memory. A stage whose
  // weights per CTA are many ring-fulls is bound by the weight stream: its
  // chunks take half the ring, so one lands while the other is consumed (the
  // LM head always; a layer when its bytes per CTA exceed two rings).
  // Otherwise a layer streams in chunks of 96 KiB for one row when the ring
  // holds two (the next layer's gate/up lands while this layer's down is
  // consumed), else 128 KiB. Set values override the automatic ones.
  const size_t ring_est = size_t(budget) > fixed ? size_t(budget) - fixed : 0;
  const size_t half_ring = std::max<size_t>(16 * 1024, (ring_est / 2) & ~size_t(16 * 1024 - 1));
  size_t layer_bytes = 0;  // weight bytes of one layer per CTA
  for (int k = 0; k < kMkLm; ++k)
    layer_bytes += (size_t(ks[k].units) + G - 1) / G * ks[k].halves * ks[k].rpu * size_t(ks[k].K) * tsz;
  size_t chunk_max = size_t(g_mk_slot_kb) * 1024;
  if (g_mk_slot_kb == 0) {
    if (layer_bytes > 2 * ring_est)
      chunk_max = std::min<size_t>(128 * 1024, half_ring);
    else
      chunk_max = (M == 1 && ring_est > 176 * 1024) ? 96 * 1024 : 128 * 1024;
  }
  const size_t lm_max = g_mk_lm_kb > 0 ? size_t(g_mk_lm_kb) * 1024 : std::min<size_t>(96 * 1024, half_ring);
  size_t biggest = 0;
  for (size_t cap = chunk_max;; cap -= 16 * 1024) {
    biggest = 0;
    for (int k = 0; k < kMkKinds; ++k) {
      MkKind& kd = p.kinds[k];
      kd.K = ks[k].K;
      kd.rpu = ks[k].rpu;
      kd.halves = ks[k].halves;
      kd.hoff = ks[k].hoff;
      kd.base = ks[k].units / G;
      kd.rem = ks[k].units % G;
      kd.pre = int(ks[k].pre);
      const size_t ub = size_t(kd.halves) * kd.rpu * kd.K * tsz;
      // the LM head streams in smaller chunks: more of them in flight
      const size_t cmax = k == kMkLm ? std::min(cap, lm_max) : cap;
      const size_t room = cmax > ks[k].pre ? cmax - ks[k].pre : 0;
      kd.upc = int(std::max<size_t>(1, room / ub));
      biggest = std::max(biggest, ks[k].pre + size_t(kd.upc) * ub);
    }
    if (fixed + biggest <= size_t(budget)) break;
    if (cap <= 16 * 1024) return kNotEligible;
  }
  p.ring_bytes = int((size_t(budget) - fixed) & ~size_t(127));
  p.l2_hint = g_mk_l2hint;
  // the next layer's rows go into L2 ahead of time only when a layer's weights
  // of this rank fit in well under half the L2 (126 MB): larger layers would
  // evict what the current one still needs
  p.l2_ahead = g_mk_l2ahead && layer_bytes * size_t(G) <= (48u << 20);
  *smem_out = mk_layout(p, tsz).total;
  const MkScratch sl = mk_scratch_layout(d);
  if (mh.mk_bytes < sl.total) return kNotEligible;  // reserved by mk_reserve
  char* s = mh.mk_scratch;
  p.qkv_ll = reinterpret_cast<uint64_t*>(s);
  p.att_ll = reinterpret_cast<uint64_t*>(s + sl.qkv);
  p.head_ll = reinterpret_cast<uint64_t*>(s + sl.qkv + sl.att);
  p.act_ll = reinterpret_cast<uint64_t*>(s + sl.qkv + sl.att + sl.head);
  p.lm_ll = reinterpret_cast<uint64_t*>(s + sl.qkv + sl.att + sl.head + sl.act);
  return MTPB_OK;
}

int mk_reserve(ModelHost& mh) {
  if (mh.mk_scratch) return MTPB_OK;
  const mtpb_model_desc& d = mh.d;
  const size_t total = mk_scratch_layout(d).total;
  MTPB_CUDA(cudaMalloc(&mh.mk_scratch, total));
  // zero words carry sequence number 0, which no step uses
  MTPB_CUDA(cudaMemset(mh.mk_scratch, 0, total));
  MTPB_CUDA(cudaMalloc(&mh.mk_layers, sizeof(MkLayer) * d.n_layers));
  mh.mk_bytes = total;
  return MTPB_OK;
}


// One decode step through the megakernel; kNotEligible when it cannot run it.
int mk_decode(ModelHost& mh, const FwdArgs& a, cudaStream_t st) {
  if (g_decode_impl != 0 || !a.decode || a.T != 1) return kNotEligible;
  const mtpb_model_desc& d = mh.d;
  if (!capturing(st)) MTPB_TRY(mk_reserve(mh));
  if (!mh.mk_scratch) return kNotEligible;
  MkParams p;
  size_t smem = 0;
  if (mk_plan(mh, a.B, a.cap, p, &smem) != MTPB_OK) return kNotEligible;
  // per-layer pointers (weights + this call's KV caches), uploaded when they change
  std::vector<MkLayer> want(d.n_layers);
  for (int l = 0; l < d.n_layers; ++l) {
    const mtpb_layer_desc& ly = mh.layers[l];
    want[l] = MkLayer{ly.ln1, ly.qkv_w, ly.qkv_b, ly.o_w, ly.ln2, ly.gu_w, ly.down_w, a.kc[l], a.vc[l]};
  }
  if (want.size() != mh.mk_host.size() ||
      std::memcmp(want.data(), mh.mk_host.data(), sizeof(MkLayer) * want.size()) != 0) {
    if (capturing(st)) return fail(MTPB_ERR_INVALID, "decode step: KV caches changed during graph capture");
    MTPB_CUDA(cudaMemcpy(mh.mk_layers, want.data(), sizeof(MkLayer) * want.size(), cudaMemcpyHostToDevice));
    mh.mk_host = want;
  }
  p.comm = mh.comm->dev;
  p.layers = mh.mk_layers;
  p.vstart = d.vocab_start;
  p.vend = d.vocab_end;
  p.vocab = d.vocab_size;
  p.embed = d.embed;
  p.lm_head = d.lm_head;
  p.final_norm = d.final_norm;
  p.cos_tab = d.cos_tab;
  p.sin_tab = d.sin_tab;
  p.rope_len = d.rope_len;
  p.eps = d.eps;
  p.scale = 1.0f / std::sqrt(float(d.head_dim));
  p.pos_ptr = a.pos_ptr;
  p.tok = a.tok_out;
  p.out_ids = a.out_ids;
  p.ld_out = a.ld_out;
  p.logits = a.logits;
  p.budget_ns = mh.comm->dev.timeout_ns;
  p.spin_ns = g_mk_spin_ns;
  p.trace = g_mk_trace;
  const int MT = mk_row_tile(a.B);
  cudaError_t err = cudaSuccess;
  const int r = d.dtype == MTPB_BF16 ? mk_launch_bf16(MT, d.head_dim, p, sm_count(), smem, st, &err)
                                     : mk_launch_f32(MT, d.head_dim, p, sm_count(), smem, st, &err);
  switch (r) {
    case kMkLaunchOk: return MTPB_OK;
    case kMkLaunchNoVariant: return kNotEligible;
    case kMkLaunchCapture: return fail(MTPB_ERR_INVALID, "decode step: run one step eagerly before graph capture");
    default: return fail_cuda(err, "decode megakernel launch");
  }
}

int model_forward(ModelHost& mh, const FwdArgs& a, cudaStream_t st) {
  if (a.decode) {
    const int r = mk_decode(mh, a, st);
    if (r != kNotEligible) return r;
  }
  if (mh.d.dtype == MTPB_BF16) return model_forward_t<bf16>(mh, a, st);
  if (mh.d.dtype == MTPB_F32) return model_forward_t<float>(mh, a, st);
  return fail(MTPB_ERR_INVALID, "unsupported dtype");
}

}  // namespace

// =====================================================================
// extern "C"
// =====================================================================
// Bumped by every mtpb_set_* call: a CUDA graph captured over the library
// bakes in the settings of its capture, so holders of a graph compare epochs.
std::atomic<uint64_t> g_settings_epoch{0};

extern "C" {

const char* mtpb_last_error(void) { return g_err.c_str(); }
int mtpb_version(void) { return 1; }
int mtpb_set_pdl(int enable) {
  g_settings_epoch.fetch_add(1);
  g_pdl = enable != 0;
  return MTPB_OK;
}
int mtpb_set_prefetch_cap(uint32_t bytes) {
  g_settings_epoch.fetch_add(1);
  g_prefetch_cap = bytes;
  return MTPB_OK;
}
int mtpb_set_gemv_ctas_per_sm(int n) {
  g_settings_epoch.fetch_add(1);
  if (n < 1 || n > 8) return fail(MTPB_ERR_INVALID, "gemv CTAs per SM must be in [1, 8]");
  g_gemv_ctas_per_sm = n;
  return MTPB_OK;
}

int mtpb_comm_create(int rank, int world, uint64_t slot_bytes, void** out) {
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return fail(MTPB_ERR_INVALID, "comm: need 1 <= world <= 8 and 0 <= rank < world");
  if (slot_bytes % 256 != 0 || slot_bytes == 0) return fail(MTPB_ERR_INVALID, "comm: slot_bytes must be a positive multiple of 256");
  auto* c = new CommHost();
  std::memset(&c->dev, 0, sizeof(c->dev));
  c->dev.rank = rank;
  c->dev.world = world;
  c->dev.slot_bytes = slot_bytes;
  c->dev.timeout_ns = 5ull * 1000 * 1000 * 1000;
  cudaGetDevice(&c->device);
  const size_t bytes = Comm::buffer_bytes(slot_bytes, world);
  cudaError_t e = cudaMalloc(&c->local, bytes);
  if (e != cudaSuccess) {
    delete c;
    return fail_cuda(e, "cudaMalloc(comm buffer)");
  }
  e = cudaMemset(c->local, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(c->local);
    delete c;
    return fail_cuda(e, "cudaMemset(comm buffer)");
  }
  c->dev.base[rank] = static_cast<char*>(c->local);
  c->open = world == 1;
  *out = c;
  return MTPB_OK;
}

int mtpb_comm_ipc_handle(void* comm, void* handle_out) {
  if (!comm || !handle_out) return fail(MTPB_ERR_INVALID, "comm_ipc_handle: null argument");
  auto* c = static_cast<CommHost*>(comm);
  cudaIpcMemHandle_t h;
  MTPB_CUDA(cudaIpcGetMemHandle(&h, c->local));
  static_assert(sizeof(h) == 64, "IPC handle size");
  std::memcpy(handle_out, &h, 64);
  return MTPB_OK;
}

int mtpb_comm_open(void* comm, const void* handles) {
  if (!comm || !handles) return fail(MTPB_ERR_INVALID, "comm_open: null argument");
  auto* c = static_cast<CommHost*>(comm);
  if (c->open) return MTPB_OK;
  for (int r = 0; r < c->dev.world; ++r) {
    if (r == c->dev.rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(handles) + 64 * r, 64);
    void* p = nullptr;
    MTPB_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    c->mapped[r] = p;
    c->dev.base[r] = static_cast<char*>(p);
  }
  c->open = true;
  return MTPB_OK;
}

int mtpb_comm_destroy(void* comm) {
  if (!comm) return MTPB_OK;
  auto* c = static_cast<CommHost*>(comm);
  for (int r = 0; r < kMaxRanks; ++r)
    if (c->mapped[r]) cudaIpcCloseMemHandle(c->mapped[r]);
  cudaFree(c->local);
  delete c;
  return MTPB_OK;
}

int mtpb_comm_set_timeout(void* comm, uint64_t ns) {
  if (!comm) return fail(MTPB_ERR_INVALID, "comm_set_timeout: null comm");
  static_cast<CommHost*>(comm)->dev.timeout_ns = ns;
  return MTPB_OK;
}

int mtpb_comm_status(void* comm, uint32_t* out) {
  CommHost* c = as_comm(comm);
  if (!c || !out) return fail(MTPB_ERR_INVALID, "comm_status: null argument");
  MTPB_CUDA(cudaDeviceSynchronize());
  MTPB_CUDA(cudaMemcpy(out, c->dev.ctl() + kCtlStatus, 4, cudaMemcpyDeviceToHost));
  return MTPB_OK;
}

int mtpb_comm_clear_status(void* comm) {
  CommHost* c = as_comm(comm);
  if (!c) return fail(MTPB_ERR_INVALID, "comm_clear_status: no communicator");
  MTPB_CUDA(cudaMemset(c->dev.ctl() + kCtlStatus, 0, 4));
  return MTPB_OK;
}

int* mtpb_comm_pos_ptr(void* comm) {
  CommHost* c = as_comm(comm);
  return c ? reinterpret_cast<int*>(c->dev.ctl() + kCtlPos) : nullptr;
}

int mtpb_comm_set_pos(void* comm, int pos, void* stream) {
  CommHost* c = as_comm(comm);
  if (!c) return fail(MTPB_ERR_INVALID, "comm_set_pos: no communicator");
  int* p = reinterpret_cast<int*>(c->dev.ctl() + kCtlPos);
  return launch(set_i32_kernel, dim3(1), dim3(1), 0, static_cast<cudaStream_t>(stream), SetI32{p, pos});
}

int mtpb_comm_pingpong(void* comm, int peer, int iters, int warm, unsigned long long* ns_out, void* stream) {
  CommHost* c = as_comm(comm);
  if (!c || !c->open) return fail(MTPB_ERR_INVALID, "pingpong: communicator not open");
  if (peer < 0 || peer >= c->dev.world || peer == c->dev.rank)
    return fail(MTPB_ERR_INVALID, "pingpong: peer must be another rank of the communicator");
  if (iters <= 0 || warm < 0 || warm >= iters || iters > (1 << 20))
    return fail(MTPB_ERR_INVALID, "pingpong: need 0 <= warm < iters <= 2^20");
  if (!ns_out) return fail(MTPB_ERR_INVALID, "pingpong: null output");
  PingParams p;
  p.comm = c->dev;
  p.peer = peer;
  p.iters = iters;
  p.warm = warm;
  // both ranks count their calls alike, so they agree on the base; 2^31 and
  // above, with room for 2^20 round trips per call
  p.base = 0x80000000u + (c->ping_calls++ % 1024u) * (2u << 20);
  p.ns_out = ns_out;
  pingpong_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
  MTPB_CUDA(cudaGetLastError());
  return MTPB_OK;
}

uint64_t mtpb_comm_slot_bytes(void* comm) {
  CommHost* c = as_comm(comm);
  return c ? c->dev.slot_bytes : 0;
}

int mtpb_linear(const void* x, int ldx, const void* w, const void* bias, void* y, int ldy, int M, int N,
                int K, int dtype, void* stream) {
  GemvParams g = gemv_base(w, bias, M, N, K, N);
  g.x = x;
  g.ldx = ldx;
  g.y = y;
  g.ldy = ldy;
  g.comm = as_comm(nullptr)->dev;
  return gemv_dispatch<kEpiStore>(dtype, g, static_cast<cudaStream_t>(stream));
}

int mtpb_linear_swiglu(const void* x, int ldx, const void* w, void* act, int ldact, int M, int I, int K,
                       int dtype, void* stream) {
  GemvParams g = gemv_base(w, nullptr, M, 2 * I, K, I);
  g.x = x;
  g.ldx = ldx;
  g.y = act;
  g.ldy = ldact;
  g.comm = as_comm(nullptr)->dev;
  return gemv_dispatch<kEpiSwiglu>(dtype, g, static_cast<cudaStream_t>(stream));
}

int mtpb_qkv_rope(const void* x, int ldx, const void* w, const void* bias, void* q_out, void* k_cache,
                  void* v_cache, int B, int T, int hq, int hkv, int hd, int K, int cap, int cache_len,
                  const int64_t* rope_pos, const float* cos_tab, const float* sin_tab, int rope_len,
                  int dtype, void* comm, void* stream) {
  if (hd % 2 != 0) return fail(MTPB_ERR_INVALID, "qkv_rope: odd head_dim");
  if (cache_len + T > cap) return fail(MTPB_ERR_INVALID, "KV cache overflow");
  const int N = (hq + 2 * hkv) * hd;
  GemvParams g = gemv_base(w, bias, B * T, N, K, N / 2);
  g.x = x;
  g.ldx = ldx;
  g.y = q_out;
  g.ldy = hq * hd;
  g.comm = as_comm(comm)->dev;
  g.cos_tab = cos_tab;
  g.sin_tab = sin_tab;
  g.rope_len = rope_len;
  g.hd = hd;
  g.hq = hq;
  g.hkv = hkv;
  g.k_cache = k_cache;
  g.v_cache = v_cache;
  g.kv_cap = cap;
  g.tpr = T;
  g.pos_base = cache_len;
  g.rope_pos = reinterpret_cast<const long long*>(rope_pos);
  return gemv_dispatch<kEpiRope>(dtype, g, static_cast<cudaStream_t>(stream));
}

int mtpb_attention(const void* q, const void* k_cache, const void* v_cache, void* out, int B, int T, int hq,
                   int hkv, int hd, int cap, int cache_len, int dtype, void* comm, void* stream) {
  if (cache_len + T > cap) return fail(MTPB_ERR_INVALID, "attention: cache_len + T exceeds the cache capacity");
  return attn_run(dtype, q, k_cache, v_cache, out, B, T, hq, hkv, hd, cap, nullptr, cache_len,
                  standalone_attn_scratch(), as_comm(comm)->dev.status(), static_cast<cudaStream_t>(stream));
}

int mtpb_rmsnorm(const void* x, const void* w, void* y, int rows, int H, float eps, int dtype, void* stream) {
  if (rows <= 0 || H <= 0) return fail(MTPB_ERR_INVALID, "rmsnorm: empty shape");
  const int grid = std::min(rows, sm_count() * 4);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl ? 1 : 0;
  if (dtype == MTPB_BF16) {
    MTPB_CUDA(cudaLaunchKernelEx(&cfg, rmsnorm_kernel<bf16>, x, w, y, rows, H, eps));
  } else if (dtype == MTPB_F32) {
    MTPB_CUDA(cudaLaunchKernelEx(&cfg, rmsnorm_kernel<float>, x, w, y, rows, H, eps));
  } else {
    return fail(MTPB_ERR_INVALID, "unsupported dtype");
  }
  return MTPB_OK;
}

int mtpb_allreduce_residual_rmsnorm(void* comm, const void* partial, const void* residual, const void* gain,
                                    const void* bias, void* out_res, void* out_norm, int rows, int H, float eps,
                                    int dtype, void* stream) {
  CommHost* c = as_comm(comm);
  if (!c || !c->open) return fail(MTPB_ERR_INVALID, "allreduce: communicator not open");
  if (rows <= 0 || H <= 0) return fail(MTPB_ERR_INVALID, "allreduce: empty shape");
  if ((out_norm == nullptr) != (gain == nullptr)) return fail(MTPB_ERR_INVALID, "allreduce: gain and out_norm go together");
  ArNormParams p;
  std::memset(&p, 0, sizeof(p));
  p.partial = partial;
  p.residual = residual;
  p.gain = gain;
  p.bias = bias;
  p.out_res = out_res;
  p.out_norm = out_norm;
  p.rows = rows;
  p.H = H;
  p.eps = eps;
  p.comm = c->dev;
  p.chan = 1;
  const int VE = vec_elems(dtype);
  if (H % VE == 0 && (!aligned16(partial))) return fail(MTPB_ERR_INVALID, "allreduce: partial must be 16-byte aligned");
  return ar_norm_run(dtype, p, static_cast<cudaStream_t>(stream));
}

int mtpb_allreduce(void* comm, void* t, int rows, int H, int dtype, void* stream) {
  return mtpb_allreduce_residual_rmsnorm(comm, t, nullptr, nullptr, nullptr, t, nullptr, rows, H, 0.f, dtype,
                                         stream);
}

int mtpb_embedding(void* comm, const int64_t* ids, const void* table, void* out, int M, int H, int64_t vstart,
                   int64_t vend, int64_t vocab, int dtype, void* stream) {
  CommHost* c = as_comm(comm);
  if (!c || !c->open) return fail(MTPB_ERR_INVALID, "embedding: communicator not open");
  if (M <= 0 || H <= 0) return fail(MTPB_ERR_INVALID, "embedding: empty shape");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int VE = vec_elems(dtype);
  if (H % VE == 0 && (!aligned16(table) || !aligned16(out)))
    return fail(MTPB_ERR_INVALID, "embedding: table and out must be 16-byte aligned");
  EmbedParams e;
  std::memset(&e, 0, sizeof(e));
  e.ids = reinterpret_cast<const long long*>(ids);
  e.table = table;
  e.M = M;
  e.H = H;
  e.vstart = vstart;
  e.vend = vend;
  e.vtotal = vocab;
  e.comm = c->dev;
  if (c->dev.world == 1) {
    e.out = out;
    return embed_run(dtype, e, std::min(M, 1024), st);
  }
  if (size_t(M) * H * dsize(dtype) > c->dev.slot_bytes)
    return fail(MTPB_ERR_INVALID, "embedding: rows x hidden exceed the communicator slot");
  // masked lookup into a local partial, then the one-shot reduce (channel 1)
  e.out = out;
  Comm solo = c->dev;
  solo.world = 1;
  e.comm = solo;
  MTPB_TRY(embed_run(dtype, e, std::min(M, 1024), st));
  return mtpb_allreduce(comm, out, M, H, dtype, stream);
}

int mtpb_argmax(void* comm, const void* logits, int M, int V_local, int64_t ld, int64_t vstart, int64_t* ids_out,
                int64_t* scratch, int dtype, void* stream) {
  CommHost* c = as_comm(comm);
  if (!c || !c->open) return fail(MTPB_ERR_INVALID, "argmax: communicator not open");
  if (M <= 0 || M > 64) return fail(MTPB_ERR_INVALID, "argmax: need 1 <= M <= 64 rows");
  if (V_local <= 0) return fail(MTPB_ERR_INVALID, "argmax: empty vocab shard");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ArgmaxRowsParams a;
  a.logits = logits;
  a.M = M;
  a.V = V_local;
  a.ld = ld;
  a.vstart = uint32_t(vstart);
  a.nan_wins = c->dev.world == 1 ? 1 : 0;
  a.part = reinterpret_cast<long long*>(scratch);
  MTPB_TRY(argmax_rows_run(dtype, a, st));
  ArgmaxFinishParams f;
  std::memset(&f, 0, sizeof(f));
  f.part = reinterpret_cast<const long long*>(scratch);
  f.nsplit = argmax_splits(V_local);
  f.M = M;
  f.comm = c->dev;
  f.chan = 1;
  f.use_coll_counter = 1;
  f.tok_out = reinterpret_cast<long long*>(ids_out);
  return launch(argmax_finish_kernel, dim3(1), dim3(64), 0, st, f);
}

int mtpb_model_create(const mtpb_model_desc* desc, void* comm, void** out) {
  if (!desc || !out) return fail(MTPB_ERR_INVALID, "model_create: null argument");
  CommHost* c = as_comm(comm);
  if (!c || !c->open) return fail(MTPB_ERR_INVALID, "model_create: communicator not open");
  const mtpb_model_desc& d = *desc;
  if (d.n_layers <= 0 || d.hidden <= 0 || d.head_dim <= 0 || d.hq_local <= 0 || d.hkv_local <= 0)
    return fail(MTPB_ERR_INVALID, "model_create: bad dimensions");
  if (d.hq_local % d.hkv_local != 0) return fail(MTPB_ERR_INVALID, "model_create: hq_local % hkv_local != 0");
  if (2 * d.n_layers + 2 > 4096) return fail(MTPB_ERR_INVALID, "model_create: too many layers");
  if (d.vocab_end - d.vocab_start <= 0 || d.vocab_size >= (int64_t(1) << 32))
    return fail(MTPB_ERR_INVALID, "model_create: bad vocab range");
  auto* mh = new ModelHost();
  mh->d = d;
  mh->layers.resize(d.n_layers);
  std::memset(mh->layers.data(), 0, sizeof(mtpb_layer_desc) * d.n_layers);
  mh->comm = c;
  *out = mh;
  return MTPB_OK;
}

int mtpb_model_set_layer(void* model, int layer, const mtpb_layer_desc* desc) {
  if (!model || !desc) return fail(MTPB_ERR_INVALID, "model_set_layer: null argument");
  auto* mh = static_cast<ModelHost*>(model);
  if (layer < 0 || layer >= mh->d.n_layers) return fail(MTPB_ERR_INVALID, "model_set_layer: layer out of range");
  mh->layers[layer] = *desc;
  return MTPB_OK;
}

int mtpb_model_reserve(void* model, int max_rows, int max_cap) {
  if (!model) return fail(MTPB_ERR_INVALID, "model_reserve: null model");
  auto* mh = static_cast<ModelHost*>(model);
  MTPB_TRY(model_reserve(*mh, max_rows, nullptr));
  // attention split scratch for decode rows (T = 1) at this capacity
  const int G = mh->d.hq_local / mh->d.hkv_local;
  int cc = 0;
  const int M = std::min(max_rows, 64);
  const int ns = attn_choose_splits(M, mh->d.hkv_local, G, max_cap, mh->d.head_dim, &cc);
  if (ns > 1) {
    AttnScratch& s = mh->ascr;
    const size_t need_o = size_t(M) * mh->d.hq_local * ns * mh->d.head_dim;
    const size_t need_ml = size_t(M) * mh->d.hq_local * ns * 2, need_c = size_t(M) * mh->d.hkv_local;
    if (need_o > s.o_elems || need_ml > s.ml_elems || need_c > s.ctr_elems) {
      cudaFree(s.part_o);
      cudaFree(s.part_ml);
      cudaFree(s.counters);
      MTPB_CUDA(cudaMalloc(&s.part_o, need_o * 4));
      MTPB_CUDA(cudaMalloc(&s.part_ml, need_ml * 4));
      MTPB_CUDA(cudaMalloc(&s.counters, need_c * 4));
      MTPB_CUDA(cudaMemset(s.counters, 0, need_c * 4));
      s.o_elems = need_o;
      s.ml_elems = need_ml;
      s.ctr_elems = need_c;
    }
  }
  return MTPB_OK;
}

int mtpb_model_destroy(void* model) {
  if (!model) return MTPB_OK;
  auto* mh = static_cast<ModelHost*>(model);
  cudaFree(mh->scratch);
  cudaFree(mh->ascr.part_o);
  cudaFree(mh->ascr.part_ml);
  cudaFree(mh->ascr.counters);
  cudaFree(mh->mk_scratch);
  cudaFree(mh->mk_layers);
  delete mh;
  return MTPB_OK;
}

int mtpb_set_decode_ring(int chunk_kb, int lm_chunk_kb, int l2_flags) {
  g_settings_epoch.fetch_add(1);
  auto bad = [](int kb) { return kb != 0 && (kb < 4 || kb > 200 || kb % 4); };
  if (bad(chunk_kb) || bad(lm_chunk_kb))
    return fail(MTPB_ERR_INVALID, "decode ring: chunk sizes in [4, 200] KiB, multiples of 4, or 0 = automatic");
  if (l2_flags < 0 || l2_flags > 3) return fail(MTPB_ERR_INVALID, "decode ring: l2 flags 0..3");
  g_mk_slot_kb = chunk_kb;
  g_mk_lm_kb = lm_chunk_kb;
  g_mk_l2hint = l2_flags & 1;
  g_mk_l2ahead = (l2_flags >> 1) & 1;
  return MTPB_OK;
}

int mtpb_set_tc_min_rows(int rows) {
  g_settings_epoch.fetch_add(1);
  if (rows < 1) return fail(MTPB_ERR_INVALID, "tensor-core GEMM row threshold must be >= 1");
  g_tc_min_rows = rows;
  return MTPB_OK;
}

int mtpb_set_tc_min_rows_decode(int rows) {
  g_settings_epoch.fetch_add(1);
  if (rows < 1) return fail(MTPB_ERR_INVALID, "tensor-core GEMM row threshold must be >= 1");
  g_tc_min_rows_decode = rows;
  return MTPB_OK;
}

int mtpb_set_allreduce_two_shot(long long min_bytes, int min_world) {
  g_settings_epoch.fetch_add(1);
  if (min_world < 2) return fail(MTPB_ERR_INVALID, "two-shot allreduce: min_world must be >= 2");
  g_ts_min_bytes = min_bytes;
  g_ts_min_world = min_world;
  return MTPB_OK;
}

int mtpb_allreduce_two_shot_cols(long long bytes, int H, int world, int dtype) {
  if (bytes < 0 || H <= 0 || world < 1) return 0;
  return ts_cols_for(size_t(bytes), H, world, dtype);
}

int mtpb_set_tc_split(int max_splits) {
  g_settings_epoch.fetch_add(1);
  if (max_splits < 1 || max_splits > 64) return -1;
  const int prev = g_tc_split_max;
  g_tc_split_max = max_splits;
  return prev;
}

int mtpb_set_tc_pair(int enable) {
  g_settings_epoch.fetch_add(1);
  const int prev = g_tc_pair;
  g_tc_pair = enable ? 1 : 0;
  return prev;
}

int mtpb_set_decode_spin(int backoff_ns) {
  g_settings_epoch.fetch_add(1);
  if (backoff_ns < 0 || backoff_ns > 100000) return fail(MTPB_ERR_INVALID, "decode spin back-off: 0 .. 100000 ns");
  g_mk_spin_ns = uint32_t(backoff_ns);
  return MTPB_OK;
}

int mtpb_set_decode_trace(void* buf) {
  g_settings_epoch.fetch_add(1);
  g_mk_trace = static_cast<unsigned long long*>(buf);
  return MTPB_OK;
}

int mtpb_set_decode_impl(int impl) {
  g_settings_epoch.fetch_add(1);
  if (impl != 0 && impl != 1) return fail(MTPB_ERR_INVALID, "decode impl must be 0 (megakernel) or 1 (kernel chain)");
  g_decode_impl = impl;
  return MTPB_OK;
}

uint64_t mtpb_settings_epoch(void) { return g_settings_epoch.load(); }

int mtpb_model_forward(void* model, const int64_t* ids, int B, int T, const int64_t* rope_pos, int cache_len,
                       void* const* k_caches, void* const* v_caches, int cap, void* logits, int last_only,
                       void* stream) {
  if (!model || !ids || !k_caches || !v_caches) return fail(MTPB_ERR_INVALID, "model_forward: null argument");
  if (B <= 0 || T <= 0) return fail(MTPB_ERR_INVALID, "model_forward: empty batch");
  auto* mh = static_cast<ModelHost*>(model);
  FwdArgs a;
  std::memset(&a, 0, sizeof(a));
  a.ids = reinterpret_cast<const long long*>(ids);
  a.B = B;
  a.T = T;
  a.rope_pos = reinterpret_cast<const long long*>(rope_pos);
  a.cache_len = cache_len;
  a.kc = k_caches;
  a.vc = v_caches;
  a.cap = cap;
  a.logits = logits;
  a.last_only = last_only;
  return model_forward(*mh, a, static_cast<cudaStream_t>(stream));
}

int mtpb_model_decode_kernels(void* model, int B, int cap, int* launches) {
  if (!model || !launches || B <= 0 || cap <= 0) return fail(MTPB_ERR_INVALID, "model_decode_kernels: bad argument");
  auto* mh = static_cast<ModelHost*>(model);
  int mk = 0;
  if (g_decode_impl == 0) {
    MTPB_TRY(mk_reserve(*mh));
    MkParams p;
    size_t smem = 0;
    mk = mk_plan(*mh, B, cap, p, &smem) == MTPB_OK ? 1 : 0;
  }
  // kernel chain: embedding, 5 per layer, final AllReduce + norm, LM head, argmax finish
  *launches = mk ? 1 : 1 + 5 * mh->d.n_layers + 2;
  return MTPB_OK;
}

int mtpb_model_decode_step(void* model, int64_t* tok, int B, void* const* k_caches, void* const* v_caches, int cap,
                           int64_t* out_ids, int ld_out, void* logits, void* stream) {
  if (!model || !tok || !k_caches || !v_caches) return fail(MTPB_ERR_INVALID, "model_decode_step: null argument");
  if (B <= 0 || B > 64) return fail(MTPB_ERR_INVALID, "model_decode_step: need 1 <= B <= 64");
  auto* mh = static_cast<ModelHost*>(model);
  FwdArgs a;
  std::memset(&a, 0, sizeof(a));
  a.ids = reinterpret_cast<const long long*>(tok);
  a.B = B;
  a.T = 1;
  a.pos_ptr = reinterpret_cast<int*>(mh->comm->dev.ctl() + kCtlPos);
  a.kc = k_caches;
  a.vc = v_caches;
  a.cap = cap;
  a.logits = logits;
  a.last_only = 0;
  a.decode = true;
  a.tok_out = reinterpret_cast<long long*>(tok);
  a.out_ids = reinterpret_cast<long long*>(out_ids);
  a.ld_out = ld_out;
  return model_forward(*mh, a, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ------------------------------------------------------------------ attention, no allocation
// mtpb_attention_noalloc keeps its split-KV partials in this file-scope device
// array instead of memory the library allocates. The array is part of the
// module image: every GPU that loads the library holds it until the process
// exits. Layout of one call (offsets rounded up to 256 bytes):
//   [0, 256)              status word of the kernel when the caller passes none
//   counters u32[M*hkv]   last-CTA merge counters, cleared by every call
//   part_ml  f32[M*hq*splits*2], part_o f32[M*hq*splits*hd]
static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[MTPB_NOALLOC_SCRATCH_BYTES];

namespace {

size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

// Device address of g_attn_noalloc_scratch on the current device, looked up
// once per device (host code cannot use the symbol itself as a pointer).
int noalloc_scratch_addr(char** out) {
  static std::mutex mu;
  static char* per_dev[64] = {};
  int dev = 0;
  MTPB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(MTPB_ERR_INVALID, "attention_noalloc: device ordinal above 63");
  std::lock_guard<std::mutex> lk(mu);
  if (!per_dev[dev]) {
    void* p = nullptr;
    MTPB_CUDA(cudaGetSymbolAddress(&p, g_attn_noalloc_scratch));
    per_dev[dev] = static_cast<char*>(p);
  }
  *out = per_dev[dev];
  return MTPB_OK;
}

}  // namespace

extern "C" int mtpb_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, void* out, int B,
                                      int T, int hq, int hkv, int hd, int cap, int cache_len, int dtype,
                                      uint32_t* status, void* stream) {
  if (!q || !k_cache || !v_cache || !out) return fail(MTPB_ERR_INVALID, "attention_noalloc: null tensor");
  if (B <= 0 || T <= 0 || hq <= 0 || hkv <= 0 || hd <= 0 || cap <= 0 || cache_len < 0)
    return fail(MTPB_ERR_INVALID, "attention_noalloc: sizes must be positive");
  if (hq % hkv != 0) return fail(MTPB_ERR_INVALID, "attention: hq must be a multiple of hkv");
  if (cache_len + T > cap) return fail(MTPB_ERR_INVALID, "attention: cache_len + T exceeds the cache capacity");
  const int M = B * T, G = hq / hkv;
  int chunk = 0;
  const int ns = attn_choose_splits(M, hkv, G, cap, hd, &chunk);
  const size_t n_ctr = size_t(M) * hkv, n_ml = size_t(M) * hq * ns * 2, n_o = size_t(M) * hq * ns * hd;
  const size_t off_ctr = 256, off_ml = off_ctr + round256(n_ctr * 4), off_o = off_ml + round256(n_ml * 4);
  const size_t need = off_o + n_o * 4;
  if (ns > 1 && need > MTPB_NOALLOC_SCRATCH_BYTES)
    return fail(MTPB_ERR_INVALID, "attention_noalloc: this shape needs " + std::to_string(need) +
                                      " bytes of scratch; the static scratch holds " +
                                      std::to_string(size_t(MTPB_NOALLOC_SCRATCH_BYTES)) +
                                      " (use fewer rows or a smaller cache capacity, or mtpb_attention)");
  char* base = nullptr;
  MTPB_TRY(noalloc_scratch_addr(&base));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // A view sized exactly to this call's needs: attn_run finds it big enough
  // and never allocates.
  AttnScratch view;
  view.counters = reinterpret_cast<uint32_t*>(base + off_ctr);
  view.part_ml = reinterpret_cast<float*>(base + off_ml);
  view.part_o = reinterpret_cast<float*>(base + off_o);
  view.ctr_elems = n_ctr;
  view.ml_elems = n_ml;
  view.o_elems = n_o;
  if (ns > 1) MTPB_CUDA(cudaMemsetAsync(view.counters, 0, n_ctr * 4, st));
  // device-side error bits go to the caller's word when it passes one
  uint32_t* status_word = status ? status : reinterpret_cast<uint32_t*>(base);
  return attn_run(dtype, q, k_cache, v_cache, out, B, T, hq, hkv, hd, cap, nullptr, cache_len, view, status_word,
                  st);
}
