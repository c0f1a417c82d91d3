// Peer-memory communicator: one cudaMalloc'd buffer per rank, mapped into
// every other rank of the node through CUDA IPC (exchanged once at init).
//
// Buffer layout of every rank (byte offsets from its base):
//   [0, kCtlBytes)              control words (local use only)
//   [kCtlBytes, +kFlagBytes)    flags[chan][parity][src_rank][cta]   (u32)
//   [kDataOff, ...)             data[chan][parity][src_rank][slot_bytes]
//
// A producer CTA on rank `src` stores its payload into data[chan][par][src]
// of EVERY rank (NVLink stores to peers, a plain store to itself), then
// raises flags[chan][par][src][cta] = seq on every rank with a system-scope
// release. A consumer on rank r waits (bounded) until the flags of all
// producers reached `seq`, then reads data[chan][par][*] from its own HBM and
// reduces in rank order 0..world-1, so every rank computes bit-identical
// sums. `par = seq & 1`; consecutive collectives alternate parity, which
// keeps a fast rank from overwriting a slot a slow rank is still reading.
//
// Channel 0 carries the model's collectives; their sequence numbers come from
// a device step counter so a captured CUDA graph can replay them. Channel 1
// carries standalone collectives (all_reduce, the fused AR+RMSNorm op), whose
// sequence numbers come from a device call counter. Channel 2 belongs to the
// decode megakernel, whose data words carry their own sequence numbers
// (LL words) and need no flags; channel 3 carries the LL form of the
// standalone collectives (same counter as channel 1).
#pragma once

#include "common.cuh"

namespace mtpb {

constexpr int kChannels = 4;
constexpr int kMaxCtas = 1024;
constexpr size_t kCtlBytes = 4096;
constexpr size_t kFlagBytes = size_t(kChannels) * 2 * kMaxRanks * kMaxCtas * sizeof(uint32_t);
constexpr size_t kDataOff = kCtlBytes + kFlagBytes;

// control word indices (u32, local buffer)
enum : int {
  kCtlStatus = 0,     // error bits (kStatus*)
  kCtlStep = 1,       // channel-0 step counter
  kCtlStepDone = 2,   // CTA completion counter of the kernel that advances kCtlStep
  kCtlColl = 3,       // channel-1 call counter
  kCtlCollDone = 4,   // CTA completion counter of the channel-1 kernels
  kCtlPos = 8,        // decode position (i32) read by the captured decode step
};

struct Comm {
  int rank;
  int world;
  char* base[kMaxRanks];  // base[r]: rank r's buffer in this address space
  uint64_t slot_bytes;
  uint64_t timeout_ns;

  __host__ __device__ uint32_t* ctl() const { return reinterpret_cast<uint32_t*>(base[rank]); }
  __host__ __device__ uint32_t* status() const { return ctl() + kCtlStatus; }

  __host__ __device__ uint32_t* flag(int dst, int chan, int par, int src, int cta) const {
    size_t idx = ((size_t(chan) * 2 + par) * kMaxRanks + src) * kMaxCtas + cta;
    return reinterpret_cast<uint32_t*>(base[dst] + kCtlBytes) + idx;
  }
  __host__ __device__ char* data(int dst, int chan, int par, int src) const {
    return base[dst] + kDataOff + ((size_t(chan) * 2 + par) * world + src) * slot_bytes;
  }
  static size_t buffer_bytes(uint64_t slot_bytes, int world) {
    return kDataOff + size_t(kChannels) * 2 * world * slot_bytes;
  }
};

// Sequence number of one collective site. Channel 0 uses
// step * nsite + site + 1 with `step` read from device memory after
// pdl_wait(); a site with `fixed != 0` uses that value instead.
struct SeqRef {
  uint32_t site;
  uint32_t nsite;
  uint32_t fixed;
};

__device__ __forceinline__ uint32_t resolve_seq(const Comm& c, const SeqRef& s) {
  if (s.fixed) return s.fixed;
  return ld_volatile_u32(c.ctl() + kCtlStep) * s.nsite + s.site + 1u;
}

// Producer side: after every thread of the CTA stored its payload, raise this
// CTA's flag on every rank. Call from all threads.
__device__ __forceinline__ void signal_peers(const Comm& c, int chan, uint32_t seq) {
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_sys();
    const int par = seq & 1;
    for (int d = 0; d < c.world; ++d) st_relaxed_sys(c.flag(d, chan, par, c.rank, blockIdx.x), seq);
  }
}

// Two-shot form (reduce-scatter, then all-gather) of a large collective: the
// columns of a row are cut into `world` slices of ts_cols columns (a multiple
// of the vector width; the last slice may be short or empty) and rank j owns
// slice j. Producers store slice j of their partial rows only into rank j's
// data[chan][par][src] (one copy of each value instead of `world`). Consumer
// CTA b of the owner sums its rows' slice over the sources in rank order,
// rounds it like the one-shot sum, and stores the result into the unused
// slice-j columns of data[chan][par][j] on every rank, then raises flag
// kAgCta + b; every rank's CTA b waits for those flags and reads each column
// from the slot of its owner. Consumers of both forms compute identical bits.
constexpr int kAgCta = 512;  // flag index offset of the all-gather step

__host__ __device__ inline int ts_owner(int col, int ts_cols, int world) {
  const int j = col / ts_cols;
  return j < world ? j : world - 1;
}

// Producer side, explicit flag index: raise flag `cta` on every rank.
__device__ __forceinline__ void signal_peers_at(const Comm& c, int chan, uint32_t seq, int cta) {
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_sys();
    const int par = seq & 1;
    for (int d = 0; d < c.world; ++d) st_relaxed_sys(c.flag(d, chan, par, c.rank, cta), seq);
  }
}

// Consumer side: wait until producer CTAs [0, nprod) of every rank signalled
// `seq`. With world == 1 nothing needs waiting (stream order suffices).
// (warp 0 polls; every thread of the block must call it)
__device__ __forceinline__ bool wait_peers(const Comm& c, int chan, uint32_t seq, int nprod) {
  if (c.world == 1) return true;
  __shared__ int s_ok;
  if (threadIdx.x < 32) {
    const int par = seq & 1;
    // every rank's producer flags in one poll (consecutive ranks' flags are
    // kMaxCtas apart)
    const bool ok = warp_poll_flags(c.flag(c.rank, chan, par, 0, 0), nprod, seq, true, c.status(), c.timeout_ns,
                                    nullptr, c.world, size_t(kMaxCtas));
    if (threadIdx.x == 0) {
      s_ok = ok ? 1 : 0;
      if (!ok) atomicOr(c.status(), kStatusTimeout);
    }
  }
  __syncthreads();
  const bool res = s_ok != 0;
  __syncthreads();
  return res;
}

// Same as wait_peers but only for producer CTA `cta` of every rank (kernels
// whose CTA c consumes exactly what CTA c of each peer produced).
__device__ __forceinline__ bool wait_peers_cta(const Comm& c, int chan, uint32_t seq, int cta) {
  if (c.world == 1) return true;
  __shared__ int s_ok2;
  if (threadIdx.x < 32) {
    const int par = seq & 1;
    const bool ok = warp_poll_flags(c.flag(c.rank, chan, par, 0, cta), 1, seq, true, c.status(), c.timeout_ns,
                                    nullptr, c.world, size_t(kMaxCtas));
    if (threadIdx.x == 0) {
      s_ok2 = ok ? 1 : 0;
      if (!ok) atomicOr(c.status(), kStatusTimeout);
    }
  }
  __syncthreads();
  const bool res = s_ok2 != 0;
  __syncthreads();
  return res;
}

// Called once per CTA at the end of a kernel that advances a device counter
// (kCtlStep or kCtlColl): the last CTA to finish stores `next` and resets the
// completion counter. Every CTA read the old value before arriving here.
__device__ __forceinline__ void advance_counter(const Comm& c, int ctr, int done, uint32_t next) {
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* ctl = c.ctl();
    if (gridDim.x == 1) {
      ctl[ctr] = next;
    } else {
      __threadfence();
      if (atomicAdd(ctl + done, 1u) == gridDim.x - 1) {
        ctl[ctr] = next;
        ctl[done] = 0;
      }
    }
  }
}

}  // namespace mtpb
