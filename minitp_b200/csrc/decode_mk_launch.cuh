// Launch interface of the decode megakernel instantiations.
//
// The kernel is compiled in its own translation units (decode_mk_bf16.cu,
// decode_mk_f32.cu), one per element type, so the build compiles them in
// parallel with the rest of the library. Each instantiation fixes the row
// tile MT (batch rows, 1 / 2 / 4 / 8) and the head dimension HD, so a kernel
// carries the code of one attention variant only; combinations without an
// instantiation are planned onto the kernel chain.
#pragma once

#include <cuda_runtime.h>

#include "decode_mk.cuh"

namespace mtpb {

enum : int {
  kMkLaunchOk = 0,
  kMkLaunchNoVariant = 1,  // no instantiation for (dtype, MT, HD)
  kMkLaunchCapture = 2,    // the first launch of a shared-memory size happened under graph capture
  kMkLaunchCuda = 3,       // a CUDA call failed (*err)
};

// True when decode_mk_kernel<T, MT, HD> is compiled (bf16: T = bf16, else fp32).
bool mk_has_variant(bool bf16, int MT, int HD);

// Cooperative launch of one CTA per SM (`grid` CTAs) with `smem` bytes of
// dynamic shared memory; raises the kernel's shared-memory attribute the
// first time a larger size is asked for (not allowed under stream capture).
int mk_launch_bf16(int MT, int HD, const MkParams& p, int grid, size_t smem, cudaStream_t st, cudaError_t* err);
int mk_launch_f32(int MT, int HD, const MkParams& p, int grid, size_t smem, cudaStream_t st, cudaError_t* err);

template <typename T, int MT, int HD>
int mk_launch_one(const MkParams& p, int grid, size_t smem, cudaStream_t st, cudaError_t* err) {
  auto kern = decode_mk_kernel<T, MT, HD>;
  static size_t smem_set = 0;
  if (smem > smem_set) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs != cudaStreamCaptureStatusNone) return kMkLaunchCapture;
    *err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (*err != cudaSuccess) return kMkLaunchCuda;
    smem_set = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMkThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  *err = cudaLaunchKernelEx(&cfg, kern, p);
  return *err == cudaSuccess ? kMkLaunchOk : kMkLaunchCuda;
}

}  // namespace mtpb
