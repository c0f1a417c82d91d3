// bf16 instantiations of the decode megakernel: head dims 64 and 128 (the
// Qwen2.5 shapes) for 1, 2, 4 and 8 rows, head dim 16 (the small test shape)
// for one row.
#include "decode_mk_launch.cuh"

namespace mtpb {

int mk_launch_bf16(int MT, int HD, const MkParams& p, int grid, size_t smem, cudaStream_t st, cudaError_t* err) {
  switch (HD * 16 + MT) {
    case 64 * 16 + 1: return mk_launch_one<bf16, 1, 64>(p, grid, smem, st, err);
    case 64 * 16 + 2: return mk_launch_one<bf16, 2, 64>(p, grid, smem, st, err);
    case 64 * 16 + 4: return mk_launch_one<bf16, 4, 64>(p, grid, smem, st, err);
    case 64 * 16 + 8: return mk_launch_one<bf16, 8, 64>(p, grid, smem, st, err);
    case 128 * 16 + 1: return mk_launch_one<bf16, 1, 128>(p, grid, smem, st, err);
    case 128 * 16 + 2: return mk_launch_one<bf16, 2, 128>(p, grid, smem, st, err);
    case 128 * 16 + 4: return mk_launch_one<bf16, 4, 128>(p, grid, smem, st, err);
    case 128 * 16 + 8: return mk_launch_one<bf16, 8, 128>(p, grid, smem, st, err);
    case 16 * 16 + 1: return mk_launch_one<bf16, 1, 16>(p, grid, smem, st, err);
    default: return kMkLaunchNoVariant;
  }
}

}  // namespace mtpb
