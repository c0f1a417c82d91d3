// fp32 instantiations of the decode megakernel (the token-parity runs): head
// dims 16, 64 and 128 for one row, head dim 64 for 4 rows.
#include "decode_mk_launch.cuh"

namespace mtpb {

bool mk_has_variant(bool bf16, int MT, int HD) {
  if (bf16) return ((HD == 64 || HD == 128) && (MT == 1 || MT == 2 || MT == 4 || MT == 8)) || (HD == 16 && MT == 1);
  return (MT == 1 && (HD == 16 || HD == 64 || HD == 128)) || (MT == 4 && HD == 64);
}

int mk_launch_f32(int MT, int HD, const MkParams& p, int grid, size_t smem, cudaStream_t st, cudaError_t* err) {
  switch (HD * 16 + MT) {
    case 16 * 16 + 1: return mk_launch_one<float, 1, 16>(p, grid, smem, st, err);
    case 64 * 16 + 1: return mk_launch_one<float, 1, 64>(p, grid, smem, st, err);
    case 64 * 16 + 4: return mk_launch_one<float, 4, 64>(p, grid, smem, st, err);
    case 128 * 16 + 1: return mk_launch_one<float, 1, 128>(p, grid, smem, st, err);
    default: return kMkLaunchNoVariant;
  }
}

}  // namespace mtpb
