// Instantiations of the 64-row super-tile attention forward for D = 128, inputs read through a residue permutation.
#include "attn_kernel_db.cuh"

namespace pa {
namespace attn {
namespace db {

int launch_d128_residue(const Tmap& tq, const Tmap& tk, const Tmap& tv, const FwdParams& P, int grid, int L,
       bool bf16, cudaStream_t stream) {
  return launch_family_db<128, true>(tq, tk, tv, P, grid, L, bf16, stream);
}

}  // namespace db
}  // namespace attn
}  // namespace pa
