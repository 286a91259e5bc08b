// Instantiations of the 64-row super-tile attention forward for D = 64, inputs read through a residue permutation.
#include "attn_kernel_db.cuh"

namespace pa {
namespace attn {
namespace db {

int launch_d64_residue(const Tmap& tq, const Tmap& tk, const Tmap& tv, const FwdParams& P, int grid, int L,
       bool bf16, cudaStream_t stream) {
  return launch_family_db<64, true>(tq, tk, tv, P, grid, L, bf16, stream);
}

}  // namespace db
}  // namespace attn
}  // namespace pa
