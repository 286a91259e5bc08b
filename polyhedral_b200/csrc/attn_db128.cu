// Instantiations of the 64-row super-tile attention forward for D = 128, inputs in kernel order.
#include "attn_kernel_db.cuh"

namespace pa {
namespace attn {
namespace db {

int launch_d128(const Tmap& tq, const Tmap& tk, const Tmap& tv, const FwdParams& P, int grid, int L,
       bool bf16, cudaStream_t stream) {
  return launch_family_db<128, false>(tq, tk, tv, P, grid, L, bf16, stream);
}

}  // namespace db
}  // namespace attn
}  // namespace pa
