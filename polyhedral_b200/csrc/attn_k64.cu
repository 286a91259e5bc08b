// Instantiations of the attention forward kernel for D = 64.
#include "attn_kernel.cuh"

namespace pa {
namespace attn {

int launch_d64(const Tmap& tq, const Tmap& tk, const Tmap& tv, const FwdParams& P, int grid, int L,
       bool bf16, cudaStream_t stream) {
  return launch_family<64, false, false>(tq, tk, tv, P, grid, L, bf16, stream);
}

}  // namespace attn
}  // namespace pa
