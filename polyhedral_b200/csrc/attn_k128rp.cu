// Instantiations of the attention forward kernel for D = 128, residue-permuted view with
// two softmax threads per row (16 softmax warps).
#include "attn_kernel.cuh"

namespace pa {
namespace attn {

int launch_d128_residue_pairs(const Tmap& tq, const Tmap& tk, const Tmap& tv, const FwdParams& P,
                          int grid, int L, bool bf16, cudaStream_t stream) {
  return launch_family<128, true, false, false, 2>(tq, tk, tv, P, grid, L, bf16, stream);
}

}  // namespace attn
}  // namespace pa
