"""polyhedral_b200 -- B200 (sm_100a) implementation of the block-sparse attention
forward path of GueroudjiAmal/polyhedral: mask predicate -> block index -> class A
permutation -> block-sparse flash attention (O and LSE) -> LSE merge of disjoint
splits.  The reference's module names are kept: ``masks_gpu``, ``blockindex``,
``permute``, ``triton_attn`` (``block_sparse_attention``)."""
from . import masks, masks_gpu  # noqa: F401

__all__ = ["masks", "masks_gpu", "blockindex", "permute", "attention", "triton_attn",
           "merge", "split", "selector", "timing"]
