"""The O epilogue writes exactly the rows and columns of O (and of LSE) it owns.  The
outputs here are views into larger tensors: O with row and head strides larger than
D, LSE with a head stride larger than N.  Each kernel family is checked: the box
stores of the one-thread and 64-row kernels (identity order, and original order
through the residue-strided 4-D view), the per-thread stores of the two-thread
kernel, and a merging part that loads the rows in place through the same boxes.
The results must match the oracle, and every element around the views keeps its
sentinel value."""
import pytest
import torch

from cases import SPECS
from test_gpu_attention import ATOL, RTOL, _assert_close, _oracle, _rand
from test_gpu_merge import _part, _union_ref

pytestmark = pytest.mark.gpu

CASES = [("window-128", 0, dict(row_threads=1)),
         ("window-128", 0, dict(row_threads=2)),
         ("window-128", 0, dict(kv_rows=64)),
         ("dilated-4", 4, dict(row_threads=1)),
         ("dilated-4", 4, dict(row_threads=2)),
         ("dilated-4", 4, dict(kv_rows=64))]


def _views(BH, N, D, dtype=torch.bfloat16):
    """O as the middle third of a [BH, N, 3D] tensor, LSE as the middle of a
    [BH, 2N] one; the rest holds sentinels."""
    big = torch.full((BH, N, 3 * D), 7.0, device="cuda", dtype=dtype)
    lse_big = torch.full((BH, 2 * N), 5.0, device="cuda")
    return big, big[..., D:2 * D], lse_big, lse_big[:, N // 2:N // 2 + N]


def _untouched(big, lse_big, N, D):
    assert (big[..., :D] == 7).all() and (big[..., 2 * D:] == 7).all()
    assert (lse_big[:, :N // 2] == 5).all() and (lse_big[:, N // 2 + N:] == 5).all()


@pytest.mark.parametrize("D,dtype", [(128, torch.bfloat16), (64, torch.float16)])
@pytest.mark.parametrize("name,s,opts", CASES)
def test_output_views(name, s, opts, D, dtype):
    from polyhedral_b200 import blockindex, masks, permute
    from polyhedral_b200.triton_attn import block_sparse_attention
    N, BH = 1024, 3
    q, k, v = _rand(BH, N, D, dtype, seed=21)
    spec = SPECS[name]
    perm = torch.from_numpy(permute.residue_perm(N, s)).cuda() if s else None
    bi = blockindex.build(masks.from_spec(*spec), N, 128, 32, perm_q=perm, perm_kv=perm)
    kvi, kvn, kvp = blockindex.to_cuda(bi)
    big, o, lse_big, lse = _views(BH, N, D, dtype)
    block_sparse_attention(q, k, v, kvi, kvn, kvp, *spec, 128, 32, residue_stride=s,
                           return_lse=True, check=True, out=o, lse_out=lse, **opts)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    tol = 3e-3 if dtype == torch.float16 else ATOL
    _assert_close(o, lse, o_ref, lse_ref, atol=tol, rtol=RTOL if tol == ATOL else 0)
    _untouched(big, lse_big, N, D)


@pytest.mark.parametrize("D,dtype", [(128, torch.bfloat16), (64, torch.float16)])
@pytest.mark.parametrize("stride2", [0, 8])
def test_merge_into_output_views(stride2, D, dtype):
    """A split whose second part merges into the first part's views (the rows in
    place come in through TMA box loads of the same strided O map)."""
    from polyhedral_b200 import masks
    N, BH = 2048, 2
    q, k, v = _rand(BH, N, D, dtype, seed=22)
    p1, p2 = masks.FarStrided(1024, 8), masks.SlidingWindow(256)
    if stride2:
        p1, p2 = masks.SlidingWindow(256), masks.FarStrided(1024, 8)
    big, o, lse_big, lse = _views(BH, N, D, dtype)
    _part(q, k, v, p1, N, 128, 32, out=o, lse_out=lse, row_threads=1)
    _part(q, k, v, p2, N, 128, 64, stride2, out=o, lse_out=lse, merge=True)
    o_ref, lse_ref = _union_ref(q, k, v, p1.dense(N) | p2.dense(N))
    assert (o.float().cpu() - o_ref).abs().max().item() < 2e-2
    fin = torch.isfinite(lse_ref)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    assert (lse.cpu()[fin] - lse_ref[fin]).abs().max().item() < 2e-2
    _untouched(big, lse_big, N, D)
