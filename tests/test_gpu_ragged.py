"""Sequence lengths that are not a multiple of an item's 256 rows: the last work item
has a second 128-row half past N (no rows to compute, none to write), and its box
stores and box loads of O reach past the tensor's end (clipped / zero-filled by the
tensor map).  Every kernel family, identity and residue order, and a merge; outputs
as views with sentinels around them, so a write past N would show."""
import pytest
import torch

from cases import SPECS
from test_gpu_attention import _assert_close, _oracle, _rand
from test_gpu_epilogue import _untouched, _views
from test_gpu_merge import _part, _union_ref

pytestmark = pytest.mark.gpu

OPTS = [dict(row_threads=1), dict(row_threads=2), dict(kv_rows=64)]


@pytest.mark.parametrize("N,s", [(1152, 0), (640, 0), (1152, 3)])
@pytest.mark.parametrize("opts", OPTS)
@pytest.mark.parametrize("name", ["causal", "window-128", "sinks4+win256"])
def test_ragged_last_item(name, opts, N, s):
    from polyhedral_b200 import blockindex, masks, permute
    from polyhedral_b200.triton_attn import block_sparse_attention
    D, BH = 128, 3
    q, k, v = _rand(BH, N, D, torch.bfloat16, seed=41)
    spec = SPECS[name]
    perm = torch.from_numpy(permute.residue_perm(N, s)).cuda() if s else None
    bi = blockindex.build(masks.from_spec(*spec), N, 128, 64, perm_q=perm, perm_kv=perm)
    kvi, kvn, kvp = blockindex.to_cuda(bi)
    big, o, lse_big, lse = _views(BH, N, D)
    block_sparse_attention(q, k, v, kvi, kvn, kvp, *spec, 128, 64, residue_stride=s,
                           return_lse=True, check=True, out=o, lse_out=lse, **opts)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    _assert_close(o, lse, o_ref, lse_ref)
    _untouched(big, lse_big, N, D)


@pytest.mark.parametrize("N", [1152, 640])
def test_ragged_merge(N):
    from polyhedral_b200 import masks
    D, BH = 128, 2
    q, k, v = _rand(BH, N, D, torch.bfloat16, seed=42)
    p1, p2 = masks.SlidingWindow(64), masks.FarStrided(64, 8)
    big, o, lse_big, lse = _views(BH, N, D)
    _part(q, k, v, p1, N, 128, 64, out=o, lse_out=lse, row_threads=1)
    _part(q, k, v, p2, N, 128, 64, out=o, lse_out=lse, merge=True)
    o_ref, lse_ref = _union_ref(q, k, v, p1.dense(N) | p2.dense(N))
    assert (o.float().cpu() - o_ref).abs().max().item() < 2e-2
    fin = torch.isfinite(lse_ref)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    assert (lse.cpu()[fin] - lse_ref[fin]).abs().max().item() < 2e-2
    _untouched(big, lse_big, N, D)
