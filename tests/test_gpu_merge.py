"""GPU LSE merge vs the oracle merge, and the split path vs attention over the
union mask."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
def test_lse_merge_matches_oracle(dtype, D):
    from polyhedral_b200 import merge
    BH, N = 3, 777
    g = torch.Generator().manual_seed(9)
    o1, o2 = (torch.randn(BH, N, D, generator=g).to(dtype) for _ in range(2))
    l1, l2 = (torch.randn(BH, N, generator=g) * 3 for _ in range(2))
    l1[0, :10] = float("-inf")
    l2[0, 5:15] = float("-inf")                     # rows 5-9 dead in both parts
    o_ref, lse_ref = O.lse_merge(o1.float().numpy(), l1.numpy(), o2.float().numpy(), l2.numpy())
    o, lse = merge.lse_merge(o1.cuda(), l1.cuda(), o2.cuda(), l2.cuda())
    np.testing.assert_allclose(o.float().cpu().numpy(), o_ref, atol=1e-2, rtol=1e-2)
    lse = lse.cpu().numpy()
    assert np.array_equal(np.isneginf(lse), np.isneginf(lse_ref))
    fin = np.isfinite(lse_ref)
    np.testing.assert_allclose(lse[fin], lse_ref[fin], atol=1e-5, rtol=1e-5)
    assert (o[0, 5:10] == 0).all()


def test_lse_merge_row_map_and_in_place():
    from polyhedral_b200 import merge, permute
    BH, N, D = 2, 512, 128
    g = torch.Generator().manual_seed(4)
    o1, o2 = (torch.randn(BH, N, D, generator=g).bfloat16().cuda() for _ in range(2))
    l1, l2 = (torch.randn(BH, N, generator=g).cuda() for _ in range(2))
    perm = torch.from_numpy(permute.residue_perm(N, 8)).cuda()
    o2p, l2p = o2.index_select(1, perm.long()), l2.index_select(1, perm.long())
    ref_o, ref_l = merge.lse_merge(o1, l1, o2, l2)
    o, lse = merge.lse_merge(o1.clone(), l1.clone(), o2p, l2p, row_map2=permute.invert(perm))
    assert torch.equal(o, ref_o) and torch.equal(lse, ref_l)
    a, b = o1.clone(), l1.clone()
    merge.lse_merge(a, b, o2, l2, out=a, lse_out=b)
    assert torch.equal(a, ref_o) and torch.equal(b, ref_l)


def test_split_equals_union_attention():
    from polyhedral_b200 import masks, split
    N, D, BH = 2048, 128, 2
    g = torch.Generator().manual_seed(12)
    q, k, v = (torch.randn(BH, N, D, generator=g).bfloat16().cuda() for _ in range(3))
    for BQ, A in ((128, 32), (128, 128), (16, 16)):
        sp = split.SplitPlan([split.SplitPart(masks.SlidingWindow(256), BQ, A, 0),
                              split.SplitPart(masks.FarStrided(256, 16), BQ, A, 16)], N)
        o, lse = sp.run(q, k, v)
        M = torch.from_numpy(O.dense_mask(O.LOCAL_STRIDED, 256, 16, 0, N))
        o_ref, lse_ref = O.attention_heads(q.float().cpu(), k.float().cpu(), v.float().cpu(), M)
        assert (o.float().cpu() - o_ref).abs().max().item() < 2e-2
        assert (lse.cpu() - lse_ref).abs().max().item() < 2e-2
