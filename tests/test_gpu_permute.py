"""GPU class-A permutation kernels vs the reference semantics (bit-exact)."""
import numpy as np
import pytest
import torch

import oracle as O
from _golden import perms, sha

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", perms(), ids=lambda c: f"N{c['N']}-s{c['s']}")
def test_residue_perm_device(case):
    from polyhedral_b200 import permute
    p = permute.residue_perm_device(case["N"], case["s"]).cpu().numpy()
    assert sha(p) == case["perm_sha"]
    inv = permute.invert(torch.from_numpy(p).cuda()).cpu().numpy()
    assert sha(inv.astype(np.int32)) == case["inv_sha"]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(3, 1024, 128), (2, 257, 64), (1, 16, 8), (2, 100, 3)])
def test_apply_perm_bit_exact(dtype, shape):
    from polyhedral_b200 import permute
    g = torch.Generator().manual_seed(3)
    x = torch.randn(*shape, generator=g).to(dtype).cuda()
    N = shape[1]
    perm = torch.from_numpy(O.residue_perm(N, 4)).cuda()
    got = permute.apply_perm(x, perm)
    ref = x.index_select(1, perm.long())
    assert torch.equal(got, ref)
    back = permute.scatter_rows(got, perm)
    assert torch.equal(back, x)
    inv = permute.invert(perm)
    assert torch.equal(permute.apply_perm(got, inv), x)


def test_apply_perm_many_and_strided_input():
    from polyhedral_b200 import permute
    base = torch.randn(4, 512, 256, device="cuda").bfloat16()
    q = base[:, :, :128]                       # row stride 256, last dim contiguous
    k = base[:, :, 128:]
    v = torch.randn(4, 512, 128, device="cuda").bfloat16()
    w = torch.randn(4, 512, 128, device="cuda").bfloat16()
    u = torch.randn(4, 512, 128, device="cuda").bfloat16()
    perm = torch.randperm(512, device="cuda").int()
    outs = permute.apply_perm_many((q, k, v, w, u), perm)
    for x, o in zip((q, k, v, w, u), outs):
        assert o.is_contiguous()
        assert torch.equal(o, x.index_select(1, perm.long()))


def test_random_permutation_invert():
    from polyhedral_b200 import permute
    perm = torch.randperm(10007, device="cuda")
    inv = permute.invert(perm)
    assert inv.dtype == perm.dtype
    assert torch.equal(perm[inv], torch.arange(10007, device="cuda"))
