"""The reference's class-B traffic emulation (gpu/triton_attn.py:99-128, driven by
gpu/exp6_traffic_multiplier.py): K/V left in original order and gathered per tile
through perm_kv (``gather_kv``), plus ``gather_mult`` - 1 extra row sets per K tile
that the result does not use, contiguous or scattered.

exp6 checks that the gathered and the physically permuted forwards agree (max abs
err <= 1e-3, exp6_traffic_multiplier.py:87-91).  Here the gathered kernel stages the
same K/V values in shared memory as the permuted one and runs the same MMAs and
softmax, so the outputs must be bit-identical; one case per mask is also held to the
CPU oracle (2e-2 abs + 1e-2 rel; 3e-3 for fp16 as gpu/test_correctness.py:23).
"""
import numpy as np
import pytest
import torch

import oracle as O
from cases import SPECS

pytestmark = pytest.mark.gpu

TILES = [(128, 128), (128, 32), (64, 64), (32, 32), (16, 16)]


def _setup(name, s, N, BQ, A, BH=2, D=64, dtype=torch.float16, seed=0, perm_np=None):
    from polyhedral_b200 import blockindex, masks
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(BH, N, D, generator=g).to(dtype).cuda() for _ in range(3))
    if perm_np is None:
        perm_np = O.residue_perm(N, s)
    perm = torch.from_numpy(perm_np).cuda()
    pi = perm.int()
    qp, kp, vp = (t.index_select(1, perm.long()) for t in (q, k, v))
    spec = SPECS[name]
    bi = blockindex.build(masks.from_spec(*spec), N, BQ, A, perm_q=perm_np, perm_kv=perm_np)
    idx = blockindex.to_cuda(bi)
    return q, k, v, qp, kp, vp, pi, spec, idx


def _attn(q, k, v, idx, spec, BQ, A, pi, **kw):
    # one softmax thread per row, as the gathered kernel, so that the comparisons
    # below are bit for bit
    from polyhedral_b200.triton_attn import block_sparse_attention
    kw.setdefault("row_threads", 1)
    return block_sparse_attention(q, k, v, *idx, *spec, BQ, A, perm_q=pi, perm_kv=pi,
                                  return_lse=True, check=True, **kw)


@pytest.mark.parametrize("D,dtype", [(64, torch.float16), (128, torch.bfloat16)])
@pytest.mark.parametrize("name,s", [("dilated-8", 8), ("dilated-4", 4), ("local256+str8", 8)])
@pytest.mark.parametrize("BQ,A", TILES)
def test_gathered_equals_permuted(name, s, BQ, A, D, dtype):
    N = 2048
    q, k, v, qp, kp, vp, pi, spec, idx = _setup(name, s, N, BQ, A, D=D, dtype=dtype)
    oc, lc = _attn(qp, kp, vp, idx, spec, BQ, A, pi)
    og, lg = _attn(qp, k, v, idx, spec, BQ, A, pi, gather_kv=True)
    assert torch.equal(og, oc) and torch.equal(lg, lc)


@pytest.mark.parametrize("name,s", [("dilated-8", 8), ("local256+str8", 8)])
def test_gathered_vs_oracle(name, s):
    N, BQ, A = 2048, 128, 32
    q, k, v, qp, kp, vp, pi, spec, idx = _setup(name, s, N, BQ, A, D=64)
    og, lg = _attn(qp, k, v, idx, spec, BQ, A, pi, gather_kv=True)
    inv = torch.from_numpy(np.argsort(pi.cpu().numpy())).long().cuda()
    o = og.index_select(1, inv).float().cpu()
    lse = lg.index_select(1, inv).cpu()
    M = torch.from_numpy(O.dense_mask(*spec, N))
    o_ref, lse_ref = O.attention_heads(q.float().cpu(), k.float().cpu(), v.float().cpu(), M)
    assert ((o - o_ref).abs() <= 3e-3 + 1e-2 * o_ref.abs()).all(), (o - o_ref).abs().max()
    fin = torch.isfinite(lse_ref)
    assert torch.equal(torch.isfinite(lse), fin)
    assert ((lse[fin] - lse_ref[fin]).abs() <= 2e-2 + 1e-2 * lse_ref[fin].abs()).all()


@pytest.mark.parametrize("scatter", [False, True])
@pytest.mark.parametrize("R", [2, 4, 16])
@pytest.mark.parametrize("BQ,A", [(128, 128), (128, 32), (16, 16)])
def test_row_multiplier_leaves_result_unchanged(R, scatter, BQ, A):
    N = 2048
    q, k, v, qp, kp, vp, pi, spec, idx = _setup("dilated-8", 8, N, BQ, A, D=64)
    oc, lc = _attn(qp, kp, vp, idx, spec, BQ, A, pi)
    og, lg = _attn(qp, k, v, idx, spec, BQ, A, pi, gather_kv=True, gather_mult=R,
                   gather_scatter=scatter)
    assert torch.equal(og, oc) and torch.equal(lg, lc)
    # the multiplier without gather_kv: K/V physically permuted, extra rows only
    o2, l2 = _attn(qp, kp, vp, idx, spec, BQ, A, pi, gather_mult=R, gather_scatter=scatter)
    assert torch.equal(o2, oc) and torch.equal(l2, lc)


@pytest.mark.parametrize("D", [64, 128])
def test_arbitrary_permutation(D):
    """A permutation whose tiles are no arithmetic progression: every K/V row of a
    tile comes from an unrelated place, and the predicate takes the per-element path."""
    N, BQ, A = 1024, 128, 32
    perm_np = np.random.default_rng(3).permutation(N).astype(np.int32)
    q, k, v, qp, kp, vp, pi, spec, idx = _setup("window-128", 0, N, BQ, A, D=D,
                                                dtype=torch.bfloat16, perm_np=perm_np)
    oc, lc = _attn(qp, kp, vp, idx, spec, BQ, A, pi)
    og, lg = _attn(qp, k, v, idx, spec, BQ, A, pi, gather_kv=True, gather_mult=3)
    assert torch.equal(og, oc) and torch.equal(lg, lc)


def test_strided_heads_and_identity_perm():
    """K/V heads further apart than N rows (a slice of a longer buffer), and no
    permutation at all (perm_kv = None reads rows in order)."""
    from polyhedral_b200 import blockindex, masks
    from polyhedral_b200.triton_attn import block_sparse_attention
    N, BQ, A, D, BH = 1024, 128, 64, 128, 3
    g = torch.Generator().manual_seed(5)
    q = torch.randn(BH, N, D, generator=g).bfloat16().cuda()
    big_k = torch.randn(BH, N + 256, D, generator=g).bfloat16().cuda()
    big_v = torch.randn(BH, N + 256, D, generator=g).bfloat16().cuda()
    k, v = big_k[:, 128:128 + N], big_v[:, 128:128 + N]
    spec = SPECS["causal"]
    bi = blockindex.build(masks.from_spec(*spec), N, BQ, A)
    idx = blockindex.to_cuda(bi)
    oc, lc = block_sparse_attention(q, k.contiguous(), v.contiguous(), *idx, *spec, BQ, A,
                                    return_lse=True, check=True, row_threads=1)
    og, lg = block_sparse_attention(q, k, v, *idx, *spec, BQ, A, return_lse=True, check=True,
                                    gather_kv=True, gather_mult=2, gather_scatter=True)
    assert torch.equal(og, oc) and torch.equal(lg, lc)


def test_gather_argument_errors():
    from polyhedral_b200 import _lib
    N, BQ, A = 1024, 128, 32
    q, k, v, qp, kp, vp, pi, spec, idx = _setup("dilated-8", 8, N, BQ, A, D=64)
    from polyhedral_b200.triton_attn import block_sparse_attention
    with pytest.raises(_lib.PolyattnError):
        block_sparse_attention(qp, k, v, *idx, *spec, BQ, A, perm_q=pi, perm_kv=pi,
                               gather_kv=True, kv_rows=64)
    with pytest.raises(_lib.PolyattnError):   # head stride not a multiple of the row stride
        kt = k.transpose(0, 1).contiguous().transpose(0, 1)
        block_sparse_attention(qp, kt, kt, *idx, *spec, BQ, A, perm_q=pi, perm_kv=pi,
                               gather_kv=True)
    with pytest.raises(ValueError):
        block_sparse_attention(qp, k, v, *idx, *spec, BQ, A, perm_q=pi, perm_kv=pi,
                               gather_mult=32)
