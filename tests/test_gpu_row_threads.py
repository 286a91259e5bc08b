"""The forward with two softmax threads per query row (``row_threads=2``: 16 softmax
warps, 64 S columns per thread, partial row maxima exchanged per super-tile) against
the CPU oracle, on the gate matrix of masks x tile shapes x head dims x dtypes, the
in-kernel residue permutation, explicit permutations with a fused inverse, dead rows
and a running maximum that grows along the row.

Tolerances as tests/test_gpu_attention.py: 2e-2 absolute + 1e-2 relative (3e-3 for
fp16 at D = 64); dead rows exactly O = 0, LSE = -inf.
"""
import numpy as np
import pytest
import torch

import oracle as O
from cases import SPECS

pytestmark = pytest.mark.gpu

from test_gpu_attention import _assert_close, _oracle, _rand, _run  # noqa: E402

TILES = [(128, 128), (128, 32), (64, 64), (16, 16)]
NAMES = ["causal", "window-128", "dilated-8", "local256+str8", "twoband-1000", "sinks4+win256"]


@pytest.mark.parametrize("D,dtype", [(128, torch.bfloat16), (64, torch.bfloat16),
                                     (64, torch.float16)])
@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("BQ,A", TILES)
def test_gate_matrix(name, BQ, A, D, dtype):
    N = 1024
    q, k, v = _rand(2, N, D, dtype, seed=N + BQ + A)
    o, lse = _run(q, k, v, name, N, BQ, A, row_threads=2)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    atol = 3e-3 if (dtype == torch.float16 and D == 64) else 2e-2
    _assert_close(o, lse, o_ref, lse_ref, atol=atol)


@pytest.mark.parametrize("name,s,A", [("dilated-4", 4, 32), ("local64+str8", 8, 32),
                                      ("far1024+str16", 16, 64), ("dilated-8", 8, 16)])
def test_residue_in_kernel(name, s, A):
    """residue_stride: q/k/v and o/lse in original order, the permutation applied by
    the kernel's tensor maps and epilogue."""
    from polyhedral_b200 import blockindex, masks, permute
    from polyhedral_b200.triton_attn import block_sparse_attention
    N = 4096 if s == 16 else 2048
    q, k, v = _rand(2, N, 128, torch.bfloat16, seed=s)
    spec = SPECS[name]
    perm = permute.residue_perm(N, s)
    bi = blockindex.build(masks.from_spec(*spec), N, 128, A, perm_q=perm, perm_kv=perm)
    idx = blockindex.to_cuda(bi)
    o, lse = block_sparse_attention(q, k, v, *idx, *spec, 128, A, residue_stride=s,
                                    return_lse=True, check=True, row_threads=2)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    _assert_close(o, lse, o_ref, lse_ref)


def test_explicit_permutation_with_fused_inverse():
    from polyhedral_b200 import blockindex, masks, permute
    from polyhedral_b200.triton_attn import block_sparse_attention
    N, name = 2048, "local256+str8"
    q, k, v = _rand(2, N, 128, torch.bfloat16, seed=9)
    p_np = permute.residue_perm(N, 8)
    perm = torch.from_numpy(p_np).cuda()
    qp, kp, vp = (t.index_select(1, perm.long()) for t in (q, k, v))
    spec = SPECS[name]
    bi = blockindex.build(masks.from_spec(*spec), N, 128, 32, perm_q=p_np, perm_kv=p_np)
    idx = blockindex.to_cuda(bi)
    o, lse = block_sparse_attention(qp, kp, vp, *idx, *spec, 128, 32, perm_q=perm,
                                    perm_kv=perm, o_row_map=perm, return_lse=True,
                                    check=True, row_threads=2)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    _assert_close(o, lse, o_ref, lse_ref)


def test_dead_rows_and_growing_maximum():
    """Rows with no live key (far band) stay O = 0 / LSE = -inf; keys scaled up along
    the row make the running maximum grow past the lazy-rescale threshold."""
    from polyhedral_b200 import masks
    N = 2048
    q, k, v = _rand(2, N, 128, torch.bfloat16, seed=31)
    beta = torch.tensor([0.0, 1.0, 3.0, 9.0]).repeat_interleave(N // 4)
    k = (k.float().cpu() * (1 + beta[None, :, None])).bfloat16().cuda()
    o, lse = _run(q, k, v, "causal", N, 128, 32, row_threads=2)
    o_ref, lse_ref = _oracle(q, k, v, "causal", N)
    _assert_close(o, lse, o_ref, lse_ref)
    far = masks.FarStrided(600, 8)
    from polyhedral_b200 import blockindex
    from polyhedral_b200.triton_attn import block_sparse_attention
    bi = blockindex.build(far, 1024, 128, 32)
    q2, k2, v2 = (t[:, :1024].contiguous() for t in (q, k, v))
    o2, l2 = block_sparse_attention(q2, k2, v2, *blockindex.to_cuda(bi), *far.spec, 128, 32,
                                    return_lse=True, check=True, row_threads=2)
    assert (o2[:, :600] == 0).all() and torch.isneginf(l2[:, :600]).all()
    M = torch.from_numpy(far.dense(1024))
    o_ref2, l_ref2 = O.attention_heads(q2.float().cpu(), k2.float().cpu(), v2.float().cpu(), M)
    _assert_close(o2, l2, o_ref2, l_ref2)


def test_argument_errors():
    from polyhedral_b200 import _lib
    N = 1024
    q, k, v = _rand(1, N, 128, torch.bfloat16)
    with pytest.raises(_lib.PolyattnError):
        _run(q, k, v, "causal", N, 128, 32, row_threads=3)
    with pytest.raises(_lib.PolyattnError):
        _run(q, k, v, "causal", N, 128, 32, row_threads=2, kv_rows=64)
    o, lse = _run(q, k, v, "causal", N, 128, 32)
    with pytest.raises(_lib.PolyattnError):
        _run(q, k, v, "causal", N, 128, 32, row_threads=2, merge=True, out=o, lse_out=lse)


@pytest.mark.parametrize("name", ["causal", "window-128", "local256+str8"])
@pytest.mark.parametrize("N,BQ,A", [(1152, 128, 32), (1152, 128, 128), (1088, 64, 64),
                                    (1040, 16, 16)])
def test_ragged_sequence(name, N, BQ, A):
    """N not a multiple of the 256-row work item: the last item's second half (or part
    of it) lies past the sequence and must not be written."""
    q, k, v = _rand(2, N, 128, torch.bfloat16, seed=N + A)
    o, lse = _run(q, k, v, name, N, BQ, A, row_threads=2)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    _assert_close(o, lse, o_ref, lse_ref)
