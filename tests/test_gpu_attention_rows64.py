"""The 64-row super-tile attention kernel (kv_rows=64: S double-buffered in TMEM)
vs the CPU oracle, on the cases the default kernel is held to: every mask kind at
every tile shape, permuted and residue-strided inputs, dead rows, running-max
growth, ragged and large tiles, and the full-size configurations 3 and 4 on
sampled rows.  Same tolerances as tests/test_gpu_attention.py."""
import pytest
import torch

from cases import SPECS
from test_gpu_attention import (ATOL, NAMES, RTOL, TILES, _assert_close, _check_sampled,
                                _gpu_inputs, _oracle, _rand, _run, _sample_rows)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("name", NAMES + ["sinks4+win256", "far1024+str16"])
def test_gate_matrix_rows64(name, D, dtype):
    N, BH = 1024, 2
    q, k, v = _rand(BH, N, D, dtype)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    tol = 3e-3 if dtype == torch.float16 else ATOL
    for BQ, A in TILES:
        o, lse = _run(q, k, v, name, N, BQ, A, kv_rows=64)
        _assert_close(o, lse, o_ref, lse_ref, atol=tol, rtol=RTOL if tol == ATOL else 0)


@pytest.mark.parametrize("name,s,N", [("dilated-4", 4, 1024), ("local64+str8", 8, 2048),
                                      ("far1024+str16", 16, 4096)])
@pytest.mark.parametrize("BQ,A", [(16, 16), (128, 32), (128, 128)])
def test_residue_stride_rows64_equals_default(name, s, N, BQ, A):
    """Same O and LSE as the default kernel up to the order of floating-point
    accumulation, and within tolerance of the oracle."""
    from polyhedral_b200 import blockindex, masks, permute
    from polyhedral_b200.triton_attn import block_sparse_attention
    q, k, v = _rand(2, N, 128, torch.bfloat16, seed=s)
    spec = SPECS[name]
    perm = torch.from_numpy(permute.residue_perm(N, s)).cuda()
    bi = blockindex.build(masks.from_spec(*spec), N, BQ, A, perm_q=perm, perm_kv=perm)
    kvi, kvn, kvp = blockindex.to_cuda(bi)
    o, lse = block_sparse_attention(q, k, v, kvi, kvn, kvp, *spec, BQ, A, residue_stride=s,
                                    return_lse=True, check=True, kv_rows=64)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    _assert_close(o, lse, o_ref, lse_ref)
    # explicit permutation path (perm_q / perm_kv / o_row_map) through the same kernel
    qp, kp, vp = permute.apply_perm_many((q, k, v), perm)
    o2, l2 = block_sparse_attention(qp, kp, vp, kvi, kvn, kvp, *spec, BQ, A, perm_q=perm,
                                    perm_kv=perm, o_row_map=perm, return_lse=True, check=True,
                                    kv_rows=64)
    assert torch.equal(o2, o) and torch.equal(l2, lse)


def test_dead_rows_rows64():
    N = 2048
    q, k, v = _rand(2, N, 128, torch.bfloat16, seed=5)
    o, lse = _run(q, k, v, "far1024+str16", N, 128, 32, kv_rows=64)
    assert (o[:, :1024] == 0).all() and torch.isneginf(lse[:, :1024]).all()
    o_ref, lse_ref = _oracle(q, k, v, "far1024+str16", N)
    _assert_close(o, lse, o_ref, lse_ref)


@pytest.mark.parametrize("name", ["causal", "dilated-8", "window-512"])
def test_running_max_growth_rows64(name):
    N, D, BH = 1024, 128, 2
    g = torch.Generator().manual_seed(11)
    q = 1.0 + 0.1 * torch.randn(BH, N, D, generator=g)
    beta = torch.tensor([0.0, 1.0, 3.0, 9.0]).repeat_interleave(N // 4)
    k = torch.randn(BH, N, D, generator=g) + beta[None, :, None]
    v = torch.randn(BH, N, D, generator=g)
    q, k, v = (t.to(torch.bfloat16).cuda() for t in (q, k, v))
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    for BQ, A in ((128, 128), (128, 32), (64, 64), (16, 16)):
        o, lse = _run(q, k, v, name, N, BQ, A, kv_rows=64)
        _assert_close(o, lse, o_ref, lse_ref)


@pytest.mark.parametrize("N,BQ,A", [(384, 128, 32), (1040, 16, 16), (640, 64, 64),
                                    (1024, 256, 256), (1536, 512, 128), (768, 48, 16)])
def test_ragged_and_large_tiles_rows64(N, BQ, A):
    q, k, v = _rand(3, N, 128, torch.bfloat16, seed=N)
    for name in ("causal", "sinks4+win256", "local64+str8"):
        o, lse = _run(q, k, v, name, N, BQ, A, kv_rows=64)
        o_ref, lse_ref = _oracle(q, k, v, name, N)
        _assert_close(o, lse, o_ref, lse_ref)


def test_config3_rows64_full_size():
    from polyhedral_b200 import attention, blockindex, masks_gpu, permute
    N = 16384
    q, k, v = _gpu_inputs(2, 16, N, 128, 2)
    perm = permute.residue_perm_device(N, 8, q.device)
    m = masks_gpu.numpy_mask("local64+str8")
    dbi = blockindex.build_device(m, N, 128, 32, perm_q=perm, perm_kv=perm)
    o, lse = attention.block_sparse_attention(q, k, v, dbi.kv_idx, dbi.kv_num, dbi.kv_partial,
                                              *m.spec, 128, 32, residue_stride=8,
                                              return_lse=True, check=True, kv_rows=64)
    torch.cuda.synchronize()
    _check_sampled(o, lse, q, k, v, "local64+str8", [0, 31], _sample_rows(N, 64))


def test_config4_rows64_full_size():
    from polyhedral_b200 import attention, blockindex, masks_gpu
    N = 8192
    q, k, v = _gpu_inputs(4, 32, N, 128, 3)
    m = masks_gpu.numpy_mask("sinks4+win512")
    dbi = blockindex.build_device(m, N, 128, 32)
    o, lse = attention.block_sparse_attention(q, k, v, dbi.kv_idx, dbi.kv_num, dbi.kv_partial,
                                              *m.spec, 128, 32, return_lse=True, check=True,
                                              kv_rows=64)
    torch.cuda.synchronize()
    _check_sampled(o, lse, q, k, v, "sinks4+win512", [0, 127], _sample_rows(N, 64))


def test_rows64_argument_errors():
    from polyhedral_b200 import _lib
    N = 1024
    q, k, v = _rand(1, N, 128, torch.bfloat16)
    with pytest.raises(_lib.PolyattnError, match="kv_rows"):
        _run(q, k, v, "causal", N, 128, 32, kv_rows=32)
    o, lse = _run(q, k, v, "causal", N, 128, 32)
    with pytest.raises(_lib.PolyattnError, match="merge"):
        _run(q, k, v, "window-128", N, 128, 32, kv_rows=64, out=o, lse_out=lse, merge=True)
