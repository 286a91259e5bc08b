"""The sm_100a block-sparse attention kernel vs the CPU oracle (gpu/reference.py
semantics) on identical inputs.

Tolerances: O and LSE within 2e-2 absolute + 1e-2 relative of the fp32 oracle
evaluated on the same (bf16 / fp16) input values; dead rows must be exactly
O = 0 and LSE = -inf.  The reference's own gate uses 3e-3 for fp16 at D = 64
(gpu/test_correctness.py:23); fp16 cases here are held to that as well.
"""
import numpy as np
import pytest
import torch

import oracle as O
from _golden import attention_c1
from cases import SPECS

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
TILES = [(128, 128), (128, 32), (64, 64), (32, 32), (16, 16), (128, 16), (16, 128)]
NAMES = ["causal", "window-128", "dilated-8", "local256+str8", "twoband-1000"]


def _assert_close(o, lse, o_ref, lse_ref, atol=ATOL, rtol=RTOL):
    o = o.float().cpu()
    o_ref = o_ref.float().cpu()
    bad = (o - o_ref).abs() > atol + rtol * o_ref.abs()
    assert not bad.any(), f"O mismatch: max abs err {(o - o_ref).abs().max().item():.3e}"
    if lse is not None:
        lse = lse.float().cpu()
        lse_ref = lse_ref.float().cpu()
        fin = torch.isfinite(lse_ref)
        assert torch.equal(torch.isfinite(lse), fin), "LSE finiteness differs"
        assert (lse[~fin] == lse_ref[~fin]).all()
        d = (lse[fin] - lse_ref[fin]).abs()
        assert (d <= atol + rtol * lse_ref[fin].abs()).all(), f"LSE max err {d.max().item():.3e}"


def _rand(BH, N, D, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(BH, N, D, generator=g).to(dtype).cuda() for _ in range(3)]


def _run(q, k, v, name, N, BQ, A, perm=None, **kw):
    from polyhedral_b200 import blockindex, masks
    from polyhedral_b200.triton_attn import block_sparse_attention
    spec = SPECS[name]
    bi = blockindex.build(masks.from_spec(*spec), N, BQ, A, perm_q=perm, perm_kv=perm)
    kvi, kvn, kvp = blockindex.to_cuda(bi)
    return block_sparse_attention(q, k, v, kvi, kvn, kvp, *spec, BQ, A, perm_q=perm,
                                  perm_kv=perm, return_lse=True, check=True, **kw)


def _oracle(q, k, v, name, N):
    M = torch.from_numpy(O.dense_mask(*SPECS[name], N))
    return O.attention_heads(q.float().cpu(), k.float().cpu(), v.float().cpu(), M)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("name", NAMES)
def test_reference_gate_matrix(name, dtype):
    """gpu/test_correctness.py:47-61: every mask at every tile shape, N=1024, D=64."""
    N, D, BH = 1024, 64, 2
    q, k, v = _rand(BH, N, D, dtype)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    tol = 3e-3 if dtype == torch.float16 else ATOL
    # row_threads: the library's choice (two threads per row at D = 64) and one thread
    for BQ, A in TILES:
        for rt in (0, 1):
            o, lse = _run(q, k, v, name, N, BQ, A, row_threads=rt)
            _assert_close(o, lse, o_ref, lse_ref, atol=tol, rtol=RTOL if tol == ATOL else 0)


@pytest.mark.parametrize("name,s", [("dilated-4", 4), ("dilated-8", 8), ("local64+str8", 8)])
@pytest.mark.parametrize("BQ,A", [(16, 16), (128, 32), (128, 128)])
def test_permuted_path(name, s, BQ, A):
    """gpu/test_correctness.py:63-82: permute Q/K/V, index the permuted mask,
    predicate in original coordinates, inverse-permute O."""
    from polyhedral_b200 import permute
    N, D, BH = 1024, 128, 2
    q, k, v = _rand(BH, N, D, torch.bfloat16, seed=1)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    perm = torch.from_numpy(permute.residue_perm(N, s)).cuda()
    qp, kp, vp = permute.apply_perm_many((q, k, v), perm)
    op, lp = _run(qp, kp, vp, name, N, BQ, A, perm=perm)
    o = op.index_select(1, permute.invert(perm).long())
    lse = lp.index_select(1, permute.invert(perm).long())
    _assert_close(o, lse, o_ref, lse_ref)
    # the fused inverse permutation writes original order directly
    of, lf = _run(qp, kp, vp, name, N, BQ, A, perm=perm, o_row_map=perm)
    assert torch.equal(of, o) and torch.equal(lf, lse)


@pytest.mark.parametrize("name,s,N", [("dilated-4", 4, 1024), ("local64+str8", 8, 2048),
                                      ("far1024+str16", 16, 4096), ("sinks4+win256", 2, 512)])
@pytest.mark.parametrize("BQ,A", [(16, 16), (128, 32), (128, 128)])
def test_residue_stride_equals_explicit_permutation(name, s, N, BQ, A):
    """The on-the-fly residue permutation (strided tensor maps) gives exactly what
    the explicit gather + permuted kernel + inverse scatter gives."""
    from polyhedral_b200 import blockindex, masks, permute
    from polyhedral_b200.triton_attn import block_sparse_attention
    q, k, v = _rand(2, N, 128, torch.bfloat16, seed=s)
    spec = SPECS[name]
    perm = torch.from_numpy(permute.residue_perm(N, s)).cuda()
    bi = blockindex.build(masks.from_spec(*spec), N, BQ, A, perm_q=perm, perm_kv=perm)
    kvi, kvn, kvp = blockindex.to_cuda(bi)
    qp, kp, vp = permute.apply_perm_many((q, k, v), perm)
    o1, l1 = block_sparse_attention(qp, kp, vp, kvi, kvn, kvp, *spec, BQ, A, perm_q=perm,
                                    perm_kv=perm, o_row_map=perm, return_lse=True, check=True)
    o2, l2 = block_sparse_attention(q, k, v, kvi, kvn, kvp, *spec, BQ, A, residue_stride=s,
                                    return_lse=True, check=True)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    _assert_close(o2, l2, o_ref, lse_ref)


def test_residue_stride_argument_errors():
    from polyhedral_b200 import _lib, blockindex, masks, permute
    from polyhedral_b200.triton_attn import block_sparse_attention
    N = 1024
    q, k, v = _rand(1, N, 128, torch.bfloat16)
    perm = torch.from_numpy(permute.residue_perm(N, 4)).cuda()
    bi = blockindex.build(masks.Dilated(4), N, 128, 32, perm_q=perm, perm_kv=perm)
    kvi, kvn, kvp = blockindex.to_cuda(bi)
    with pytest.raises(ValueError):
        block_sparse_attention(q, k, v, kvi, kvn, kvp, 2, 4, 0, 0, 128, 32, residue_stride=4,
                               perm_q=perm)
    with pytest.raises(_lib.PolyattnError, match="multiple of 128"):
        block_sparse_attention(q, k, v, kvi, kvn, kvp, 2, 4, 0, 0, 128, 32, residue_stride=16)


def test_config1_full():
    """Configuration 1: window-128, B1 H4 N1024 D64, fp32 ~N(0,1) seed 0, cast to bf16."""
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 4, 1024, 64, generator=g).reshape(4, 1024, 64) for _ in range(3))
    qb, kb, vb = (x.bfloat16().cuda() for x in (q, k, v))
    for BQ, A in TILES:
        o, lse = _run(qb, kb, vb, "window-128", 1024, BQ, A)
        o_ref, lse_ref = _oracle(qb, kb, vb, "window-128", 1024)
        _assert_close(o, lse, o_ref, lse_ref)
    # against the reference's own fp32 output (inputs differ by the bf16 rounding)
    ref, _ = attention_c1()
    assert (o.float().cpu() - torch.from_numpy(ref)).abs().max().item() < 3e-2


def test_dead_rows_and_all_dead():
    N, D = 2048, 128
    q, k, v = _rand(2, N, D, torch.bfloat16, seed=5)
    o, lse = _run(q, k, v, "far1024+str16", N, 128, 32)
    assert (o[:, :1024] == 0).all() and torch.isneginf(lse[:, :1024]).all()
    o_ref, lse_ref = _oracle(q, k, v, "far1024+str16", N)
    _assert_close(o, lse, o_ref, lse_ref)
    from polyhedral_b200 import blockindex, masks
    from polyhedral_b200.triton_attn import block_sparse_attention
    bi = blockindex.build(masks.FarStrided(4096, 16), N, 128, 32)
    kvi, kvn, kvp = blockindex.to_cuda(bi)
    o, lse = block_sparse_attention(q, k, v, kvi, kvn, kvp, 6, 4096, 16, 0, 128, 32,
                                    return_lse=True, check=True)
    assert (o == 0).all() and torch.isneginf(lse).all()


@pytest.mark.parametrize("name", ["causal", "dilated-8", "window-512"])
def test_running_max_growth(name):
    """Scores that grow from one quarter of the keys to the next by about 16, 49
    and 147 (log2 units): the online softmax has to move its reference max as the
    max grows, including growth far beyond what exponentials taken against the old
    reference can hold."""
    N, D, BH = 1024, 128, 2
    g = torch.Generator().manual_seed(11)
    q = 1.0 + 0.1 * torch.randn(BH, N, D, generator=g)
    beta = torch.tensor([0.0, 1.0, 3.0, 9.0]).repeat_interleave(N // 4)
    k = torch.randn(BH, N, D, generator=g) + beta[None, :, None]
    v = torch.randn(BH, N, D, generator=g)
    q, k, v = (t.to(torch.bfloat16).cuda() for t in (q, k, v))
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    for BQ, A in ((128, 128), (128, 32), (64, 64), (16, 16)):
        o, lse = _run(q, k, v, name, N, BQ, A)
        _assert_close(o, lse, o_ref, lse_ref)


@pytest.mark.parametrize("N,BQ,A", [(384, 128, 32), (1040, 16, 16), (640, 64, 64),
                                    (1024, 256, 256), (1536, 512, 128), (768, 48, 16)])
def test_ragged_and_large_tiles(N, BQ, A):
    q, k, v = _rand(3, N, 128, torch.bfloat16, seed=N)
    for name in ("causal", "sinks4+win256", "local64+str8"):
        o_ref, lse_ref = _oracle(q, k, v, name, N)
        for rt in (0, 1):
            o, lse = _run(q, k, v, name, N, BQ, A, row_threads=rt)
            _assert_close(o, lse, o_ref, lse_ref)


def test_strided_inputs_scale_and_plan_reuse():
    from polyhedral_b200 import attention, blockindex, masks
    N, D = 1024, 128
    base = torch.randn(2, N, 3 * D, device="cuda").bfloat16()
    q, k, v = base[..., :D], base[..., D:2 * D], base[..., 2 * D:]
    bi = blockindex.build_device(masks.SinksWindow(4, 256), N, 128, 32)
    plan = attention.make_plan(bi.kv_idx, bi.kv_num, bi.kv_partial, N, 128, 32)
    M = torch.from_numpy(O.dense_mask(*SPECS["sinks4+win256"], N))
    for scale in (None, 0.05):
        o_ref, lse_ref = O.attention_heads(q.float().cpu(), k.float().cpu(), v.float().cpu(), M,
                                           scale=scale)
        for _ in range(2):
            o, lse = attention.block_sparse_attention(
                q, k, v, None, None, None, *SPECS["sinks4+win256"], 128, 32, scale=scale,
                plan=plan, return_lse=True, check=True)
            _assert_close(o, lse, o_ref, lse_ref)


# ------------------------------------------------------------- full-size configs
def _sampled_oracle(q, k, v, name, heads, rows):
    """fp64 oracle on selected heads / original rows only."""
    N = q.shape[1]
    M = torch.from_numpy(O.dense_mask(*SPECS[name], N, rows=rows))
    outs, lses = [], []
    for h in heads:
        qh = q[h, rows].double().cpu()
        s = (qh @ k[h].double().cpu().T) * q.shape[-1] ** -0.5
        s = s.masked_fill(~M, float("-inf"))
        p = torch.nan_to_num(torch.softmax(s, -1), nan=0.0)
        outs.append(p @ v[h].double().cpu())
        lses.append(torch.logsumexp(s, -1))
    return torch.stack(outs), torch.stack(lses)


def _sample_rows(N, n=96, seed=0):
    rng = np.random.default_rng(seed)
    r = set(rng.choice(N, n, replace=False).tolist()) | {0, 1, 127, 128, N // 2, N - 1}
    return np.array(sorted(r))


def _gpu_inputs(B, H, N, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(B * H, N, D, device="cuda", generator=g).bfloat16() for _ in range(3)]


def _check_sampled(o, lse, q, k, v, name, heads, rows):
    o_ref, lse_ref = _sampled_oracle(q, k, v, name, heads, rows)
    _assert_close(o[heads][:, rows], lse[heads][:, rows], o_ref, lse_ref)


def test_config2_dilated4_rp4_full_size():
    from polyhedral_b200 import blockindex, masks, permute
    from polyhedral_b200.triton_attn import block_sparse_attention
    N = 8192
    q, k, v = _gpu_inputs(1, 16, N, 128, 1)
    perm = permute.residue_perm_device(N, 4)
    bi = blockindex.build_device(masks.Dilated(4), N, 128, 32, perm_q=perm, perm_kv=perm)
    o, lse = block_sparse_attention(q, k, v, bi.kv_idx, bi.kv_num, bi.kv_partial,
                                    *SPECS["dilated-4"], 128, 32, residue_stride=4,
                                    return_lse=True, check=True)
    _check_sampled(o, lse, q, k, v, "dilated-4", [0, 7, 15], _sample_rows(N))


@pytest.mark.parametrize("BQ,A", [(16, 16), (128, 32), (128, 128)])
def test_config3_local64_str8_rp8_full_size(BQ, A):
    from polyhedral_b200 import permute
    N = 16384
    q, k, v = _gpu_inputs(2, 16, N, 128, 2)
    perm = permute.residue_perm_device(N, 8)
    qp, kp, vp = permute.apply_perm_many((q, k, v), perm)
    o, lse = _run(qp, kp, vp, "local64+str8", N, BQ, A, perm=perm, o_row_map=perm)
    _check_sampled(o, lse, q, k, v, "local64+str8", [0, 31], _sample_rows(N, 64))


@pytest.mark.parametrize("A", [32, 128])
def test_config4_sinks_window_full_size(A):
    N = 8192
    q, k, v = _gpu_inputs(4, 32, N, 128, 3)
    o, lse = _run(q, k, v, "sinks4+win512", N, 128, A)
    _check_sampled(o, lse, q, k, v, "sinks4+win512", [0, 64, 127], _sample_rows(N, 64))


def test_config5_split_merge_full_size():
    from polyhedral_b200 import split
    N = 32768
    q, k, v = _gpu_inputs(2, 64, N, 128, 4)
    sp = split.local_strided_split(1024, 16, N, BQ=128, A=32)
    o, lse = sp.run(q, k, v)
    torch.cuda.synchronize()
    _check_sampled(o, lse, q, k, v, "local1024+str16", [0, 127], _sample_rows(N, 48))


@pytest.mark.parametrize("name,N,want", [("dilated-8", 2048, 8), ("local64+str8", 2048, 2),
                                         ("window-128", 1024, 0), ("sinks4+win256", 1024, 0)])
def test_selector_prepare_end_to_end(name, N, want):
    """The selector's executable choice, built and run on the GPU, against the
    oracle on the original mask (inputs and outputs in original order)."""
    from polyhedral_b200 import masks, selector
    m = masks.from_spec(*SPECS[name])
    cp = selector.prepare(m, N, 128, 32)
    assert cp.stride == want
    q, k, v = _rand(2, N, 128, torch.bfloat16, seed=N + want)
    o, lse = cp.run(q, k, v)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    _assert_close(o, lse, o_ref, lse_ref)


@pytest.mark.parametrize("name,N,A", [("local64+str8", 2048, 64), ("local256+str8", 4096, 32)])
def test_selector_prepare_split_end_to_end(name, N, A):
    """allow_split: band + lattice unions come back as a split (window part on the
    64-row kernel, lattice part in its residue basis merging in its epilogue),
    against the oracle on the union mask."""
    from polyhedral_b200 import masks, selector
    m = masks.from_spec(*SPECS[name])
    sc = selector.prepare(m, N, 128, A, allow_split=True)
    assert isinstance(sc, selector.SplitChoice), sc
    assert [p.stride for p in sc.plan.parts] == [0, 8]
    q, k, v = _rand(2, N, 128, torch.bfloat16, seed=N + A)
    o, lse = sc.run(q, k, v)
    o_ref, lse_ref = _oracle(q, k, v, name, N)
    _assert_close(o, lse, o_ref, lse_ref)
    # without allow_split the same call keeps the single class A basis
    assert not isinstance(selector.prepare(m, N, 128, A), selector.SplitChoice)


@pytest.mark.parametrize("name,N", [("dilated-4", 8192), ("local64+str8", 16384),
                                    ("window-128", 1024), ("local256+str8", 4096)])
def test_selector_device_costs_equal_closed_form(name, N):
    """Class-A costs measured by building each candidate's block index on the GPU
    equal the selector's closed forms, integer for integer."""
    from polyhedral_b200 import masks, selector
    m = masks.from_spec(*SPECS[name])
    for BQ, A in ((128, 32), (128, 128), (16, 16)):
        dev = selector.costs_device(m, N, BQ, A)
        host = {k: v for k, v in selector.costs(m, N, BQ, A).items()
                if not selector.is_class_b(k)}
        assert dev == host, (BQ, A)
    # a mask that is not diagonally invariant still gets device costs
    sk = masks.SinksWindow(4, 512)
    assert selector.costs(sk, 8192, 128, 32) is None
    assert selector.costs_device(sk, 8192, 128, 32)["identity"] == 5320704


@pytest.mark.parametrize("kv_rows", [0, 64])
def test_sched_heads_groups_give_identical_results(kv_rows):
    """Scheduling the work items in head groups (sched_heads) changes the order of
    the items only: every output bit is the same, ragged last group included."""
    N, BH = 2048, 5
    q, k, v = _rand(BH, N, 128, torch.bfloat16, seed=77)
    ref = _run(q, k, v, "local256+str8", N, 128, 32, kv_rows=kv_rows)
    for g in (1, 2, 3, BH, 64):
        o, lse = _run(q, k, v, "local256+str8", N, 128, 32, kv_rows=kv_rows, sched_heads=g)
        assert torch.equal(o, ref[0]) and torch.equal(lse, ref[1]), g


def test_stream_handle_follows_current_stream():
    """Every launch goes to torch's current stream, also inside a stream context and
    for every way of naming the device."""
    from polyhedral_b200 import _lib
    dev = torch.device("cuda:0")
    # (a NULL handle, the default stream, reads back as None through ctypes)
    assert (_lib.stream_handle().value or 0) == torch.cuda.current_stream().cuda_stream
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for d in (None, 0, dev, torch.device("cuda"), "cuda:0"):
            assert (_lib.stream_handle(d).value or 0) == s.cuda_stream, d
        q, k, v = _rand(1, 1024, 128, torch.bfloat16, seed=3)
        o, lse = _run(q, k, v, "causal", 1024, 128, 32)
    torch.cuda.synchronize()
    o_ref, lse_ref = _oracle(q, k, v, "causal", 1024)
    _assert_close(o, lse, o_ref, lse_ref)


def test_plan_cache():
    """set_plan_cache(True): a call without ``plan`` reuses the work list of an earlier
    call with the same index tensors (unchanged since) on the same stream; an in-place
    change of an index tensor, or another stream, builds a new one; the results are
    those of calls without the cache."""
    from polyhedral_b200 import attention, blockindex, masks
    from polyhedral_b200.triton_attn import block_sparse_attention
    N = 1024
    q, k, v = _rand(2, N, 128, torch.bfloat16, seed=8)
    spec = SPECS["window-128"]
    kvi, kvn, kvp = blockindex.to_cuda(blockindex.build(masks.from_spec(*spec), N, 128, 32))
    ref = block_sparse_attention(q, k, v, kvi, kvn, kvp, *spec, 128, 32, return_lse=True)
    attention.set_plan_cache(True)
    try:
        for _ in range(3):
            o, lse = block_sparse_attention(q, k, v, kvi, kvn, kvp, *spec, 128, 32,
                                            return_lse=True, check=True)
            assert torch.equal(o, ref[0]) and torch.equal(lse, ref[1])
        assert len(attention._PLAN_CACHE) == 1
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            o, lse = block_sparse_attention(q, k, v, kvi, kvn, kvp, *spec, 128, 32,
                                            return_lse=True, check=True)
        torch.cuda.synchronize()
        assert torch.equal(o, ref[0]) and len(attention._PLAN_CACHE) == 2
        kvn.zero_()            # no listed tile for any row: every row dead
        o, lse = block_sparse_attention(q, k, v, kvi, kvn, kvp, *spec, 128, 32,
                                        return_lse=True, check=True)
        assert (o == 0).all() and torch.isneginf(lse).all()
        assert len(attention._PLAN_CACHE) == 2      # the stale entry was replaced
    finally:
        attention.set_plan_cache(False)
    assert len(attention._PLAN_CACHE) == 0
