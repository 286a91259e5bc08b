"""GPU LSE merge vs the oracle merge, and the split path vs attention over the
union mask."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [40, 64, 128])
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


@pytest.mark.parametrize("A1,kv1,A2", [(64, 64, 64), (32, 64, 128), (16, 0, 32), (64, "rt2", 64)])
def test_band_lattice_split_equals_union(A1, kv1, A2):
    """Configuration 3's split: window-64 (identity; the 64-row kernel writes O/LSE)
    + far64+str8 (residue-8 applied by the kernel, merging in its epilogue) equals
    attention over local64+str8."""
    from polyhedral_b200 import masks, split
    N, D, BH = 2048, 128, 2
    g = torch.Generator().manual_seed(13)
    q, k, v = (torch.randn(BH, N, D, generator=g).bfloat16().cuda() for _ in range(3))
    if kv1 == "rt2":     # window part with two softmax threads per row
        sp = split.SplitPlan([split.SplitPart(masks.SlidingWindow(64), 128, A1, 0, 0, 2),
                              split.SplitPart(masks.FarStrided(64, 8), 128, A2, 8)], N)
    else:
        sp = split.local_strided_split(64, 8, N, BQ=128, A=A2, A_window=A1, window_kv_rows=kv1)
    o, lse = sp.run(q, k, v)
    M = torch.from_numpy(O.dense_mask(O.LOCAL_STRIDED, 64, 8, 0, N))
    o_ref, lse_ref = O.attention_heads(q.float().cpu(), k.float().cpu(), v.float().cpu(), M)
    err = (o.float().cpu() - o_ref).abs()
    assert (err <= 2e-2 + 1e-2 * o_ref.abs()).all(), err.max()
    assert (lse.cpu() - lse_ref).abs().max().item() < 2e-2


def _union_ref(q, k, v, M):
    return O.attention_heads(q.float().cpu(), k.float().cpu(), v.float().cpu(),
                             torch.from_numpy(M))


def _part(q, k, v, mask, N, BQ, A, stride=0, **kw):
    from polyhedral_b200 import attention, blockindex, permute
    perm = permute.residue_perm_device(N, stride, q.device) if stride else None
    dbi = blockindex.build_device(mask, N, BQ, A, perm_q=perm, perm_kv=perm, device=q.device)
    kind, p0, p1, p2 = mask.spec
    return attention.block_sparse_attention(q, k, v, dbi.kv_idx, dbi.kv_num, dbi.kv_partial,
                                            kind, p0, p1, p2, BQ, A, residue_stride=stride,
                                            return_lse=True, check=True, **kw)


@pytest.mark.parametrize("stride2", [0, 8])
@pytest.mark.parametrize("BQ,A", [(128, 32), (128, 128), (64, 64), (16, 16)])
def test_fused_merge_matches_union(stride2, BQ, A):
    """Part 2 merged into part 1 by the attention epilogue equals attention over
    the union mask; rows dead in part 1 (far band) and rows dead in both."""
    from polyhedral_b200 import masks
    N, D, BH = 2048, 128, 2
    g = torch.Generator().manual_seed(21)
    q, k, v = (torch.randn(BH, N, D, generator=g).bfloat16().cuda() for _ in range(3))
    p1, p2 = masks.FarStrided(1024, 8), masks.SlidingWindow(256)
    if stride2:   # part 2 in a residue basis: the far lattice band
        p1, p2 = masks.SlidingWindow(256), masks.FarStrided(1024, 8)
    o, lse = _part(q, k, v, p1, N, BQ, A)
    _part(q, k, v, p2, N, BQ, A, stride2, out=o, lse_out=lse, merge=True)
    M = p1.dense(N) | p2.dense(N)
    o_ref, lse_ref = _union_ref(q, k, v, M)
    assert (o.float().cpu() - o_ref).abs().max().item() < 2e-2
    fin = torch.isfinite(lse_ref)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    assert (lse.cpu()[fin] - lse_ref[fin]).abs().max().item() < 2e-2
    # both parts dead: rows where neither mask has a live key stay O = 0, LSE = -inf
    q2 = q[:, :512].contiguous()
    k2, v2 = k[:, :512].contiguous(), v[:, :512].contiguous()
    far, far2 = masks.FarStrided(600, 8), masks.FarStrided(700, 4)
    o, lse = _part(q2, k2, v2, far, 512, 128, 32)
    _part(q2, k2, v2, far2, 512, 128, 32, out=o, lse_out=lse, merge=True)
    assert (o == 0).all() and torch.isneginf(lse).all()


@pytest.mark.parametrize("w,s,A1,A2", [(1024, 16, 128, 64), (256, 16, 128, 64), (64, 8, 64, 64)])
def test_c5_shaped_split_rp16_merging(w, s, A1, A2):
    """Configuration 5's split shapes at N = 4096: the window part at 128 x A1 in the
    identity basis writes O / LSE, then the far lattice at 128 x 64 in the residue-s
    basis merges into them in its epilogue; against the union mask."""
    from polyhedral_b200 import masks
    N, D, BH = 4096, 128, 2
    g = torch.Generator().manual_seed(w + s)
    q, k, v = (torch.randn(BH, N, D, generator=g).bfloat16().cuda() for _ in range(3))
    p1, p2 = masks.SlidingWindow(w), masks.FarStrided(w, s)
    o, lse = _part(q, k, v, p1, N, 128, A1)
    _part(q, k, v, p2, N, 128, A2, s, out=o, lse_out=lse, merge=True)
    o_ref, lse_ref = _union_ref(q, k, v, p1.dense(N) | p2.dense(N))
    err = (o.float().cpu() - o_ref).abs()
    assert (err <= 2e-2 + 1e-2 * o_ref.abs()).all(), err.max()
    fin = torch.isfinite(lse_ref)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    assert (lse.cpu()[fin] - lse_ref[fin]).abs().max().item() < 2e-2


def test_fused_merge_equals_merge_kernel():
    """The fused merge and attention + pa_lse_merge agree within one bf16 rounding
    (the fused path merges this part's fp32 result before rounding)."""
    from polyhedral_b200 import masks, merge
    N, D, BH = 1024, 64, 3
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(BH, N, D, generator=g).bfloat16().cuda() for _ in range(3))
    a, b = masks.SlidingWindow(100), masks.FarStrided(100, 4)
    o1, l1 = _part(q, k, v, a, N, 128, 32)
    o2, l2 = _part(q, k, v, b, N, 128, 32)
    ref_o, ref_l = merge.lse_merge(o1, l1, o2, l2)
    o, lse = o1.clone(), l1.clone()
    _part(q, k, v, b, N, 128, 32, out=o, lse_out=lse, merge=True)
    assert (o.float() - ref_o.float()).abs().max().item() < 1.6e-2
    assert (lse - ref_l).abs().max().item() < 1e-5


def test_fused_merge_argument_errors():
    from polyhedral_b200 import _lib, masks
    N = 512
    q, k, v = (torch.zeros(1, N, 128, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    with pytest.raises(ValueError):
        _part(q, k, v, masks.Causal(), N, 128, 32, merge=True)


def test_reference_style_driver_runs_on_the_dropin(tmp_path):
    """A driver written the way the reference's gpu/exp*.py are (bare-name imports,
    bench.time_ms / report, identity vs residue-permuted run) runs through
    ``python -m polyhedral_b200.dropin`` and agrees with itself across the
    permutation."""
    import subprocess
    import sys
    import textwrap
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    script = tmp_path / "driver.py"
    script.write_text(textwrap.dedent("""
        import sys
        sys.path.insert(0, __file__.rsplit("/", 1)[0])
        import torch
        import blockindex, bench, masks_gpu, permute
        from triton_attn import block_sparse_attention
        N, D, BH, name, s = 2048, 64, 4, "dilated-8", 8
        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(BH, N, D, generator=g).half().cuda() for _ in range(3))
        m, spec = masks_gpu.numpy_mask(name), masks_gpu.triton_params(name)
        rows = []
        for BQ, A in ((128, 128), (16, 16)):
            kvi, kvn, kvp = blockindex.to_cuda(blockindex.build(m, N, BQ, A))
            f0 = lambda: block_sparse_attention(q, k, v, kvi, kvn, kvp, *spec, BQ, A,
                                                num_warps=4, num_stages=2)
            p = torch.from_numpy(permute.residue_perm(N, s)).cuda()
            pk = blockindex.to_cuda(blockindex.build(m, N, BQ, A, perm_q=p, perm_kv=p))
            qp, kp, vp = (permute.apply_perm(x, p) for x in (q, k, v))
            f1 = lambda: block_sparse_attention(qp, kp, vp, *pk, *spec, BQ, A, perm_q=p)
            o0 = f0()
            o1 = f1().index_select(1, permute.invert(p).long())
            err = (o0.float() - o1.float()).abs().max().item()
            assert err < 1e-2, err
            t0, _ = bench.time_ms(f0, warmup=3, reps=10)
            t1, _ = bench.time_ms(f1, warmup=3, reps=10)
            rows.append((f"{BQ}x{A}", t0, t1))
        bench.report(rows, [("tile", 8), ("identity", 10), ("rp8", 10)], title="driver")
        print("DRIVER OK")
    """))
    r = subprocess.run([sys.executable, "-m", "polyhedral_b200.dropin", str(script)], cwd=root,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "DRIVER OK" in r.stdout
