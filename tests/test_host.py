"""Host-side logic of the product package (no GPU): mask objects, the spec table,
the split decomposition and the host residue permutation, checked against the
oracle and the reference's golden counts."""
import numpy as np
import pytest

import oracle as O
from _golden import counts, perms, sha
from cases import SPECS
from polyhedral_b200 import masks, masks_gpu, permute, split


@pytest.mark.parametrize("name", sorted(masks_gpu.SPECS))
def test_spec_table_matches_oracle_predicate(name):
    kind, p0, p1, p2, ctor = masks_gpu.SPECS[name]
    assert (kind, p0, p1, p2) == SPECS[name]
    m = ctor()
    assert tuple(m.spec) == (kind, p0, p1, p2)
    N = 300
    np.testing.assert_array_equal(m.dense(N), O.dense_mask(kind, p0, p1, p2, N))
    for q in (0, 1, 17, 299):
        np.testing.assert_array_equal(m.row_cols(q, N), O.dense_mask(kind, p0, p1, p2, N)[q])


@pytest.mark.parametrize("name", sorted(masks_gpu.SPECS))
def test_check_agreement(name):
    assert masks_gpu.check_agreement(name, N=256)


@pytest.mark.parametrize("name", sorted(masks_gpu.SPECS))
def test_live_count_closed_form(name):
    m = masks_gpu.numpy_mask(name)
    for N in (1, 7, 100, 512, 1500):
        assert m.live_count(N) == int(m.dense(N).sum()), (name, N)


def test_live_count_matches_reference_counts():
    live = counts()["live"]
    for key, val in live.items():
        name, N = key.split("@")
        if name in masks_gpu.SPECS:
            assert masks_gpu.numpy_mask(name).live_count(int(N)) == val, key


@pytest.mark.parametrize("case", perms(), ids=lambda c: f"N{c['N']}-s{c['s']}")
def test_host_residue_perm(case):
    p = permute.residue_perm(case["N"], case["s"])
    assert p.dtype == np.int32 and sha(p) == case["perm_sha"]


def test_config5_split_is_a_disjoint_cover():
    union = masks.LocalStrided(1024, 16)
    parts = [split.SplitPart(masks.SlidingWindow(1024), 128, 128, 0),
             split.SplitPart(masks.FarStrided(1024, 16), 128, 32, 16)]
    assert split.check_disjoint_cover(union, parts, 3000)
    assert sum(p.mask.live_count(32768) for p in parts) == union.live_count(32768)


def test_config3_split_is_a_disjoint_cover():
    """Band + lattice (configuration 3) = window-64 (identity) + far64+str8 (residue-8)."""
    union = masks.LocalStrided(64, 8)
    parts = [split.SplitPart(masks.SlidingWindow(64), 128, 64, 0, 64),
             split.SplitPart(masks.FarStrided(64, 8), 128, 64, 8)]
    assert split.check_disjoint_cover(union, parts, 3000)
    assert sum(p.mask.live_count(16384) for p in parts) == union.live_count(16384)


def test_split_refuses_64_row_merging_part():
    import pytest
    with pytest.raises(ValueError, match="first part"):
        split.SplitPlan([split.SplitPart(masks.SlidingWindow(64), 128, 64, 0),
                         split.SplitPart(masks.FarStrided(64, 8), 128, 64, 8, 64)], 1024,
                        device="cpu")


def test_flex_mask_mod_far_strided():
    import torch
    M = masks_gpu.dense_bool("far1024+str16", 2048, device="cpu")
    assert not M[:1024].any()
    assert bool(M[1024, 0]) and not bool(M[1025, 0]) and bool(M[2047, 2047 - 1024])
    np.testing.assert_array_equal(M.numpy(), masks.FarStrided(1024, 16).dense(2048))
    assert torch.equal(M, masks_gpu.dense_bool("far1024+str16", 2048, device="cpu"))


def test_report_table(capsys):
    """The drivers' table printer: right-aligned cells, floats with three decimals."""
    from polyhedral_b200 import timing
    timing.report([("a", 1.23456, 7), ("bb", 10.0, 12)], [("x", 4), ("t", 9), ("n", 5)],
                  title="T", note="done")
    out = capsys.readouterr().out.splitlines()
    assert out[1:3] == ["T", "-" * 18]
    assert out[3] == "   x        t    n"
    assert out[4] == "   a    1.235    7"
    assert out[5] == "  bb   10.000   12"
    assert out[-1] == "done"


def test_on_device_switches_only_for_another_device(monkeypatch):
    """Library calls run with the tensors' device current: a no-op context when it is
    current already, torch.cuda.device(index) otherwise."""
    import contextlib
    import torch
    from polyhedral_b200 import _lib
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    assert isinstance(_lib.on_device(torch.device("cuda:0")), contextlib.nullcontext)
    assert isinstance(_lib.on_device("cuda"), contextlib.nullcontext)
    ctx = _lib.on_device(torch.device("cuda", 1))
    assert isinstance(ctx, torch.cuda.device) and ctx.idx == 1
    assert _lib.on_device(3).idx == 3


def test_drop_cached_plan():
    from polyhedral_b200 import attention
    a, b = object(), object()
    attention._PLAN_CACHE.clear()
    attention._PLAN_CACHE[1] = ((), (), a)
    attention._PLAN_CACHE[2] = ((), (), b)
    attention._PLAN_CACHE[3] = ((), (), a)
    attention._drop_cached(a)
    assert list(attention._PLAN_CACHE) == [2]
    attention._PLAN_CACHE.clear()
