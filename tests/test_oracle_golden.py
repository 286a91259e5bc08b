"""Pins the CPU oracle to the reference: every oracle function reproduces the
golden vectors the reference's own code produced (tests/golden/make_golden.py)."""
import numpy as np
import pytest
import torch

import oracle as O
from _golden import (attention_c1, attention_small, blockindex_configs, blockindex_small,
                     kernel_math, perms, sha)
from cases import SPECS, oracle_mask


@pytest.mark.parametrize("case", blockindex_small(), ids=lambda c: "{name}-N{N}-{BQ}x{A}-s{s}".format(**c[0]))
def test_block_index_matches_reference_small(case):
    m, kv_idx, kv_num, kv_partial = case
    M = oracle_mask(m["name"], m["N"], m["s"])
    got = O.block_index(M, m["BQ"], m["A"])
    np.testing.assert_array_equal(got[0], kv_idx)
    np.testing.assert_array_equal(got[1], kv_num)
    np.testing.assert_array_equal(got[2], kv_partial)
    assert got[3] == m["elements"] and got[4] == m["live"]


@pytest.mark.parametrize("case", [c for c in blockindex_configs() if c["N"] <= 8192],
                         ids=lambda c: "{config}-{name}-{BQ}x{A}-s{s}".format(**c))
def test_block_index_matches_reference_config_sizes(case):
    M = oracle_mask(case["name"], case["N"], case["s"])
    kv_idx, kv_num, kv_partial, elements, live = O.block_index(M, case["BQ"], case["A"])
    assert sha(kv_idx) == case["kv_idx"]
    assert sha(kv_num) == case["kv_num"]
    assert sha(kv_partial) == case["kv_partial"]
    assert (elements, live) == (case["elements"], case["live"])


@pytest.mark.parametrize("case", perms(), ids=lambda c: f"N{c['N']}-s{c['s']}")
def test_residue_perm_and_invert(case):
    p = O.residue_perm(case["N"], case["s"])
    assert sha(p.astype(np.int32)) == case["perm_sha"]
    inv = O.invert(p)
    assert sha(inv.astype(np.int32)) == case["inv_sha"]
    if case["perm"] is not None:
        assert p.tolist() == case["perm"]
        assert inv.tolist() == case["inv"]


def test_residue_perm_known_answer():
    # gpu/permute.py:12-16 on N=16, s=4
    assert O.residue_perm(16, 4).tolist() == [0, 4, 8, 12, 1, 5, 9, 13, 2, 6, 10, 14, 3, 7, 11, 15]


def _inputs(BH, N, D, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(BH, N, D, generator=g) for _ in range(3)]


def test_attention_matches_reference_small():
    meta, z = attention_small()
    for m in meta:
        q, k, v = _inputs(m["BH"], m["N"], m["D"], m["seed"])
        assert (sha(q.numpy()), sha(k.numpy()), sha(v.numpy())) == (m["q_sha"], m["k_sha"], m["v_sha"])
        M = torch.from_numpy(O.dense_mask(*SPECS[m["name"]], m["N"]))
        if "dead_row" in m:
            M = M.clone()
            M[m["dead_row"]] = False
        o, lse = O.attention(q, k, v, M)
        ref = z[m["key"] + "_o"]
        np.testing.assert_allclose(o.numpy(), ref, atol=1e-6, rtol=1e-5)
        if "dead_row" in m:
            assert np.all(o.numpy()[:, m["dead_row"]] == 0)
            assert np.isneginf(lse.numpy()[:, m["dead_row"]]).all()


def test_attention_matches_reference_config1():
    ref, meta = attention_c1()
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 4, 1024, 64, generator=g).reshape(4, 1024, 64) for _ in range(3))
    assert sha(q.numpy()) == meta["q_sha"]
    M = torch.from_numpy(O.dense_mask(*SPECS["window-128"], 1024))
    o, lse = O.attention_heads(q, k, v, M)
    np.testing.assert_allclose(o.numpy(), ref, atol=1e-6, rtol=1e-5)
    # LSE agrees with a float64 logsumexp of the same masked scores
    s = (q.double() @ k.double().transpose(-1, -2)) * 64 ** -0.5
    s = s.masked_fill(~M[None], float("-inf"))
    np.testing.assert_allclose(lse.numpy(), torch.logsumexp(s, -1).numpy(), atol=1e-5)


def test_online_softmax_matches_reference_kernel_math():
    cases, z = kernel_math()
    from polyhedral_b200 import masks as PM
    rng = np.random.default_rng(0)
    N, D = 256, 16
    q, k, v = (rng.standard_normal((N, D)) for _ in range(3))
    ctor = {"window-64": lambda: PM.SlidingWindow(64), "window-32": lambda: PM.SlidingWindow(32),
            "dilated-8": lambda: PM.Dilated(8), "causal": lambda: PM.Causal()}
    for i, c in enumerate(cases):
        M = ctor[c["name"]]().dense(N)
        got = O.online_softmax_blockwise(M, q, k, v, c["BQ"], c["A"])
        np.testing.assert_allclose(got, z[f"k{i}"], atol=1e-12)


def test_minus_inf_sentinel_is_the_bug():
    """-inf as the running-max start poisons a row dead in its first tile
    (tests/test_kernel_math.py:75-80 pins the same)."""
    from polyhedral_b200 import masks as PM
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((256, 16)) for _ in range(3))
    M = PM.SlidingWindow(64).dense(256)
    assert not np.isfinite(O.online_softmax_blockwise(M, q, k, v, 128, 128, m_init=-np.inf)).all()


def test_lse_merge_of_disjoint_split_equals_union():
    """The merge (compose.py:7-17) reproduces attention over the union."""
    N, D = 512, 32
    q, k, v = _inputs(2, N, D, 11)
    union = O.dense_mask(O.LOCAL_STRIDED, 64, 16, 0, N)
    p1 = O.dense_mask(O.WINDOW, 64, 0, 0, N)
    p2 = O.dense_mask(O.FAR_STRIDED, 64, 16, 0, N)
    assert not (p1 & p2).any() and np.array_equal(p1 | p2, union)
    o1, l1 = O.attention(q, k, v, torch.from_numpy(p1))
    o2, l2 = O.attention(q, k, v, torch.from_numpy(p2))
    ou, lu = O.attention(q, k, v, torch.from_numpy(union))
    o, lse = O.lse_merge(o1.numpy(), l1.numpy(), o2.numpy(), l2.numpy())
    np.testing.assert_allclose(o, ou.numpy(), atol=1e-5)
    np.testing.assert_allclose(lse, lu.numpy(), atol=1e-5)
    # rows dead in part 2 (d < 64 only) take part 1 unchanged
    assert np.isneginf(l2.numpy()[:, :64]).all()
