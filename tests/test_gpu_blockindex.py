"""GPU block-index builder vs the reference (bit-exact): the golden arrays of
every small case and the SHA-256 of the full-size configuration indices."""
import numpy as np
import pytest
import torch

import oracle as O
from _golden import blockindex_configs, blockindex_small, sha
from cases import SPECS

pytestmark = pytest.mark.gpu


def _build(name, N, BQ, A, s, dense=False):
    from polyhedral_b200 import blockindex, masks
    spec = SPECS[name]
    if dense:
        M = O.dense_mask(*spec, N)
        if s:
            M = O.permuted_mask(M, O.residue_perm(N, s))

        class _Dense:
            def row_cols(self, q, N_):
                return M[q]
        return blockindex.build(_Dense(), N, BQ, A)
    perm = O.residue_perm(N, s) if s else None
    return blockindex.build(masks.from_spec(*spec), N, BQ, A, perm_q=perm, perm_kv=perm)


@pytest.mark.parametrize("case", blockindex_small(),
                         ids=lambda c: "{name}-N{N}-{BQ}x{A}-s{s}".format(**c[0]))
def test_block_index_small(case):
    m, kv_idx, kv_num, kv_partial = case
    bi = _build(m["name"], m["N"], m["BQ"], m["A"], m["s"])
    np.testing.assert_array_equal(bi.kv_idx, kv_idx)
    np.testing.assert_array_equal(bi.kv_num, kv_num)
    np.testing.assert_array_equal(bi.kv_partial, kv_partial)
    assert (bi.elements, bi.live) == (m["elements"], m["live"])


@pytest.mark.parametrize("case", blockindex_small()[::7],
                         ids=lambda c: "{name}-N{N}-{BQ}x{A}-s{s}".format(**c[0]))
def test_block_index_dense_path(case):
    m, kv_idx, kv_num, kv_partial = case
    bi = _build(m["name"], m["N"], m["BQ"], m["A"], m["s"], dense=True)
    np.testing.assert_array_equal(bi.kv_idx, kv_idx)
    np.testing.assert_array_equal(bi.kv_partial, kv_partial)
    assert (bi.elements, bi.live) == (m["elements"], m["live"])


@pytest.mark.parametrize("case", blockindex_configs(),
                         ids=lambda c: "{config}-{name}-{BQ}x{A}-s{s}".format(**c))
def test_block_index_full_size_configs(case):
    bi = _build(case["name"], case["N"], case["BQ"], case["A"], case["s"])
    assert bi.kv_idx.shape[1] == case["max_kv"]
    assert sha(bi.kv_idx) == case["kv_idx"]
    assert sha(bi.kv_num) == case["kv_num"]
    assert sha(bi.kv_partial) == case["kv_partial"]
    assert (bi.elements, bi.live) == (case["elements"], case["live"])


def test_device_index_padding_and_stats():
    from polyhedral_b200 import blockindex, masks
    dbi = blockindex.build_device(masks.SlidingWindow(128), 1024, 128, 32)
    torch.cuda.synchronize()
    num = dbi.kv_num.cpu().numpy()
    idx = dbi.kv_idx.cpu().numpy()
    for i, n in enumerate(num):
        assert (idx[i, n:] == 0).all()
        assert (np.diff(idx[i, :n]) > 0).all()
    st = dbi.stats.cpu().tolist()
    assert st[2] == num.max() and st[3] == num.sum()


def test_all_dead_mask_gives_empty_index():
    from polyhedral_b200 import blockindex, masks
    bi = blockindex.build(masks.FarStrided(4096, 16), 1024, 128, 32)
    assert bi.kv_idx.shape == (8, 0) and (bi.kv_num == 0).all()
    assert bi.elements == 0 and bi.live == 0
