"""Selector (host policy) against the reference's own answers: every cost table
and every select() result in tests/golden/counts.json was produced by
src/polyattn/selector.py:210-264 on the same masks, lengths and tile shapes."""
import itertools

import numpy as np
import pytest

from polyhedral_b200 import masks, masks_gpu, selector
from _golden import counts

COUNTS = counts()


def _key(key):
    name, rest = key.split("@")
    N, tile = rest.split(":")
    BQ, A = (int(x) for x in tile.split("x"))
    return name, int(N), BQ, A


@pytest.mark.parametrize("key", sorted(COUNTS["selector"]))
def test_costs_match_reference(key):
    name, N, BQ, A = _key(key)
    got = selector.costs(masks_gpu.numpy_mask(name), N, BQ, A)
    assert got == COUNTS["selector"][key]


@pytest.mark.parametrize("key", sorted(COUNTS["select"]))
def test_select_matches_reference(key):
    name, N, BQ, A = _key(key)
    assert selector.select(masks_gpu.numpy_mask(name), N, BQ, A) == COUNTS["select"][key]


def test_sinks_is_not_invariant():
    assert selector.offsets_of(masks.SinksWindow(4, 512), 1024) is None
    assert selector.costs(masks.SinksWindow(4, 512), 1024, 128, 32) is None


def test_identity_cost_equals_block_index_elements():
    """tile_cost is the element count a tiled block index lists: check it
    against a brute-force tiling of the dense mask at small N."""
    N = 256
    for m, (BQ, A) in itertools.product(
            [masks.Causal(), masks.SlidingWindow(40), masks.Dilated(3), masks.LocalStrided(16, 5),
             masks.TwoBand(8, 100, 16), masks.FarStrided(32, 4)],
            [(16, 16), (32, 8), (64, 32), (128, 128)]):
        M = m.dense(N)
        tiles = M.reshape(N // BQ, BQ, N // A, A).any(axis=(1, 3)).sum()
        runs = selector.offsets_of(m, N)
        assert selector.tile_cost(runs, N, BQ, A) == tiles * BQ * A, (m, BQ, A)


def test_residue_cost_equals_permuted_tiling():
    """The block decomposition equals tiling the explicitly permuted mask."""
    from polyhedral_b200 import permute
    N = 512
    for m, s, (BQ, A) in itertools.product(
            [masks.Dilated(4), masks.LocalStrided(16, 8), masks.SlidingWindow(24)],
            [2, 4, 8], [(16, 16), (32, 16), (64, 32)]):
        if (N // s) % BQ or (N // s) % A:
            continue
        p = permute.residue_perm(N, s)
        M = m.dense(N)[np.ix_(p, p)]
        tiles = M.reshape(N // BQ, BQ, N // A, A).any(axis=(1, 3)).sum()
        got = selector.costs(m, N, BQ, A)[f"residue-perm-{s}"]
        assert got == tiles * BQ * A, (m, s, BQ, A)


def test_ragged_refused():
    with pytest.raises(selector.RaggedNotSupported):
        selector.costs(masks.Causal(), 1000, 128, 32)


def test_select_class_a_configs():
    """What the kernel runs for the benchmark configurations: c2 -> rp4 (the
    reference's argmin at 128x32 is class-B stridefold-4), c3 -> rp8, c4 ->
    identity (not diagonally invariant)."""
    sa = selector.select_class_a
    assert sa(masks_gpu.numpy_mask("dilated-4"), 8192, 128, 32) == ("residue-perm-4", 4)
    assert selector.select(masks_gpu.numpy_mask("dilated-4"), 8192, 128, 32) == "stridefold-4"
    assert sa(masks_gpu.numpy_mask("local64+str8"), 16384, 128, 32) == ("residue-perm-8", 8)
    assert sa(masks_gpu.numpy_mask("sinks4+win512"), 8192, 128, 32) == ("identity", 0)
    assert sa(masks.FarStrided(1024, 16), 32768, 128, 32)[1] == 16


def test_select_split_configs():
    """Band + lattice unions of configurations 3 and 5: the split into the band
    (identity) and the lattice beyond it (its residue basis) computes far fewer
    tiles than any single executable basis."""
    c3 = selector.select_split(masks_gpu.numpy_mask("local64+str8"), 16384, 128, 64)
    assert c3["split"] and c3["single"][:2] == ("residue-perm-8", 8)
    assert [(p[0].name, p[1], p[2]) for p in c3["parts"]] == [
        ("window-64", "identity", 0), ("far64+str8", "residue-perm-8", 8)]
    assert sum(p[3] for p in c3["parts"]) < 0.6 * c3["single"][2]
    c5 = selector.select_split(masks_gpu.numpy_mask("local1024+str16"), 32768, 128, 64)
    assert c5["split"] and c5["parts"][1][1:3] == ("residue-perm-16", 16)
    assert selector.select_split(masks.Dilated(4), 1024, 128, 32) is None
    assert selector.select_split(masks_gpu.numpy_mask("sinks4+win512"), 1024, 128, 32) is None


def test_select_split_part_costs_equal_tilings():
    """Each part's cost is the tiling of that part in its basis, brute force."""
    from polyhedral_b200 import permute
    N = 1024
    for (w, s), (BQ, A) in itertools.product([(64, 8), (16, 4), (100, 8)],
                                             [(128, 32), (16, 16), (64, 64)]):
        c = selector.select_split(masks.LocalStrided(w, s), N, BQ, A)
        assert c["single"][2] == selector.costs(masks.LocalStrided(w, s), N, BQ, A)[c["single"][0]]
        for part, name, stride, elems in c["parts"]:
            M = part.dense(N)
            if stride:
                p = permute.residue_perm(N, stride)
                M = M[np.ix_(p, p)]
            tiles = M.reshape(N // BQ, BQ, N // A, A).any(axis=(1, 3)).sum()
            assert elems == tiles * BQ * A, (w, s, BQ, A, part.name)
        live = sum(int(p[0].dense(N).sum()) for p in c["parts"])
        assert live == int(masks.LocalStrided(w, s).dense(N).sum())
