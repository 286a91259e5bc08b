"""Transform selector: which row/column reordering makes a mask cheapest to tile,
decided from the predicate alone -- the host policy of the reference's
``src/polyattn/selector.py:210-264`` (``costs`` / ``select``).

Nothing here builds the N x N mask.  A mask whose liveness depends only on the
diagonal offset d = q - kv is summarised by its offset set D as a few sorted
runs of consecutive offsets (read from one row, then checked on a handful of
others: ``offsets_of``).  Every cost is then exact arithmetic on those runs:

* identity: tile (I, J) of a BQ x A tiling sees exactly the offsets
  [v - A + 1, v + BQ - 1] with v = I*BQ - J*A, so it is listed iff D meets that
  window.  The elements computed are BQ*A times the number of tile pairs whose
  v lies in the union of the widened runs; for each such v (a multiple of
  g = gcd(BQ, A)) the pairs form one residue class of I, counted in closed form.
* residue-perm-s (class A, what this library's kernel runs): sorting both axes
  by (i mod s, i div s) turns the mask into an s x s grid of (N/s)-square
  blocks; block (c1, c2) is diagonally invariant with offsets
  {w : w*s + (c1 - c2) in D}, and s - |c1 - c2| blocks share each difference.
  Exact only when the tiles nest in the blocks (N/s divisible by BQ and A);
  otherwise the candidate is left out.
* shear and stridefold-s (class B: a per-query gather, costed so that the
  selector's answer matches the reference's, but not executed here): the mask
  becomes an N x width staircase in which column c holds one offset d and is
  live for rows q >= d; a column block is live from the first row block that
  reaches its smallest offset.

``select`` returns the reference's answer (ties broken towards class A, then
by candidate order); ``select_class_a`` restricts the choice to what the
kernel executes and returns the residue stride to pass as ``residue_stride``;
``prepare`` builds everything the forward needs for that choice on the GPU.

``select_split`` adds the composition the reference only counts
(src/polyattn/experiments/compose.py:1-24, 36-44): a band + lattice union
LocalStrided(w, s) is the disjoint union of SlidingWindow(w) and FarStrided(w, s);
each part takes its own cheapest executable basis, and the split wins when its
elements are fewer than the best single basis' by more than ``SPLIT_MARGIN``
(the merge is fused into the second part's epilogue, but it rereads O and LSE).
``prepare(..., allow_split=True)`` then builds a ``split.SplitPlan``.
"""
from math import gcd

import numpy as np

__all__ = ["CANDIDATES", "RaggedNotSupported", "offsets_of", "tile_cost", "costs",
           "select", "select_class_a", "is_class_b", "stride_of", "prepare", "ClassAPlan",
           "costs_device", "select_split", "SPLIT_MARGIN"]

# A split must compute this fraction fewer elements than the best single basis.
SPLIT_MARGIN = 0.10

CANDIDATES = (["identity", "shear"]
              + [f"stridefold-{s}" for s in (2, 4, 8)]
              + [f"residue-perm-{s}" for s in (2, 3, 4, 6, 8, 12, 16, 32)])

# Offsets expanded one by one (class B staircases) above this many are not costed.
_EXPAND_CAP = 1 << 22


class RaggedNotSupported(NotImplementedError):
    """N not divisible by the tile sides: the closed forms bill whole tiles at
    the ragged edge, so no cost is returned rather than a slightly wrong one."""


def _runs(sorted_vals):
    """Sorted distinct integers -> inclusive runs [(lo, hi), ...]."""
    v = np.asarray(sorted_vals, dtype=np.int64)
    if v.size == 0:
        return []
    cut = np.flatnonzero(np.diff(v) != 1)
    lo = np.concatenate(([v[0]], v[cut + 1]))
    hi = np.concatenate((v[cut], [v[-1]]))
    return [(int(a), int(b)) for a, b in zip(lo, hi)]


def _union(runs):
    """Merge overlapping or touching runs."""
    out = []
    for lo, hi in sorted(runs):
        if out and lo <= out[-1][1] + 1:
            out[-1][1] = max(out[-1][1], hi)
        else:
            out.append([lo, hi])
    return [(a, b) for a, b in out]


def offsets_of(mask, N, checks=6):
    """The diagonal offset set of `mask` at length N as sorted runs, or None when
    the mask is not diagonally invariant.  Reads the last row (which sees every
    offset 0..N-1) and confirms on `checks` rows spread over [N/4, N-2] that each
    row q is exactly {q - d : d in D, d <= q}."""
    last = np.asarray(mask.row_cols(N - 1, N), dtype=bool)
    d = np.sort((N - 1) - np.flatnonzero(last))
    if d.size == 0:
        return []
    for q in np.linspace(N // 4, N - 2, checks).astype(int):
        q = int(q)
        expect = np.zeros(N, dtype=bool)
        expect[q - d[d <= q]] = True
        if not np.array_equal(expect, np.asarray(mask.row_cols(q, N), dtype=bool)):
            return None
    return _runs(d)


def _pairs_at(v, N, BQ, A, g):
    """For each offset v (multiples of g), the number of tile pairs (I, J) with
    I*BQ - J*A = v, 0 <= I < N/BQ, 0 <= J < N/A."""
    v = np.asarray(v, dtype=np.int64)
    # J = (I*BQ - v) / A must be an integer in [0, N/A): I*BQ in [v, v + N - A]
    i_lo = np.maximum(0, -((-v) // BQ))
    i_hi = np.minimum(N // BQ - 1, (v + N - A) // BQ)
    m = A // g                       # I*BQ = v (mod A)  <=>  I = i0 (mod m)
    if m == 1:
        i0 = np.zeros_like(v)
    else:
        i0 = ((v // g) % m) * pow((BQ // g) % m, -1, m) % m
    first = i_lo + (i0 - i_lo) % m
    return np.where(first > i_hi, 0, (i_hi - first) // m + 1)


def tile_cost(runs, N, BQ, A):
    """Elements computed (BQ*A per listed tile) by a BQ x A tiling of the
    diagonally invariant mask with offset runs `runs`; None when N is ragged."""
    if not runs:
        return 0
    if N % BQ or N % A:
        return None
    g = gcd(BQ, A)
    total = 0
    for lo, hi in _union([(a - BQ + 1, b + A - 1) for a, b in runs]):
        first = -((-lo) // g) * g
        if first > hi:
            continue
        total += int(_pairs_at(np.arange(first, hi + 1, g, dtype=np.int64), N, BQ, A, g).sum())
    return total * BQ * A


def _class_runs(runs, s, delta):
    """Runs of {w : w*s + delta in D} for the offset runs of D."""
    out = []
    for lo, hi in runs:
        a = -((-(lo - delta)) // s)
        b = (hi - delta) // s
        if a <= b:
            out.append((a, b))
    return _union(out)


def _cost_residue(runs, N, s, BQ, A):
    if N % s:
        return None
    nb = N // s
    if nb % BQ or nb % A:
        return None
    total = 0
    for delta in range(1 - s, s):
        sub = _class_runs(runs, s, delta)
        if sub:
            total += (s - abs(delta)) * tile_cost(sub, nb, BQ, A)
    return total


def _expand(runs):
    if sum(b - a + 1 for a, b in runs) > _EXPAND_CAP:
        return None
    return np.concatenate([np.arange(a, b + 1, dtype=np.int64) for a, b in runs])


def _staircase(d, N, BQ, A, width, column):
    """Elements of the N x width staircase in which the column of offset d is
    column(d) and is live for rows q >= d; the last column block is billed at
    its true width."""
    cols = column(d)
    blocks = cols // A
    nblk = int(blocks.max()) + 1
    dmin = np.full(nblk, np.iinfo(np.int64).max, dtype=np.int64)
    np.minimum.at(dmin, blocks, d)
    present = dmin != np.iinfo(np.int64).max
    b = np.flatnonzero(present)
    dm = dmin[present]
    i_first = np.maximum(0, -((-(dm - BQ + 1)) // BQ))
    rows = np.maximum(0, N // BQ - i_first)
    widths = np.minimum(A, width - b * A)
    return int((rows * BQ * widths).sum())


def _cost_shear(runs, N, BQ, A):
    d = _expand(runs)
    if d is None:
        return None
    dmax = int(d[-1])
    return _staircase(d, N, BQ, A, dmax - int(d[0]) + 1, lambda x: dmax - x)


def _cost_stridefold(runs, N, s, BQ, A):
    d = _expand(runs)
    if d is None or d[0] < 0 or np.any(d % s):
        return None
    return _staircase(d, N, BQ, A, int(d[-1]) // s + 1, lambda x: x // s)


def stride_of(name):
    """The stride s of 'residue-perm-s' / 'stridefold-s', 0 for the others."""
    return int(name.rsplit("-", 1)[1]) if name[-1].isdigit() else 0


def is_class_b(name):
    """Class B (shear, stridefold) gathers per query block; class A permutes once."""
    return name == "shear" or name.startswith("stridefold-")


def costs(mask, N, BQ, A, runs=None):
    """{candidate: elements computed} for every candidate that applies, or None
    when the mask is not diagonally invariant.  Raises RaggedNotSupported when
    N is not a multiple of BQ and A."""
    if N % BQ or N % A:
        raise RaggedNotSupported(f"N={N} is not a multiple of BQ={BQ} and A={A}")
    if runs is None:
        runs = offsets_of(mask, N)
    if runs is None:
        return None
    out = {}
    for name in CANDIDATES:
        s = stride_of(name)
        if name == "identity":
            c = tile_cost(runs, N, BQ, A)
        elif name == "shear":
            c = _cost_shear(runs, N, BQ, A) if runs else 0
        elif name.startswith("stridefold-"):
            c = _cost_stridefold(runs, N, s, BQ, A) if runs else 0
        else:
            c = _cost_residue(runs, N, s, BQ, A)
        if c is not None:
            out[name] = c
    return out


def _rank(c):
    return lambda k: (c[k], is_class_b(k), CANDIDATES.index(k))


def select(mask, N, BQ, A):
    """The candidate with the fewest elements; on equal counts class A wins, then
    candidate order.  'identity' for a mask that is not diagonally invariant."""
    c = costs(mask, N, BQ, A)
    if not c:
        return "identity"
    return min(c, key=_rank(c))


def select_class_a(mask, N, BQ, A):
    """(name, residue_stride) of the cheapest candidate this library executes:
    identity (stride 0) or a residue permutation.  The kernel additionally needs
    N/s divisible by 128 for its strided tensor maps; strides that miss it are
    skipped."""
    c = costs(mask, N, BQ, A)
    if not c:
        return "identity", 0
    ok = {k: v for k, v in c.items()
          if k == "identity" or (k.startswith("residue-perm-")
                                 and (N // stride_of(k)) % 128 == 0)}
    name = min(ok, key=_rank(ok))
    return name, stride_of(name)


def costs_device(mask, N, BQ, A, device="cuda"):
    """{candidate: elements computed} for identity and every residue-perm-s with
    N/s a multiple of BQ and A, measured by building each candidate's block index
    on the GPU (``blockindex.build_device``, the tiles it lists times BQ*A).  Works
    for masks that are not diagonally invariant as well, where the closed forms of
    ``costs`` do not apply; on invariant masks it equals ``costs`` exactly."""
    import torch
    from . import blockindex, permute
    out, stats = {}, []
    for name in CANDIDATES:
        if is_class_b(name):
            continue
        s = stride_of(name)
        if s and (N % s or (N // s) % BQ or (N // s) % A):
            continue
        perm = permute.residue_perm_device(N, s, device) if s else None
        dbi = blockindex.build_device(mask, N, BQ, A, perm_q=perm, perm_kv=perm, device=device)
        stats.append((name, dbi.stats))
    torch.cuda.synchronize(device)
    for name, st in stats:
        out[name] = int(st[0].item())
    return out


class ClassAPlan:
    """What ``prepare`` chose and built for one mask: the candidate, the residue
    stride (0 = identity basis), the device block index of the mask in that basis
    and the attention work list.  ``run(q, k, v)`` takes and returns tensors in
    original row order."""

    def __init__(self, mask, N, BQ, A, name, stride, index, plan):
        self.mask, self.N, self.BQ, self.A = mask, N, BQ, A
        self.name, self.stride, self.index, self.plan = name, stride, index, plan

    def run(self, q, k, v, scale=None, return_lse=True):
        from . import attention
        kind, p0, p1, p2 = self.mask.spec
        return attention.block_sparse_attention(
            q, k, v, None, None, None, kind, p0, p1, p2, self.BQ, self.A, scale=scale,
            residue_stride=self.stride, plan=self.plan, return_lse=return_lse)


def select_split(mask, N, BQ, A):
    """Single basis vs band + lattice split for a LocalStrided(w, s) mask.

    Returns {"single": (name, stride, elements), "parts": [(mask, name, stride,
    elements), ...], "split": bool} -- ``split`` True when the parts' elements
    undercut the single basis by more than ``SPLIT_MARGIN`` -- or None for a mask
    that is not a band + lattice union."""
    from . import masks as M
    spec = getattr(mask, "spec", None)
    if spec is None or int(spec[0]) != M.LOCAL_STRIDED:
        return None
    w, s = int(spec[1]), int(spec[2])
    name, stride = select_class_a(mask, N, BQ, A)
    single = (name, stride, costs(mask, N, BQ, A)[name])
    parts = []
    for part in (M.SlidingWindow(w), M.FarStrided(w, s)):
        pc = costs(part, N, BQ, A)
        pname, pstride = select_class_a(part, N, BQ, A)
        parts.append((part, pname, pstride, pc[pname] if pc else None))
    total = sum(p[3] for p in parts) if all(p[3] is not None for p in parts) else None
    split = total is not None and total < (1.0 - SPLIT_MARGIN) * single[2]
    return {"single": single, "parts": parts, "split": split}


class SplitChoice:
    """What ``prepare(..., allow_split=True)`` built for a band + lattice union:
    the parts with their bases and the ``split.SplitPlan``.  ``run(q, k, v)`` takes
    and returns tensors in original row order."""

    def __init__(self, mask, N, BQ, A, choice, plan):
        self.mask, self.N, self.BQ, self.A = mask, N, BQ, A
        self.name = "split: " + " + ".join(f"{p[0].name} [{p[1]}]" for p in choice["parts"])
        self.choice, self.plan = choice, plan

    def run(self, q, k, v, scale=None, return_lse=True):
        o, lse = self.plan.run(q, k, v, scale=scale)
        return (o, lse) if return_lse else o


def prepare(mask, N, BQ, A, device="cuda", allow_split=False):
    """Choose the executable basis with ``select_class_a`` and build, on the GPU,
    the block index of the mask in that basis and the forward's work list.  With
    ``allow_split``, a band + lattice union that ``select_split`` finds cheaper as
    a split is built as one instead (the window part on the 64-row kernel, which
    suits its partial tiles)."""
    from . import attention, blockindex, permute
    if allow_split:
        choice = select_split(mask, N, BQ, A)
        if choice is not None and choice["split"]:
            from . import split
            parts = [split.SplitPart(pm, BQ, A, pstride, 64 if i == 0 else 0)
                     for i, (pm, _, pstride, _) in enumerate(choice["parts"])]
            return SplitChoice(mask, N, BQ, A, choice, split.SplitPlan(parts, N, device))
    name, stride = select_class_a(mask, N, BQ, A)
    perm = permute.residue_perm_device(N, stride, device) if stride else None
    index = blockindex.build_device(mask, N, BQ, A, perm_q=perm, perm_kv=perm, device=device)
    plan = attention.make_plan(index.kv_idx, index.kv_num, index.kv_partial, N, BQ, A,
                               residue_stride=stride)
    return ClassAPlan(mask, N, BQ, A, name, stride, index, plan)
