"""Attention over a union of differing mask families by disjoint split + LSE merge.

A mask M that is the disjoint union of parts P1 + P2 + ... is computed as one
block-sparse attention per part -- each part in its own best basis (identity or a
class A residue permutation) -- and the partial (O_i, LSE_i) are combined with the
log-sum-exp merge.  This is the execution side of the reference's composition
study (src/polyattn/experiments/compose.py:7-17: split, per-part class-A basis,
merge), which the reference only counts.  Disjointness is required: an element in
two parts would be counted twice in the softmax denominator.

A part in a residue-permuted basis runs on Q/K/V in their original row order: the
kernel reads the permuted order through strided tensor maps (``residue_stride``),
evaluates the predicate in original coordinates and writes O/LSE back in original
order, so no part copies Q/K/V.  Every part after the first merges its result into
the O/LSE already written (the attention epilogue's ``merge``), so the split costs no
separate merge pass over O.
"""
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import attention, blockindex, masks, permute, shard


@dataclass
class SplitPart:
    mask: object            # polyhedral_b200.masks object (has .spec)
    BQ: int
    A: int
    stride: int = 0         # residue-permutation stride; 0 = identity basis
    kv_rows: int = 0        # attention kernel's KV super-tile (0/128, or 64: first part only)
    row_threads: int = 0    # softmax threads per query row (2: first part only)


class SplitPlan:
    """Mask-only preprocessing of a split (block indices, permutations, work
    lists), built once and reused by ``run`` for every (q, k, v)."""

    def __init__(self, parts, N, device="cuda"):
        self.N = N
        self.parts = list(parts)
        self.device = torch.device(device)
        if any(part.kv_rows == 64 or part.row_threads == 2 for part in self.parts[1:]):
            raise ValueError("only the first part can use kv_rows=64 or row_threads=2: later "
                             "parts merge in their epilogue, which those kernels do not")
        self.perms, self.indices, self.plans = [], [], []
        for part in self.parts:
            perm = None
            if part.stride:
                perm = permute.residue_perm_device(N, part.stride, self.device)
            dbi = blockindex.build_device(part.mask, N, part.BQ, part.A, perm_q=perm,
                                          perm_kv=perm, device=self.device)
            plan = attention.make_plan(dbi.kv_idx, dbi.kv_num, dbi.kv_partial, N, part.BQ,
                                       part.A, residue_stride=part.stride)
            self.perms.append(perm)
            self.indices.append(dbi)
            self.plans.append(plan)

    def run(self, q, k, v, scale=None, out=None, lse_out=None):
        """(o, lse) of the union mask, rows in original order.  The first part
        writes O / LSE; each later part merges its result into them in its own
        epilogue (``merge=True``), so no separate merge pass runs."""
        BH, N, D = q.shape
        o = out if out is not None else torch.empty_like(q)
        lse = lse_out if lse_out is not None else torch.empty((BH, N), dtype=torch.float32,
                                                              device=q.device)
        for i, part in enumerate(self.parts):
            kind, p0, p1, p2 = part.mask.spec
            attention.block_sparse_attention(
                q, k, v, None, None, None, kind, p0, p1, p2, part.BQ, part.A,
                scale=scale, residue_stride=part.stride, plan=self.plans[i], return_lse=True,
                out=o, lse_out=lse, merge=i > 0, kv_rows=part.kv_rows,
                row_threads=part.row_threads)
        return o, lse

    def run_part(self, i, q, k, v, o, lse, scale=None):
        """Part i alone, as ``run`` launches it (merging into o / lse when i > 0)."""
        part = self.parts[i]
        kind, p0, p1, p2 = part.mask.spec
        return attention.block_sparse_attention(
            q, k, v, None, None, None, kind, p0, p1, p2, part.BQ, part.A, scale=scale,
            residue_stride=part.stride, plan=self.plans[i], return_lse=True, out=o,
            lse_out=lse, merge=i > 0, kv_rows=part.kv_rows, row_threads=part.row_threads)

    def run_shard(self, q, k, v, rank, world, scale=None, out=None, lse_out=None):
        """This rank's share of ``run``: the contiguous (batch, head) range
        ``shard.shard_bh(BH, rank, world)`` of the full-size q, k, v (views, no copy),
        with the same plans; returns that range's (o, lse) (rows of out / lse_out
        when given, full-size).  No collective: ``shard.gather`` assembles the whole
        result when a caller needs it on one rank."""
        sh = shard.shard_bh(q.shape[0], rank, world)
        return sh.run(lambda q_, k_, v_, out, lse_out: self.run(q_, k_, v_, scale=scale, out=out,
                                                                  lse_out=lse_out),
                      q, k, v, out=out, lse_out=lse_out)

    def live_count(self):
        return sum(int(p.mask.live_count(self.N)) for p in self.parts)


def local_strided_split(w, s, N, BQ=128, A=32, stride=None, device="cuda", A_window=None,
                        window_kv_rows=0):
    """LocalStrided(w, s) = SlidingWindow(w) [identity, tiles BQ x A_window (default
    A), KV super-tile ``window_kv_rows``] + FarStrided(w, s) [residue permutation by
    `stride`, default s, tiles BQ x A]."""
    parts = [SplitPart(masks.SlidingWindow(w), BQ, A_window or A, 0, window_kv_rows),
             SplitPart(masks.FarStrided(w, s), BQ, A, stride or s)]
    return SplitPlan(parts, N, device)


def check_disjoint_cover(union_mask, parts, N):
    """True when the parts are pairwise disjoint and their union is the mask
    (compose.py:69-70 asserts exact reconstruction).  Host check, small N."""
    M = union_mask.dense(N)
    acc = np.zeros_like(M, dtype=np.int32)
    for p in parts:
        acc += p.mask.dense(N).astype(np.int32)
    return bool((acc <= 1).all() and np.array_equal(acc.astype(bool), M))
