"""CPU restatement of the reference's block-sparse attention path.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke`` and the
CPU-baseline leg of ``bench.py``, as the checker.  The product never calls it.

Each function cites the reference code it restates (paths relative to the
reference checkout, GueroudjiAmal/polyhedral).  Integer work (mask, block index,
permutations) is numpy; floating-point attention is torch on the CPU in fp32,
the same arithmetic the reference oracle uses.
"""
import numpy as np

__all__ = [
    "CAUSAL", "WINDOW", "DILATED", "LOCAL_STRIDED", "TWOBAND", "SINKS", "FAR_STRIDED",
    "dense_mask", "block_index", "residue_perm", "invert", "apply_perm",
    "attention", "attention_heads", "online_softmax_blockwise", "lse_merge",
    "permuted_mask",
]

# Mask kinds, numbered as gpu/masks_gpu.py:9 numbers them.  FAR_STRIDED is the one
# addition: the lattice half of configuration 5's disjoint split (d >= p0 and
# d % p1 == 0), which no reference kind can express on its own.
CAUSAL, WINDOW, DILATED, LOCAL_STRIDED, TWOBAND, SINKS, FAR_STRIDED = range(7)


def _pred(kind, p0, p1, p2, qi, kj):
    """Element predicate on original coordinates, as gpu/masks_gpu.py:37-53."""
    d = qi - kj
    causal = d >= 0
    if kind == CAUSAL:
        return causal
    if kind == WINDOW:
        return causal & (d < p0)
    if kind == DILATED:
        return causal & (d % p0 == 0)
    if kind == LOCAL_STRIDED:
        return causal & ((d < p0) | (d % p1 == 0))
    if kind == TWOBAND:
        return causal & ((d < p0) | ((d >= p1) & (d < p1 + p2)))
    if kind == SINKS:
        return causal & ((d < p0) | (kj < p1))
    if kind == FAR_STRIDED:
        return causal & (d >= p0) & (d % p1 == 0)
    raise ValueError(f"unknown mask kind {kind}")


def dense_mask(kind, p0, p1, p2, N, rows=None):
    """bool [len(rows), N]: mask[i, j] for original coordinates (masks_gpu.dense_bool,
    gpu/masks_gpu.py:56-61).  ``rows`` restricts to a subset of query rows."""
    qi = (np.arange(N) if rows is None else np.asarray(rows))[:, None].astype(np.int64)
    kj = np.arange(N, dtype=np.int64)[None, :]
    return _pred(kind, p0, p1, p2, qi, kj)


def permuted_mask(M, perm_q, perm_kv=None):
    """The mask seen by a kernel run on permuted rows/columns: ``M[p][:, p]``
    (gpu/test_correctness.py:71)."""
    perm_kv = perm_q if perm_kv is None else perm_kv
    return M[np.asarray(perm_q)][:, np.asarray(perm_kv)]


def block_index(M, BQ, A):
    """Tile classification of an explicit N x N mask, as gpu/blockindex.py:32-51.

    Returns (kv_idx [nq, max_kv] int32, kv_num [nq] int32, kv_partial [nq, max_kv]
    int8, elements, live).  A tile is listed when any element is live and flagged
    partial unless every element is live; listed tiles are in ascending order and
    each row is zero-padded to the longest row's count.
    """
    N = M.shape[0]
    if N % BQ or N % A or M.shape[1] != N:
        raise ValueError("N must be a multiple of BQ and A")
    nq, nk = N // BQ, N // A
    t = M.reshape(nq, BQ, nk, A)
    live_tile = t.any(axis=(1, 3))
    full_tile = t.all(axis=(1, 3))
    kv_num = live_tile.sum(axis=1).astype(np.int32)
    max_kv = int(kv_num.max()) if nq else 0
    kv_idx = np.zeros((nq, max_kv), np.int32)
    kv_partial = np.zeros((nq, max_kv), np.int8)
    for i in range(nq):
        cols = np.nonzero(live_tile[i])[0]
        kv_idx[i, :len(cols)] = cols
        kv_partial[i, :len(cols)] = np.where(full_tile[i, cols], 0, 1)
    elements = int(live_tile.sum()) * BQ * A
    return kv_idx, kv_num, kv_partial, elements, int(M.sum())


def residue_perm(N, s):
    """Positions ordered by (i mod s, i div s) -- gpu/permute.py:12-16.

    Written as the concatenation of the residue classes, which is the order a
    stable sort on that key produces.
    """
    return np.concatenate([np.arange(r, N, s) for r in range(s)]).astype(np.int32)


def invert(perm):
    """inv[perm[i]] = i (gpu/permute.py:27-31)."""
    perm = np.asarray(perm)
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.size, dtype=perm.dtype)
    return inv


def apply_perm(x, perm):
    """Row gather ``out[:, p] = x[:, perm[p]]`` on [BH, N, D] (gpu/permute.py:22-24)."""
    return np.ascontiguousarray(np.asarray(x)[:, np.asarray(perm)])


def attention(q, k, v, mask, scale=None, with_lse=True):
    """Dense masked attention in fp32 on the CPU (gpu/reference.py:5-13).

    q, k, v: torch tensors [BH, N, D] (any float dtype; computed in fp32).
    mask: torch bool [N, N] (True = live).  Returns (o fp32, lse fp32): rows with
    no live key give o = 0 (the reference's nan_to_num) and lse = -inf.
    LSE = logsumexp over the live scaled scores (natural log), from the same
    scores the reference softmaxes.
    """
    import torch
    scale = scale or q.shape[-1] ** -0.5
    s = (q.float() @ k.float().transpose(-1, -2)) * scale
    s = s.masked_fill(~mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    o = p @ v.float()
    lse = torch.logsumexp(s, dim=-1) if with_lse else None
    return o, lse


def attention_heads(q, k, v, mask, scale=None, heads=None, row_chunk=None):
    """``attention`` evaluated head by head (and optionally in row chunks) so the
    [N, N] score matrix of one head is the largest temporary.  ``heads`` selects a
    subset of the BH axis."""
    import torch
    heads = range(q.shape[0]) if heads is None else heads
    N = q.shape[1]
    row_chunk = row_chunk or N
    outs, lses = [], []
    for h in heads:
        o_parts, l_parts = [], []
        for r0 in range(0, N, row_chunk):
            r1 = min(N, r0 + row_chunk)
            o, lse = attention(q[h:h + 1, r0:r1], k[h:h + 1], v[h:h + 1],
                               mask[r0:r1], scale)
            o_parts.append(o)
            l_parts.append(lse)
        outs.append(torch.cat(o_parts, 1))
        lses.append(torch.cat(l_parts, 1))
    return torch.cat(outs, 0), torch.cat(lses, 0)


def online_softmax_blockwise(M, q, k, v, BQ, A, m_init=-1e30, scale=None):
    """Tile-by-tile online softmax in float64, the arithmetic of the reference
    kernel's inner loop (gpu/triton_attn.py:83-182) as its CPU simulation states
    it (tests/test_kernel_math.py:27-48): finite running-max sentinel, masked
    scores at -inf, and an ``l > 0`` guard so a row live nowhere returns zeros.
    q, k, v: float64 [N, D]; M: bool [N, N]."""
    N, D = q.shape
    scale = D ** -0.5 if scale is None else scale
    live_tile = M.reshape(N // BQ, BQ, N // A, A).any(axis=(1, 3))
    out = np.zeros((N, D))
    for i in range(N // BQ):
        r = slice(i * BQ, (i + 1) * BQ)
        m = np.full(BQ, float(m_init))
        l = np.zeros(BQ)
        acc = np.zeros((BQ, D))
        for j in np.nonzero(live_tile[i])[0]:
            c = slice(j * A, (j + 1) * A)
            s = np.where(M[r, c], (q[r] @ k[c].T) * scale, -np.inf)
            m_new = np.maximum(m, s.max(axis=1))
            with np.errstate(invalid="ignore"):
                alpha = np.exp(m - m_new)
                p = np.exp(s - m_new[:, None])
            l = l * alpha + p.sum(axis=1)
            acc = acc * alpha[:, None] + p @ v[c]
            m = m_new
        out[r] = acc / np.where(l > 0, l, 1.0)[:, None]
    return out


def lse_merge(o1, lse1, o2, lse2):
    """Combine two attentions over DISJOINT masks into the attention over their
    union: the log-sum-exp merge argued in src/polyattn/experiments/compose.py:7-17
    (and costed at :107-118; the reference never executes it).

    o_i: [..., N, D] float, lse_i: [..., N] float (natural log, -inf for a row
    with no live key in that part).  Returns (o, lse) in float64 numpy.
    """
    o1, o2 = np.asarray(o1, np.float64), np.asarray(o2, np.float64)
    l1, l2 = np.asarray(lse1, np.float64), np.asarray(lse2, np.float64)
    m = np.maximum(l1, l2)
    dead = np.isneginf(m)
    m_safe = np.where(dead, 0.0, m)
    w1 = np.exp(l1 - m_safe)
    w2 = np.exp(l2 - m_safe)
    den = w1 + w2
    den_safe = np.where(den > 0, den, 1.0)
    o = (w1[..., None] * o1 + w2[..., None] * o2) / den_safe[..., None]
    lse = np.where(dead, -np.inf, m_safe + np.log(den_safe))
    return o, lse
