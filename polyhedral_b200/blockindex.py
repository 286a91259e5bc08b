"""Block-sparse tile index at any (BQ, A), built on the GPU.

Same interface and bit-identical result as the reference's ``gpu/blockindex.py``
(:16-58): for each query block, the ascending ids of the KV tiles holding any live
element (``kv_idx``, zero-padded to the longest row), how many (``kv_num``), and
whether each listed tile is partial (``kv_partial``); ``elements`` = tiles * BQ * A
and ``live``.

The classification runs in ``pa_block_index`` (csrc/blockindex.cu) straight from
the mask predicate, in the coordinates of permuted rows/columns when ``perm_q`` /
``perm_kv`` are given, without materialising the N x N mask.  Masks without a
predicate spec (e.g. an explicit boolean matrix) are classified from their dense
rows by ``pa_block_index_dense``.
"""
import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib


@dataclass
class BlockIndex:
    BQ: int
    A: int
    N: int
    kv_idx: np.ndarray       # [n_q_blocks, max_kv] int32
    kv_num: np.ndarray       # [n_q_blocks] int32
    kv_partial: np.ndarray   # [n_q_blocks, max_kv] int8
    elements: int
    live: int

    @property
    def waste(self):
        return self.elements / self.live


@dataclass
class DeviceBlockIndex:
    """Device-resident block index: rows of ``kv_idx`` / ``kv_partial`` are
    ``stride`` = N/A wide (zero past ``kv_num``), and ``stats`` holds
    [elements, live, max_kv, tiles] as int64 -- nothing is copied to the host."""
    BQ: int
    A: int
    N: int
    kv_idx: "torch.Tensor"
    kv_num: "torch.Tensor"
    kv_partial: "torch.Tensor"
    stats: "torch.Tensor"

    @property
    def stride(self):
        return self.kv_idx.shape[1]

    def to_host(self):
        """The reference-layout BlockIndex (one device->host copy)."""
        st = self.stats.cpu().tolist()
        elements, live, max_kv = int(st[0]), int(st[1]), int(st[2])
        kv_idx = self.kv_idx[:, :max_kv].cpu().numpy().astype(np.int32, copy=False)
        kv_partial = self.kv_partial[:, :max_kv].cpu().numpy().astype(np.int8, copy=False)
        return BlockIndex(self.BQ, self.A, self.N, np.ascontiguousarray(kv_idx),
                          self.kv_num.cpu().numpy(), np.ascontiguousarray(kv_partial),
                          elements, live)


def _spec_of(mask):
    spec = getattr(mask, "spec", None)
    if spec is not None:
        return tuple(int(x) for x in spec)
    if isinstance(mask, (tuple, list)) and len(mask) == 4:
        return tuple(int(x) for x in mask)
    return None


def _perm_tensor(perm, N, device):
    import torch
    if perm is None:
        return None
    t = torch.as_tensor(np.asarray(perm) if not isinstance(perm, torch.Tensor) else perm)
    if t.numel() != N:
        raise ValueError(f"permutation has {t.numel()} entries, expected N={N}")
    return t.to(device=device, dtype=torch.int32).contiguous()


def build_device(mask, N, BQ, A, perm_q=None, perm_kv=None, device="cuda", stream=None):
    """Classify on the GPU; returns a DeviceBlockIndex without synchronising.

    ``mask``: a mask object with a ``spec`` (polyhedral_b200.masks), a
    (kind, p0, p1, p2) tuple, or any object with ``row_cols(q, N)`` (classified
    from its dense rows).  ``perm_q`` / ``perm_kv`` (permuted position -> original
    index) give the block index of M[perm_q][:, perm_kv]; ``perm_kv`` defaults to
    ``perm_q``.
    """
    import torch
    if N % BQ or N % A:
        raise AssertionError("N must be a multiple of BQ and A")
    device = torch.device(device)
    if perm_kv is None:
        perm_kv = perm_q
    nq, nk = N // BQ, N // A
    kv_idx = torch.empty((nq, nk), dtype=torch.int32, device=device)
    kv_num = torch.empty((nq,), dtype=torch.int32, device=device)
    kv_partial = torch.empty((nq, nk), dtype=torch.int8, device=device)
    stats = torch.empty((4,), dtype=torch.int64, device=device)
    s = stream if stream is not None else _lib.stream_handle(device)
    spec = _spec_of(mask)
    if spec is not None:
        pq = _perm_tensor(perm_q, N, device)
        pk = _perm_tensor(perm_kv, N, device)
        pred = _lib.PaPred(*spec)
        _lib.call("pa_block_index", ctypes.byref(pred), N, BQ, A,
                  pq.data_ptr() if pq is not None else None,
                  pk.data_ptr() if pk is not None else None,
                  kv_idx.data_ptr(), nk, kv_num.data_ptr(), kv_partial.data_ptr(),
                  stats.data_ptr(), s, device=device)
        keep = (pq, pk)
    else:
        M = np.stack([np.asarray(mask.row_cols(q, N), dtype=bool) for q in range(N)])
        if perm_q is not None:
            M = M[np.asarray(perm_q)][:, np.asarray(perm_kv)]
        Md = torch.from_numpy(M.astype(np.uint8)).to(device)
        _lib.call("pa_block_index_dense", Md.data_ptr(), N, BQ, A, kv_idx.data_ptr(), nk,
                  kv_num.data_ptr(), kv_partial.data_ptr(), stats.data_ptr(), s, device=device)
        keep = (Md,)
    dbi = DeviceBlockIndex(BQ, A, N, kv_idx, kv_num, kv_partial, stats)
    dbi._keepalive = keep   # inputs must outlive the asynchronous kernel
    return dbi


def build(mask, N, BQ, A, perm_q=None, perm_kv=None, device="cuda"):
    """The reference's ``build(mask, N, BQ, A)`` (gpu/blockindex.py:32-51), computed
    on the GPU; returns host arrays in the reference layout.  ``perm_q`` /
    ``perm_kv`` are additive extensions (see ``build_device``)."""
    assert N % BQ == 0 and N % A == 0
    return build_device(mask, N, BQ, A, perm_q, perm_kv, device).to_host()


def to_cuda(bi, device="cuda"):
    """(kv_idx, kv_num, kv_partial) on the device (gpu/blockindex.py:54-58)."""
    import torch
    if isinstance(bi, DeviceBlockIndex):
        return bi.kv_idx, bi.kv_num, bi.kv_partial
    return (torch.from_numpy(bi.kv_idx).to(device),
            torch.from_numpy(bi.kv_num).to(device),
            torch.from_numpy(bi.kv_partial).to(device))
