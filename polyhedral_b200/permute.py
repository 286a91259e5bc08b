"""Class A re-indexing on the GPU (the reference's ``gpu/permute.py``, :12-38).

A residue permutation relabels Q/K/V rows once so a lattice mask becomes block
diagonal.  ``apply_perm`` / ``scatter_rows`` copy rows bit for bit with the
``pa_permute_rows`` kernel (csrc/permute.cu); up to four tensors share a launch.
"""
import ctypes

import numpy as np

from . import _lib


def residue_perm(N, s):
    """int32[N]: perm[p] = original index at permuted position p, positions
    ordered by (i mod s, i div s) (gpu/permute.py:12-16).  A host array, as in the
    reference; ``residue_perm_device`` builds it on the GPU."""
    return np.concatenate([np.arange(r, N, s) for r in range(s)]).astype(np.int32)


def identity_perm(N):
    return np.arange(N, dtype=np.int32)


def residue_perm_device(N, s, device="cuda"):
    import torch
    out = torch.empty(N, dtype=torch.int32, device=device)
    _lib.call("pa_residue_perm", N, s, out.data_ptr(), _lib.stream_handle(out.device),
              device=out.device)
    return out


def _as_dev_perm(perm, N, device):
    import torch
    if not isinstance(perm, torch.Tensor):
        perm = torch.from_numpy(np.asarray(perm, dtype=np.int32))
    if perm.numel() != N:
        raise ValueError(f"permutation has {perm.numel()} entries, expected {N}")
    return perm.to(device=device, dtype=torch.int32).contiguous()


def _check_rows(x):
    import torch
    if not x.is_cuda:
        raise RuntimeError("row permutation runs on the GPU only; got a CPU tensor")
    if x.dim() != 3:
        raise ValueError(f"expected [BH, N, D], got shape {tuple(x.shape)}")
    if x.stride(2) != 1:
        raise ValueError("last dimension must be contiguous")
    return x


def _permute(tensors, perm, scatter, outs=None):
    import torch
    tensors = [_check_rows(t) for t in tensors]
    BH, N, D = tensors[0].shape
    for t in tensors:
        if tuple(t.shape) != (BH, N, D) or t.dtype != tensors[0].dtype:
            raise ValueError("all tensors must share shape and dtype")
    p = _as_dev_perm(perm, N, tensors[0].device)
    outs = outs or [torch.empty((BH, N, D), dtype=t.dtype, device=t.device) for t in tensors]
    es = tensors[0].element_size()
    s = _lib.stream_handle(tensors[0].device)
    for i in range(0, len(tensors), 4):
        group = list(zip(tensors[i:i + 4], outs[i:i + 4]))
        arr = (_lib.PaRows * len(group))()
        for j, (src, dst) in enumerate(group):
            arr[j] = _lib.PaRows(src.data_ptr(), dst.data_ptr(),
                                 src.stride(0) * es, src.stride(1) * es,
                                 dst.stride(0) * es, dst.stride(1) * es)
        _lib.call("pa_permute_rows", arr, len(group), BH, N, D * es, p.data_ptr(),
                  1 if scatter else 0, s, device=tensors[0].device)
    return outs


def apply_perm(x, perm):
    """x: [BH, N, D] -> rows reordered so position p holds original row perm[p]
    (gpu/permute.py:22-24).  Returns a new contiguous tensor."""
    return _permute([x], perm, scatter=False)[0]


def apply_perm_many(tensors, perm):
    """``apply_perm`` on several same-shaped tensors in one launch per four."""
    return _permute(list(tensors), perm, scatter=False)


def scatter_rows(x, perm):
    """Inverse of ``apply_perm``: out[:, perm[p]] = x[:, p] -- equal to
    ``x.index_select(1, invert(perm))`` (gpu/test_correctness.py:77)."""
    return _permute([x], perm, scatter=True)[0]


def invert(perm):
    """inv[perm[i]] = i (gpu/permute.py:27-31), on the GPU; same dtype as perm."""
    import torch
    if not isinstance(perm, torch.Tensor) or not perm.is_cuda:
        raise RuntimeError("invert runs on the GPU: pass a CUDA tensor")
    N = perm.numel()
    p32 = perm.to(torch.int32).contiguous()
    inv = torch.empty_like(p32)
    _lib.call("pa_invert_perm", p32.data_ptr(), N, inv.data_ptr(), _lib.stream_handle(perm.device),
              device=perm.device)
    return inv.to(perm.dtype)


def permutation_cost_ms(q, k, v, perm, reps=50):
    """Time of permuting Q, K and V (one launch), reported separately from the
    attention (gpu/permute.py:34-38)."""
    from .timing import time_ms
    return time_ms(lambda: apply_perm_many((q, k, v), perm), reps=reps)[0]
