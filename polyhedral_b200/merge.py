"""Log-sum-exp merge of attentions over disjoint masks (``pa_lse_merge``,
csrc/merge.cu).  The reference argues for this combine and costs it
(src/polyattn/experiments/compose.py:7-17, :107-118) but never runs it."""
import ctypes

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.PA_BF16, torch.float16: _lib.PA_F16}


def lse_merge(o1, lse1, o2, lse2, row_map2=None, out=None, lse_out=None):
    """Attention over P1 + P2 (disjoint) from the attentions over P1 and P2.

    o1, o2: [BH, N, D] bf16/fp16; lse1, lse2: [BH, N] fp32 (natural log, -inf for
    a row with no live key in that part).  ``row_map2[r]`` is the row of o2/lse2
    holding row r (for a part computed on permuted rows pass ``invert(perm)``).
    ``out`` may be ``o1`` and ``lse_out`` may be ``lse1`` (in place).
    Returns (o, lse)."""
    BH, N, D = o1.shape
    if o2.shape != o1.shape or lse1.shape != (BH, N) or lse2.shape != (BH, N):
        raise ValueError("shape mismatch between the two parts")
    if o1.dtype not in _DTYPES or o2.dtype != o1.dtype:
        raise TypeError("o1/o2 must share dtype bf16 or fp16")
    if lse1.dtype != torch.float32 or lse2.dtype != torch.float32:
        raise TypeError("lse must be float32")
    for t in (o1, o2, lse1, lse2):
        if not t.is_cuda:
            raise RuntimeError("lse_merge runs on the GPU only")
        if t.stride(-1) != 1:
            raise ValueError("last dimension must be contiguous")
    o = out if out is not None else torch.empty_like(o1)
    lse = lse_out if lse_out is not None else torch.empty_like(lse1)
    rm = None
    if row_map2 is not None:
        rm = torch.as_tensor(row_map2).to(device=o1.device, dtype=torch.int32).contiguous()
    a = _lib.PaMergeArgs()
    a.o1, a.lse1, a.o2, a.lse2 = o1.data_ptr(), lse1.data_ptr(), o2.data_ptr(), lse2.data_ptr()
    a.o, a.lse = o.data_ptr(), lse.data_ptr()
    a.BH, a.N, a.D, a.dtype = BH, N, D, _DTYPES[o1.dtype]
    a.o1_bh_stride, a.o1_row_stride = o1.stride(0), o1.stride(1)
    a.o2_bh_stride, a.o2_row_stride = o2.stride(0), o2.stride(1)
    a.o_bh_stride, a.o_row_stride = o.stride(0), o.stride(1)
    a.lse1_bh_stride, a.lse2_bh_stride, a.lse_bh_stride = (lse1.stride(0), lse2.stride(0),
                                                           lse.stride(0))
    a.row_map2 = rm.data_ptr() if rm is not None else None
    _lib.call("pa_lse_merge", ctypes.byref(a), _lib.stream_handle(o1.device), device=o1.device)
    return o, lse
