"""Block-sparse attention forward on sm_100a -- the drop-in for the reference's
``block_sparse_attention`` (gpu/triton_attn.py:185-241).

Same arguments, defaults and checks as the reference: q, k, v are [BH, N, D]
with a contiguous last dimension; ``kv_idx`` / ``kv_num`` / ``kv_partial`` come
from ``blockindex``; ``perm_q`` / ``perm_kv`` (permuted position -> original index)
say where the physically permuted rows came from, so the predicate is evaluated in
original coordinates; ``perm_kv`` defaults to ``perm_q``.  The kernel is the
tcgen05/TMEM one in csrc/attn.cu; there is no other implementation.

Extensions (keyword-only): ``return_lse`` returns (o, lse) with lse [BH, N] fp32
(natural log, -inf for a row with no live key); ``o_row_map`` writes row r of the
result at ``o_row_map[r]`` (pass ``perm_q`` to get O back in original order, fusing
the inverse permutation); ``plan`` reuses a work list built once by ``make_plan`` (``set_plan_cache(True)``
keeps the lists of calls without one, keyed on their index tensors and stream);
``out`` / ``lse_out`` supply output buffers; ``check`` synchronises and raises if
the kernel reported a device-side failure; ``residue_stride=s`` takes q, k, v (and
returns o, lse) in ORIGINAL row order and runs on their residue permutation by s
without copying them (the kernel's tensor maps read row p of the permuted order
directly; the block index is still that of the permuted mask); ``merge=True`` (with
``out`` and ``lse_out``) treats them as holding the result of an attention over a
disjoint mask on the same rows and merges this one into them in the epilogue
(log-sum-exp merge, as ``merge.lse_merge``), so a split runs without a merge pass;
``kv_rows=64`` selects the 64-row super-tile kernel (S double-buffered in TMEM, and
each 128-row half computes only the tiles live for it: faster on bands narrower than
an item's 256 rows, slower on mostly full tiles; not with ``merge``).  ``sched_heads=G`` runs the work items in groups of G heads, one group
after another (default: all heads in one group); groups whose K/V fit in L2 cut DRAM
re-reads when all heads' K/V do not.  ``row_threads=2`` splits every query row's
softmax over two threads (64 columns each; not with ``merge``, ``kv_rows=64`` or
gathered K/V), ``row_threads=1`` keeps one; the default (0) lets the library choose:
two for tiles at most 32 columns wide or D = 64, where they measured faster.
``num_warps`` / ``num_stages`` are accepted and ignored.

The reference's class-B traffic emulation (gpu/triton_attn.py:99-128) keeps its
meaning: ``gather_kv=True`` takes k and v in ORIGINAL order and reads row j of the
kernel order from row ``perm_kv[j]`` per tile (four-row TMA gathers), so the result
equals the one on physically permuted k / v; ``gather_mult=R`` makes every K tile
read R - 1 more sets of A rows that the result does not use, rows ``row(j) + r*A``
(``gather_scatter=False``) or ``perm_kv[j + r*A]`` (``gather_scatter=True``),
mod N.  Not with ``residue_stride``, ``merge`` or ``kv_rows=64``.
"""
import collections
import ctypes
import weakref

import torch

from . import _lib

CAUSAL, WINDOW, DILATED, LOCAL_STRIDED, TWOBAND, SINKS, FAR_STRIDED = range(7)

_DTYPES = {torch.bfloat16: _lib.PA_BF16, torch.float16: _lib.PA_F16}


class AttnPlan:
    """Device work list for one block index and K/V permutation (``pa_attn_plan``):
    the per-256-row union of listed tiles with each 128-row half's
    dead/full/partial status, the original-column progression of every listed
    tile, ordered longest first.  Reusable by every forward on the same index and
    ``perm_kv``."""

    def __init__(self, kv_idx, kv_num, kv_partial, N, BQ, A, perm_kv=None, device=None,
                 residue_stride=0):
        device = device or kv_num.device
        self.N, self.BQ, self.A = int(N), int(BQ), int(A)
        self.residue_stride = int(residue_stride)
        self.kv_idx, self.kv_num, self.kv_partial = kv_idx, kv_num, kv_partial
        self.kv_stride = int(kv_idx.shape[1]) if kv_idx.dim() == 2 else 0
        self.perm_kv = _perm(perm_kv, N, device)
        a = _args_skeleton(N, BQ, A, kv_idx, kv_num, kv_partial, self.kv_stride)
        a.perm_kv = _ptr(self.perm_kv)
        a.residue_stride = self.residue_stride
        nbytes = _lib.load().pa_attn_workspace_size(ctypes.byref(a))
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _lib.call("pa_attn_plan", ctypes.byref(a), self.workspace.data_ptr(), nbytes,
                  _lib.stream_handle(self.workspace.device), device=self.workspace.device)

    def status(self):
        """Device status of the most recent forward on this plan (synchronises): 0
        when it finished cleanly, else the code of the bounded wait that ran out."""
        st = _lib.c_i32(0)
        lib = _lib.load()
        with _lib.on_device(self.workspace.device):
            lib.pa_attn_status(self.workspace.data_ptr(), ctypes.byref(st),
                               _lib.stream_handle(self.workspace.device))
        return int(st.value)


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _args_skeleton(N, BQ, A, kv_idx, kv_num, kv_partial, kv_stride):
    a = _lib.PaAttnArgs()
    a.N, a.BQ, a.A = int(N), int(BQ), int(A)
    a.BH, a.D, a.dtype = 1, 128, _lib.PA_BF16
    a.kv_idx = _ptr(kv_idx) if kv_stride else None
    a.kv_num = _ptr(kv_num)
    a.kv_partial = _ptr(kv_partial) if kv_stride else None
    a.kv_stride = int(kv_stride)
    # placeholders: the plan reads only the block index and perm_kv
    a.q = a.k = a.v = a.o = _ptr(kv_num)
    return a


def make_plan(kv_idx, kv_num, kv_partial, N, BQ, A, perm_kv=None, residue_stride=0):
    """Build the forward's work list once for a block index (and the K/V
    permutation, explicit or residue, the forward will be given, if any)."""
    return AttnPlan(_index_tensor(kv_idx, torch.int32, kv_num.device),
                    _index_tensor(kv_num, torch.int32, kv_num.device),
                    _index_tensor(kv_partial, torch.int8, kv_num.device), N, BQ, A,
                    perm_kv=perm_kv, residue_stride=residue_stride)


# Work lists built by calls without ``plan``, kept when ``set_plan_cache(True)``: the
# reference's drivers call the forward over and over with one block index, and the
# list depends on that index only.
_PLAN_CACHE = collections.OrderedDict()
_PLAN_CACHE_SIZE = 8
_plan_cache_on = False


def set_plan_cache(on):
    """Reuse the work list of a call without ``plan`` for later calls with the same
    block-index tensors (the same objects, unmodified by torch since: their version
    counters), the same perm_kv, N, BQ, A, residue_stride, and the same stream, so that
    calls on different streams never share a workspace.  Off by default: a write to
    the index tensors that bypasses torch (another library's kernel, a DLPack alias)
    would leave a stale list; call ``clear_plan_cache`` after one.  At most
    ``_PLAN_CACHE_SIZE`` lists are kept.  ``dropin`` turns it on for the reference's
    driver scripts, which never rewrite their indices."""
    global _plan_cache_on
    _plan_cache_on = bool(on)
    if not on:
        clear_plan_cache()


def clear_plan_cache():
    _PLAN_CACHE.clear()


def _drop_cached(plan):
    """Forget a cached work list (after a forward on it reported a device failure,
    so that the next call builds a fresh one)."""
    for key in [k for k, (_, _, p) in _PLAN_CACHE.items() if p is plan]:
        del _PLAN_CACHE[key]


def _cached_plan(kv_idx, kv_num, kv_partial, N, BQ, A, perm_kv, pk, residue_stride, stream):
    objs = (kv_idx, kv_num, kv_partial, perm_kv)
    if not all(t is None or isinstance(t, torch.Tensor) for t in objs):
        return make_plan(kv_idx, kv_num, kv_partial, N, BQ, A, perm_kv=pk,
                         residue_stride=residue_stride)
    key = tuple(id(t) for t in objs) + (int(N), int(BQ), int(A), int(residue_stride), stream)
    vers = tuple(None if t is None else t._version for t in objs)
    hit = _PLAN_CACHE.get(key)
    if hit is not None:
        refs, v, plan = hit
        if v == vers and all((r() if r is not None else None) is t for r, t in zip(refs, objs)):
            _PLAN_CACHE.move_to_end(key)
            return plan
    plan = make_plan(kv_idx, kv_num, kv_partial, N, BQ, A, perm_kv=pk,
                     residue_stride=residue_stride)
    _PLAN_CACHE[key] = (tuple(None if t is None else weakref.ref(t) for t in objs), vers, plan)
    while len(_PLAN_CACHE) > _PLAN_CACHE_SIZE:
        _PLAN_CACHE.popitem(last=False)
    return plan


def _index_tensor(t, dtype, device):
    t = torch.as_tensor(t)
    if t.dtype != dtype:
        t = t.to(dtype)
    return t.to(device).contiguous()


def _perm(p, N, device):
    if p is None:
        return None
    t = torch.as_tensor(p)
    if t.numel() != N:
        raise ValueError(f"permutation has {t.numel()} entries, expected N={N}")
    return t.to(device=device, dtype=torch.int32).contiguous()


def block_sparse_attention(q, k, v, kv_idx, kv_num, kv_partial,
                           kind, p0, p1, p2, BQ, A, scale=None,
                           perm_q=None, perm_kv=None, gather_kv=False,
                           gather_mult=1, gather_scatter=True,
                           num_warps=4, num_stages=2, *, return_lse=False,
                           o_row_map=None, plan=None, out=None, lse_out=None,
                           check=False, residue_stride=0, merge=False, kv_rows=0,
                           sched_heads=0, row_threads=0):
    """q, k, v: [BH, N, D] (bf16 or fp16, D in {64, 128}), on one CUDA device.
    Returns o [BH, N, D] (same dtype), or (o, lse) with ``return_lse``."""
    gather_mult = max(int(gather_mult), 1)     # <= 1 reads no extra rows, as the reference
    if gather_mult > 16:
        raise ValueError(f"gather_mult={gather_mult}: at most 16")
    BH, N, D = q.shape
    assert N % BQ == 0 and N % A == 0, "cost model and kernel both assume this"
    assert k.shape == v.shape == q.shape
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("block_sparse_attention runs on the GPU only")
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"q/k/v must share dtype bf16 or fp16, got {q.dtype}/{k.dtype}/{v.dtype}")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.stride(2) != 1:
            raise ValueError(f"{name}: last dimension must be contiguous")
    dev = q.device
    residue_stride = int(residue_stride or 0)
    if residue_stride and (perm_q is not None or perm_kv is not None or o_row_map is not None):
        raise ValueError("residue_stride implies the permutation; pass no perm_q, perm_kv "
                         "or o_row_map with it")
    pq = _perm(perm_q, N, dev)
    pk = _perm(perm_kv, N, dev) if perm_kv is not None else pq
    rmap = _perm(o_row_map, N, dev)

    if plan is None and _plan_cache_on:
        plan = _cached_plan(kv_idx, kv_num, kv_partial, N, BQ, A,
                            perm_kv if perm_kv is not None else perm_q, pk, residue_stride,
                            _lib.stream_handle(dev).value)
    elif plan is None:
        plan = make_plan(kv_idx, kv_num, kv_partial, N, BQ, A, perm_kv=pk,
                         residue_stride=residue_stride)
    else:
        if (plan.N, plan.BQ, plan.A) != (N, BQ, A):
            raise ValueError("plan was built for a different (N, BQ, A)")
        if plan.residue_stride != residue_stride:
            raise ValueError("plan was built for a different residue_stride")
        if (plan.perm_kv is None) != (pk is None) or (
                pk is not None and plan.perm_kv.data_ptr() != pk.data_ptr()
                and not torch.equal(plan.perm_kv, pk)):
            raise ValueError("plan was built for a different perm_kv")

    if merge and (out is None or lse_out is None):
        raise ValueError("merge=True merges into out / lse_out: pass both")
    o = out if out is not None else torch.empty((BH, N, D), dtype=q.dtype, device=dev)
    lse = None
    if return_lse or merge:
        lse = lse_out if lse_out is not None else torch.empty((BH, N), dtype=torch.float32,
                                                              device=dev)

    a = _lib.PaAttnArgs()
    a.q, a.k, a.v, a.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    a.lse = _ptr(lse)
    a.BH, a.N, a.D, a.dtype = BH, N, D, _DTYPES[q.dtype]
    a.q_bh_stride, a.q_row_stride = q.stride(0), q.stride(1)
    a.k_bh_stride, a.k_row_stride = k.stride(0), k.stride(1)
    a.v_bh_stride, a.v_row_stride = v.stride(0), v.stride(1)
    a.o_bh_stride, a.o_row_stride = o.stride(0), o.stride(1)
    a.lse_bh_stride = lse.stride(0) if lse is not None else 0
    a.kv_idx = _ptr(plan.kv_idx) if plan.kv_stride else None
    a.kv_num = _ptr(plan.kv_num)
    a.kv_partial = _ptr(plan.kv_partial) if plan.kv_stride else None
    a.kv_stride = plan.kv_stride
    a.BQ, a.A = BQ, A
    a.perm_q, a.perm_kv, a.o_row_map = _ptr(pq), _ptr(pk), _ptr(rmap)
    a.pred = _lib.PaPred(int(kind), int(p0), int(p1), int(p2))
    a.scale = float(scale) if scale else 0.0
    a.residue_stride = residue_stride
    a.merge = 1 if merge else 0
    a.kv_rows = int(kv_rows or 0)
    a.gather_kv = 1 if gather_kv else 0
    a.gather_mult = gather_mult
    a.gather_scatter = 1 if gather_scatter else 0
    a.sched_heads = int(sched_heads or 0)
    a.row_threads = int(row_threads or 0)
    ws = plan.workspace
    _lib.call("pa_attn_fwd", ctypes.byref(a), ws.data_ptr(), ws.numel(),
              _lib.stream_handle(dev), device=dev)
    if check:
        st = plan.status()
        if st:
            _drop_cached(plan)
            raise _lib.PolyattnError("pa_attn_fwd", _lib.PA_ERR_DEVICE,
                                     f"device status {st} (a bounded wait ran out)")
    return (o, lse) if return_lse else o
