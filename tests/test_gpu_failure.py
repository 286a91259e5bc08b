"""Failure detection of the attention forward, exercised without a GPU fault.

Every barrier wait in the forward kernels is bounded; when one runs out the kernel
records a status code in its workspace, stops issuing work, drains the copies and
MMAs it issued, frees TMEM and exits, so the context stays usable.  The test hook
``pa_attn_fwd_withheld`` never issues one Q-tile load (a barrier that nothing
completes) and gives every wait a 2 ms limit (0.5 ms for the MMA issuer's waits on
Q tiles, so theirs is the wait that runs out first): the MMA issuer's wait on that
tile must run out, ``pa_attn_status`` must report code 1 (a Q-tile wait), and the next
ordinary forward on the same workspace must report 0 and produce the same result
as before the failure.  (The reference's only failure handling is the Triton launch
retry of gpu/triton_attn.py:224-240.)
"""
import ctypes

import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

DEV_TIMEOUT_Q = 1


def _setup(kv_rows, row_threads, merge, N=2048, BH=3):
    from polyhedral_b200 import attention, blockindex, masks
    spec = (O.LOCAL_STRIDED, 256, 8, 0)
    dbi = blockindex.build_device(masks.from_spec(*spec), N, 128, 32)
    plan = attention.make_plan(dbi.kv_idx, dbi.kv_num, dbi.kv_partial, N, 128, 32)
    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = (torch.randn(BH, N, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    kw = dict(plan=plan, return_lse=True, kv_rows=kv_rows, row_threads=row_threads)
    return spec, plan, q, k, v, kw


def _args_of(plan, q, k, v, o, lse, spec, kv_rows, row_threads, merge):
    from polyhedral_b200 import _lib
    a = _lib.PaAttnArgs()
    BH, N, D = q.shape
    a.q, a.k, a.v, a.o, a.lse = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr()
    a.BH, a.N, a.D, a.dtype = BH, N, D, _lib.PA_BF16
    a.q_bh_stride, a.q_row_stride = q.stride(0), q.stride(1)
    a.k_bh_stride, a.k_row_stride = k.stride(0), k.stride(1)
    a.v_bh_stride, a.v_row_stride = v.stride(0), v.stride(1)
    a.o_bh_stride, a.o_row_stride = o.stride(0), o.stride(1)
    a.lse_bh_stride = lse.stride(0)
    a.kv_idx, a.kv_num, a.kv_partial = (plan.kv_idx.data_ptr(), plan.kv_num.data_ptr(),
                                        plan.kv_partial.data_ptr())
    a.kv_stride, a.BQ, a.A = plan.kv_stride, 128, 32
    a.pred = _lib.PaPred(*spec)
    a.kv_rows, a.row_threads, a.merge = kv_rows, row_threads, int(merge)
    return a


@pytest.mark.parametrize("kv_rows,row_threads,merge", [(0, 1, False), (0, 2, False),
                                                       (64, 1, False), (0, 1, True)])
def test_bounded_wait_runs_out_and_reports(kv_rows, row_threads, merge):
    from polyhedral_b200 import _lib
    from polyhedral_b200.triton_attn import block_sparse_attention
    lib = _lib.load()
    spec, plan, q, k, v, kw = _setup(kv_rows, row_threads, merge)
    BH, N, D = q.shape
    # a clean forward first: the result the forward after the failure must repeat
    o0 = torch.zeros_like(q)
    l0 = torch.full((BH, N), float("-inf"), device="cuda")
    ref = block_sparse_attention(q, k, v, None, None, None, *spec, 128, 32, out=o0, lse_out=l0,
                                 merge=merge, check=True, **kw)
    assert plan.status() == 0
    o1 = torch.zeros_like(q)
    l1 = torch.full((BH, N), float("-inf"), device="cuda")
    a = _args_of(plan, q, k, v, o1, l1, spec, kv_rows, row_threads, merge)
    ws = plan.workspace
    stream = _lib.stream_handle(q.device)
    rc = lib.pa_attn_fwd_withheld(ctypes.byref(a), ws.data_ptr(), ws.numel(), 2_000_000, stream)
    assert rc == 0, lib.pa_last_error()
    st = ctypes.c_int32(0)
    assert lib.pa_attn_status(ws.data_ptr(), ctypes.byref(st), stream) == _lib.PA_ERR_DEVICE
    assert st.value == DEV_TIMEOUT_Q
    assert plan.status() == DEV_TIMEOUT_Q
    # the context is usable and the next ordinary forward on the same plan is clean
    o2 = torch.zeros_like(q)
    l2 = torch.full((BH, N), float("-inf"), device="cuda")
    out = block_sparse_attention(q, k, v, None, None, None, *spec, 128, 32, out=o2, lse_out=l2,
                                 merge=merge, check=True, **kw)
    assert plan.status() == 0
    assert torch.equal(out[0], ref[0]) and torch.equal(out[1], ref[1])


def test_cached_plan_clean_after_failure():
    """A failure recorded by one forward does not stick to the work list: the next
    check=True call that reuses the cached plan runs cleanly and does not raise."""
    from polyhedral_b200 import _lib, attention, blockindex, masks
    from polyhedral_b200.triton_attn import block_sparse_attention
    lib = _lib.load()
    N = 1024
    spec = (O.WINDOW, 128, 0, 0)
    kvi, kvn, kvp = blockindex.to_cuda(blockindex.build(masks.from_spec(*spec), N, 128, 32))
    q, k, v = (torch.randn(2, N, 128, device="cuda").bfloat16() for _ in range(3))
    attention.set_plan_cache(True)
    try:
        ref = block_sparse_attention(q, k, v, kvi, kvn, kvp, *spec, 128, 32, return_lse=True,
                                     check=True)
        assert len(attention._PLAN_CACHE) == 1
        (_, _, plan), = attention._PLAN_CACHE.values()
        o = torch.empty_like(q)
        lse = torch.empty(2, N, device="cuda")
        a = _args_of(plan, q, k, v, o, lse, spec, 0, 1, False)
        ws = plan.workspace
        assert lib.pa_attn_fwd_withheld(ctypes.byref(a), ws.data_ptr(), ws.numel(), 2_000_000,
                                        _lib.stream_handle(q.device)) == 0
        assert plan.status() == DEV_TIMEOUT_Q
        out = block_sparse_attention(q, k, v, kvi, kvn, kvp, *spec, 128, 32, return_lse=True,
                                     check=True)
        assert len(attention._PLAN_CACHE) == 1 and plan.status() == 0
        assert torch.equal(out[0], ref[0]) and torch.equal(out[1], ref[1])
    finally:
        attention.set_plan_cache(False)


def test_withheld_rejects_bad_limits():
    from polyhedral_b200 import _lib
    lib = _lib.load()
    spec, plan, q, k, v, kw = _setup(0, 1, False, N=1024, BH=1)
    o = torch.empty_like(q)
    lse = torch.empty(1, 1024, device="cuda")
    a = _args_of(plan, q, k, v, o, lse, spec, 0, 1, False)
    ws = plan.workspace
    for bad in (0, 10, 2_000_000_000):
        assert lib.pa_attn_fwd_withheld(ctypes.byref(a), ws.data_ptr(), ws.numel(), bad,
                                        None) == _lib.PA_ERR_ARG
