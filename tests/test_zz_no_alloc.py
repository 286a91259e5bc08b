"""pa_attn_fwd_noalloc -- the forward for callers that cannot allocate device
memory -- against the regular pa_attn_plan + pa_attn_fwd path.

Some users of this library run where they may not allocate GPU memory (inside
another framework's pool, under a fixed budget, or through a binding with no
device allocator); the no-alloc entry point keeps its work list in a fixed array
inside the library instead of a caller workspace.  This test calls both entry
points through the C ABI on the same inputs and requires bit-identical outputs
(the same kernels run on the same data), reads the no-alloc call's own device
status from the library's array (pa_attn_noalloc_status), and does so for two
calls in a row with different masks, sizes and tile shapes: the array keeps the
first call's contents, so the second call shows that nothing stale is read.  It
lives in its own file named to be collected last, and runs alone in a fresh
process as well.
"""
import ctypes

import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def _args(q, k, v, o, lse, dbi, spec, s, BQ, A):
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
    a.kv_idx, a.kv_num, a.kv_partial = (dbi.kv_idx.data_ptr(), dbi.kv_num.data_ptr(),
                                        dbi.kv_partial.data_ptr())
    a.kv_stride, a.BQ, a.A = dbi.kv_idx.shape[1], BQ, A
    a.residue_stride = s
    a.pred = _lib.PaPred(*spec)
    a.scale = 0.0
    return a


# two calls in a row: a dense index with a large work list first, then a sparser one
# with another N, tile shape and basis, whose work list is smaller and laid out
# differently in the same array
SEQUENCES = {
    "causal then dilated-4 rp4": [((O.CAUSAL, 0, 0, 0), 4096, 0, 128, 16),
                                  ((O.DILATED, 4, 0, 0), 2048, 4, 128, 32)],
    "dilated-4 rp4 then sinks": [((O.DILATED, 4, 0, 0), 4096, 4, 128, 32),
                                 ((O.SINKS, 512, 4, 0), 2048, 0, 16, 16)],
}


@pytest.mark.parametrize("seq", sorted(SEQUENCES))
def test_noalloc_matches_workspace_path(seq):
    from polyhedral_b200 import _lib, blockindex, masks, permute
    lib = _lib.load()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    stream = _lib.stream_handle(dev)
    outs = []
    for call, (spec, N, s, BQ, A) in enumerate(SEQUENCES[seq]):
        perm = permute.residue_perm_device(N, s, dev) if s else None
        dbi = blockindex.build_device(masks.from_spec(*spec), N, BQ, A, perm_q=perm,
                                      perm_kv=perm, device=dev)
        g = torch.Generator(device=dev).manual_seed(100 + call)
        q, k, v = (torch.randn(4, N, 128, device=dev, generator=g).bfloat16() for _ in range(3))
        o_ref, o_na = torch.empty_like(q), torch.full_like(q, float("nan"))
        l_ref = torch.empty(4, N, device=dev)
        l_na = torch.full((4, N), float("nan"), device=dev)
        # existing entry point with a caller-allocated workspace
        a = _args(q, k, v, o_ref, l_ref, dbi, spec, s, BQ, A)
        nbytes = lib.pa_attn_workspace_size(ctypes.byref(a))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        assert lib.pa_attn_plan(ctypes.byref(a), ws.data_ptr(), nbytes, stream) == 0
        assert lib.pa_attn_fwd(ctypes.byref(a), ws.data_ptr(), nbytes, stream) == 0
        st = ctypes.c_int32(-1)
        assert lib.pa_attn_status(ws.data_ptr(), ctypes.byref(st), stream) == 0 and st.value == 0
        # the entry point that allocates nothing, and its own status word
        b = _args(q, k, v, o_na, l_na, dbi, spec, s, BQ, A)
        rc = lib.pa_attn_fwd_noalloc(ctypes.byref(b), stream)
        assert rc == 0, lib.pa_last_error()
        st = ctypes.c_int32(-1)
        rc = lib.pa_attn_noalloc_status(ctypes.byref(st), stream)
        assert rc == 0 and st.value == 0, (rc, st.value, lib.pa_last_error())
        # the same kernels on the same inputs: bit-identical results
        assert torch.equal(o_na, o_ref)
        assert torch.equal(l_na, l_ref)
        outs.append(o_na.float().abs().sum().item())
    assert outs[0] != outs[1]   # the two calls really computed different things


def test_noalloc_rejects_oversize_request():
    from polyhedral_b200 import _lib
    lib = _lib.load()
    a = _lib.PaAttnArgs()
    a.q = a.k = a.v = a.o = a.kv_num = 256
    a.BH, a.N, a.D, a.dtype, a.BQ, a.A = 1, 65536, 128, _lib.PA_BF16, 128, 16
    assert lib.pa_attn_workspace_size(ctypes.byref(a)) > (4 << 20)
    assert lib.pa_attn_fwd_noalloc(ctypes.byref(a), None) == _lib.PA_ERR_ARG
    assert b"static scratch" in lib.pa_last_error()
