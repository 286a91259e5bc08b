"""The C-ABI library loads without a GPU, exports every entry point the header
declares with the argument structs laid out as the header lays them out, and
rejects bad arguments before any launch (these calls touch no device)."""
import ctypes
import re
from pathlib import Path

import pytest

from polyhedral_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "polyattn.h"


def _declared_functions():
    text = HEADER.read_text()
    return set(re.findall(r"^\s*PA_API\s+(?:const\s+)?[a-z_0-9]+\*?\s+\**(pa_[a-z_0-9]+)\s*\(", text, re.M))


def _struct_fields(name):
    text = HEADER.read_text()
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), text, re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        decl = re.sub(r"^(const\s+)?[a-z_0-9]+\s*\**\s*", "", decl)
        for part in decl.split(","):
            fields.append(part.strip().lstrip("*").strip())
    return fields


@pytest.fixture(scope="module")
def lib():
    from polyhedral_b200 import build
    build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    declared = _declared_functions()
    assert len(declared) >= 12
    assert declared == set(_lib.SIGNATURES), declared ^ set(_lib.SIGNATURES)
    for name in declared:
        assert hasattr(lib, name), name


@pytest.mark.parametrize("cname,pyname", [("pa_pred", "PaPred"), ("pa_rows", "PaRows"),
                                          ("pa_attn_args", "PaAttnArgs"),
                                          ("pa_merge_args", "PaMergeArgs")])
def test_struct_layout_matches_header(cname, pyname):
    fields = _struct_fields(cname)
    py = [f[0] for f in getattr(_lib, pyname)._fields_]
    assert fields == py


def test_abi_version(lib):
    assert lib.pa_abi_version() == _lib.ABI_VERSION


def test_argument_errors_before_launch(lib):
    pred = _lib.PaPred(_lib.c_i32(1), 128, 0, 0)
    # N not a multiple of BQ
    rc = lib.pa_block_index(ctypes.byref(pred), 1000, 128, 32, None, None, ctypes.c_void_p(16), 64,
                            ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), None)
    assert rc == _lib.PA_ERR_ARG
    assert b"multiple of BQ" in lib.pa_last_error()
    # unknown kind
    bad = _lib.PaPred(99, 0, 0, 0)
    rc = lib.pa_block_index(ctypes.byref(bad), 1024, 128, 32, None, None, ctypes.c_void_p(16), 64,
                            ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), None)
    assert rc == _lib.PA_ERR_ARG and b"unknown mask kind" in lib.pa_last_error()
    # DILATED needs a positive stride
    d0 = _lib.PaPred(2, 0, 0, 0)
    rc = lib.pa_block_index(ctypes.byref(d0), 1024, 128, 32, None, None, ctypes.c_void_p(16), 64,
                            ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), None)
    assert rc == _lib.PA_ERR_ARG
    # attention: unsupported head dim, bad tile
    a = _lib.PaAttnArgs()
    a.q = a.k = a.v = a.o = a.kv_num = 16
    a.BH, a.N, a.D, a.dtype, a.BQ, a.A = 1, 1024, 96, 0, 128, 32
    assert lib.pa_attn_fwd(ctypes.byref(a), ctypes.c_void_p(256), 1 << 20, None) == _lib.PA_ERR_ARG
    assert b"D=96" in lib.pa_last_error()
    a.D, a.A = 128, 48
    assert lib.pa_attn_plan(ctypes.byref(a), ctypes.c_void_p(256), 1 << 20, None) == _lib.PA_ERR_ARG
    a.A = 32
    assert lib.pa_attn_workspace_size(ctypes.byref(a)) > 0
    # workspace too small
    assert lib.pa_attn_fwd(ctypes.byref(a), ctypes.c_void_p(256), 16, None) == _lib.PA_ERR_ARG
    # gathered K/V: multiplier range, combinations, head stride vs row stride
    a.k_row_stride = a.v_row_stride = 128
    a.k_bh_stride = a.v_bh_stride = 1024 * 128
    a.gather_kv, a.gather_mult = 1, 17
    assert lib.pa_attn_fwd(ctypes.byref(a), ctypes.c_void_p(256), 1 << 20, None) == _lib.PA_ERR_ARG
    assert b"gather_mult=17" in lib.pa_last_error()
    a.gather_mult, a.residue_stride = 4, 4
    assert lib.pa_attn_fwd(ctypes.byref(a), ctypes.c_void_p(256), 1 << 20,
                           None) == _lib.PA_ERR_UNSUPPORTED
    a.residue_stride, a.kv_rows = 0, 64
    assert lib.pa_attn_fwd(ctypes.byref(a), ctypes.c_void_p(256), 1 << 20,
                           None) == _lib.PA_ERR_UNSUPPORTED
    a.kv_rows, a.k_bh_stride = 0, 100
    assert lib.pa_attn_fwd(ctypes.byref(a), ctypes.c_void_p(256), 1 << 20,
                           None) == _lib.PA_ERR_UNSUPPORTED
    assert b"multiple of its row stride" in lib.pa_last_error()
    a.k_bh_stride, a.sched_heads = 1024 * 128, -1
    assert lib.pa_attn_fwd(ctypes.byref(a), ctypes.c_void_p(256), 1 << 20, None) == _lib.PA_ERR_ARG
    assert b"sched_heads=-1" in lib.pa_last_error()
    a.sched_heads, a.perm_kv = 0, 20
    assert lib.pa_attn_fwd(ctypes.byref(a), ctypes.c_void_p(256), 1 << 20, None) == _lib.PA_ERR_ARG
    assert b"16-byte aligned perm_kv" in lib.pa_last_error()
    # merge: null pointers
    m = _lib.PaMergeArgs()
    assert lib.pa_lse_merge(ctypes.byref(m), None) == _lib.PA_ERR_ARG
    # permute: too many tensors
    rows = (_lib.PaRows * 5)()
    assert lib.pa_permute_rows(rows, 5, 1, 16, 256, ctypes.c_void_p(16), 0, None) == _lib.PA_ERR_ARG


def test_python_layer_raises_without_gpu_work():
    import torch
    from polyhedral_b200 import attention, permute
    with pytest.raises(RuntimeError):
        permute.apply_perm(torch.zeros(1, 4, 8), torch.arange(4))
    q = torch.zeros(1, 256, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="GPU only"):
        attention.block_sparse_attention(q, q, q, None, None, None, 1, 128, 0, 0, 128, 32)
    with pytest.raises(ValueError, match="gather_mult"):
        attention.block_sparse_attention(q, q, q, None, None, None, 1, 128, 0, 0, 128, 32,
                                         gather_mult=17)
    with pytest.raises(AssertionError):
        attention.block_sparse_attention(q, q, q, None, None, None, 1, 128, 0, 0, 100, 32)
