"""ctypes binding of ``libpolyattn_sm100.so`` (declared in ``include/polyattn.h``).

The library is built in-tree by ``polyhedral_b200.build``.  There is no other
implementation behind these calls: if the library is missing, every operation
raises instead of computing anything on the CPU.
"""
import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpolyattn_sm100.so"

PA_OK, PA_ERR_ARG, PA_ERR_CUDA, PA_ERR_UNSUPPORTED, PA_ERR_DEVICE = 0, -1, -2, -3, -4
PA_BF16, PA_F16 = 0, 1

c_i32, c_i64, c_f32, c_vp, c_sz = (ctypes.c_int32, ctypes.c_int64, ctypes.c_float,
                                   ctypes.c_void_p, ctypes.c_size_t)


class PaPred(ctypes.Structure):
    _fields_ = [("kind", c_i32), ("p0", c_i32), ("p1", c_i32), ("p2", c_i32)]


class PaRows(ctypes.Structure):
    _fields_ = [("src", c_vp), ("dst", c_vp),
                ("src_bh_stride", c_i64), ("src_row_stride", c_i64),
                ("dst_bh_stride", c_i64), ("dst_row_stride", c_i64)]


class PaAttnArgs(ctypes.Structure):
    _fields_ = [("q", c_vp), ("k", c_vp), ("v", c_vp), ("o", c_vp), ("lse", c_vp),
                ("BH", c_i32), ("N", c_i32), ("D", c_i32), ("dtype", c_i32),
                ("q_bh_stride", c_i64), ("q_row_stride", c_i64),
                ("k_bh_stride", c_i64), ("k_row_stride", c_i64),
                ("v_bh_stride", c_i64), ("v_row_stride", c_i64),
                ("o_bh_stride", c_i64), ("o_row_stride", c_i64),
                ("lse_bh_stride", c_i64),
                ("kv_idx", c_vp), ("kv_num", c_vp), ("kv_partial", c_vp),
                ("kv_stride", c_i32), ("BQ", c_i32), ("A", c_i32),
                ("perm_q", c_vp), ("perm_kv", c_vp), ("o_row_map", c_vp),
                ("pred", PaPred), ("scale", c_f32), ("residue_stride", c_i32),
                ("merge", c_i32), ("kv_rows", c_i32),
                ("gather_kv", c_i32), ("gather_mult", c_i32), ("gather_scatter", c_i32),
                ("sched_heads", c_i32), ("row_threads", c_i32)]


class PaMergeArgs(ctypes.Structure):
    _fields_ = [("o1", c_vp), ("lse1", c_vp), ("o2", c_vp), ("lse2", c_vp),
                ("o", c_vp), ("lse", c_vp),
                ("BH", c_i32), ("N", c_i32), ("D", c_i32), ("dtype", c_i32),
                ("o1_bh_stride", c_i64), ("o1_row_stride", c_i64),
                ("o2_bh_stride", c_i64), ("o2_row_stride", c_i64),
                ("o_bh_stride", c_i64), ("o_row_stride", c_i64),
                ("lse1_bh_stride", c_i64), ("lse2_bh_stride", c_i64),
                ("lse_bh_stride", c_i64), ("row_map2", c_vp)]


# name -> (restype, argtypes); every symbol include/polyattn.h declares
SIGNATURES = {
    "pa_last_error": (ctypes.c_char_p, []),
    "pa_abi_version": (ctypes.c_int, []),
    "pa_block_index": (ctypes.c_int, [ctypes.POINTER(PaPred), c_i32, c_i32, c_i32, c_vp, c_vp,
                                      c_vp, c_i32, c_vp, c_vp, c_vp, c_vp]),
    "pa_block_index_dense": (ctypes.c_int, [c_vp, c_i32, c_i32, c_i32, c_vp, c_i32, c_vp, c_vp,
                                            c_vp, c_vp]),
    "pa_residue_perm": (ctypes.c_int, [c_i32, c_i32, c_vp, c_vp]),
    "pa_invert_perm": (ctypes.c_int, [c_vp, c_i32, c_vp, c_vp]),
    "pa_permute_rows": (ctypes.c_int, [ctypes.POINTER(PaRows), c_i32, c_i32, c_i32, c_i32, c_vp,
                                       c_i32, c_vp]),
    "pa_attn_workspace_size": (c_sz, [ctypes.POINTER(PaAttnArgs)]),
    "pa_attn_plan": (ctypes.c_int, [ctypes.POINTER(PaAttnArgs), c_vp, c_sz, c_vp]),
    "pa_attn_fwd": (ctypes.c_int, [ctypes.POINTER(PaAttnArgs), c_vp, c_sz, c_vp]),
    "pa_attn_status": (ctypes.c_int, [c_vp, ctypes.POINTER(c_i32), c_vp]),
    "pa_attn_fwd_withheld": (ctypes.c_int, [ctypes.POINTER(PaAttnArgs), c_vp, c_sz, c_i64, c_vp]),
    "pa_attn_fwd_noalloc": (ctypes.c_int, [ctypes.POINTER(PaAttnArgs), c_vp]),
    "pa_attn_noalloc_status": (ctypes.c_int, [ctypes.POINTER(c_i32), c_vp]),
    "pa_lse_merge": (ctypes.c_int, [ctypes.POINTER(PaMergeArgs), c_vp]),
}

ABI_VERSION = 8

_lib = None


class PolyattnError(RuntimeError):
    """A C-ABI call returned an error code."""

    def __init__(self, fn, code, msg):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


def load():
    """Load the library once; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("POLYATTN_LIB", LIB_PATH))
    if not path.exists():
        raise RuntimeError(
            f"{path} is missing: build it with `python -m polyhedral_b200.build` "
            "(there is no fallback implementation)")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.pa_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{path}: ABI {lib.pa_abi_version()} != expected {ABI_VERSION}")
    _lib = lib
    return lib


def on_device(device):
    """Context in which `device` is the current CUDA device.  The library launches on
    the current device, so a call on tensors of another device switches to theirs for
    its duration (a no-op context when it is current already, the common case)."""
    import contextlib
    import torch
    idx = device if isinstance(device, int) else torch.device(device).index
    if idx is None or idx == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(idx)


def call(name, *args, device=None):
    """Call a C-ABI entry point and raise PolyattnError on a nonzero status; with
    `device`, that device is current during the call."""
    lib = load()
    if device is None:
        rc = getattr(lib, name)(*args)
    else:
        with on_device(device):
            rc = getattr(lib, name)(*args)
    if rc != PA_OK:
        msg = lib.pa_last_error().decode(errors="replace")
        raise PolyattnError(name, rc, msg)
    return rc


def stream_handle(device=None):
    """Raw cudaStream_t of torch's current stream on `device`.  Read through torch's
    raw-stream accessor when it has one (no Stream object is built per call, which
    is most of a small call's host time), else through ``current_stream``."""
    import torch
    if device is None:
        idx = torch.cuda.current_device()
    elif isinstance(device, int):
        idx = device
    else:
        device = torch.device(device)
        idx = device.index if device.index is not None else torch.cuda.current_device()
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return ctypes.c_void_p(raw(idx))
    return ctypes.c_void_p(torch.cuda.current_stream(idx).cuda_stream)
