"""One mask definition, three consumers: the host mask objects, the CUDA kernels'
(kind, p0, p1, p2) predicate, and a torch ``mask_mod`` -- the reference's
``gpu/masks_gpu.py`` surface (:9-70), with the configurations' masks added.

``check_agreement`` compares the host rows with the torch predicate instead of
trusting that they agree.
"""
from . import masks

# Kernel mask kinds; d = q_idx - kv_idx throughout (gpu/masks_gpu.py:9).
CAUSAL, WINDOW, DILATED, LOCAL_STRIDED, TWOBAND, SINKS = 0, 1, 2, 3, 4, 5
# Lattice half of a disjoint window/lattice split: d >= p0 and d % p1 == 0.
FAR_STRIDED = 6

SPECS = {
    "causal":          (CAUSAL, 0, 0, 0, lambda: masks.Causal()),
    "window-128":      (WINDOW, 128, 0, 0, lambda: masks.SlidingWindow(128)),
    "window-512":      (WINDOW, 512, 0, 0, lambda: masks.SlidingWindow(512)),
    "window-64":       (WINDOW, 64, 0, 0, lambda: masks.SlidingWindow(64)),
    "window-1024":     (WINDOW, 1024, 0, 0, lambda: masks.SlidingWindow(1024)),
    "dilated-4":       (DILATED, 4, 0, 0, lambda: masks.Dilated(4)),
    "dilated-8":       (DILATED, 8, 0, 0, lambda: masks.Dilated(8)),
    "dilated-16":      (DILATED, 16, 0, 0, lambda: masks.Dilated(16)),
    "local256+str8":   (LOCAL_STRIDED, 256, 8, 0, lambda: masks.LocalStrided(256, 8)),
    "local64+str8":    (LOCAL_STRIDED, 64, 8, 0, lambda: masks.LocalStrided(64, 8)),
    "local1024+str16": (LOCAL_STRIDED, 1024, 16, 0, lambda: masks.LocalStrided(1024, 16)),
    "far64+str8":      (FAR_STRIDED, 64, 8, 0, lambda: masks.FarStrided(64, 8)),
    "far1024+str16":   (FAR_STRIDED, 1024, 16, 0, lambda: masks.FarStrided(1024, 16)),
    "twoband-1024":    (TWOBAND, 128, 1024, 128, lambda: masks.TwoBand(128, 1024)),
    "twoband-1000":    (TWOBAND, 128, 1000, 128, lambda: masks.TwoBand(128, 1000)),
    "sinks4+win256":   (SINKS, 256, 4, 0, lambda: masks.SinksWindow(4, 256)),
    "sinks4+win8":     (SINKS, 8, 4, 0, lambda: masks.SinksWindow(4, 8)),
    "sinks4+win512":   (SINKS, 512, 4, 0, lambda: masks.SinksWindow(4, 512)),
}


def numpy_mask(name):
    return SPECS[name][4]()


def triton_params(name):
    """(kind, p0, p1, p2) -- the name kept from the reference; the parameters
    now feed the CUDA kernels."""
    kind, p0, p1, p2, _ = SPECS[name]
    return kind, p0, p1, p2


kernel_params = triton_params


def flex_mask_mod(name):
    """A torch mask_mod(b, h, q, kv) for the named mask."""
    kind, p0, p1, p2, _ = SPECS[name]
    if kind == CAUSAL:
        return lambda b, h, q, kv: q >= kv
    if kind == WINDOW:
        return lambda b, h, q, kv: (q >= kv) & (q - kv < p0)
    if kind == DILATED:
        return lambda b, h, q, kv: (q >= kv) & ((q - kv) % p0 == 0)
    if kind == LOCAL_STRIDED:
        return lambda b, h, q, kv: (q >= kv) & (((q - kv) < p0) | ((q - kv) % p1 == 0))
    if kind == TWOBAND:
        return lambda b, h, q, kv: (q >= kv) & (((q - kv) < p0)
                                                | (((q - kv) >= p1) & ((q - kv) < p1 + p2)))
    if kind == SINKS:
        return lambda b, h, q, kv: (q >= kv) & (((q - kv) < p0) | (kv < p1))
    if kind == FAR_STRIDED:
        return lambda b, h, q, kv: ((q - kv) >= p0) & ((q - kv) % p1 == 0)
    raise ValueError(kind)


def dense_bool(name, N, device="cuda"):
    """[N, N] bool, True where live: the ground truth implementations are checked
    against."""
    import torch
    q = torch.arange(N, device=device)[:, None]
    kv = torch.arange(N, device=device)[None, :]
    return flex_mask_mod(name)(None, None, q, kv)


def check_agreement(name, N=512):
    """Host mask rows == torch predicate, element for element."""
    import numpy as np
    import torch
    a = torch.from_numpy(np.stack([numpy_mask(name).row_cols(q, N) for q in range(N)]))
    b = dense_bool(name, N, device="cpu")
    return bool(torch.equal(a, b.cpu()))
