"""Mask specs and helpers shared by the tests (oracle-side construction of the
same masks the product evaluates)."""
import numpy as np

import oracle as O

# name -> (kind, p0, p1, p2): the reference's SPECS plus the configurations' masks
SPECS = {
    "causal": (O.CAUSAL, 0, 0, 0),
    "window-128": (O.WINDOW, 128, 0, 0),
    "window-512": (O.WINDOW, 512, 0, 0),
    "window-64": (O.WINDOW, 64, 0, 0),
    "window-1024": (O.WINDOW, 1024, 0, 0),
    "dilated-4": (O.DILATED, 4, 0, 0),
    "dilated-8": (O.DILATED, 8, 0, 0),
    "dilated-16": (O.DILATED, 16, 0, 0),
    "local256+str8": (O.LOCAL_STRIDED, 256, 8, 0),
    "local64+str8": (O.LOCAL_STRIDED, 64, 8, 0),
    "local1024+str16": (O.LOCAL_STRIDED, 1024, 16, 0),
    "far64+str8": (O.FAR_STRIDED, 64, 8, 0),
    "far1024+str16": (O.FAR_STRIDED, 1024, 16, 0),
    "twoband-1024": (O.TWOBAND, 128, 1024, 128),
    "twoband-1000": (O.TWOBAND, 128, 1000, 128),
    "sinks4+win256": (O.SINKS, 256, 4, 0),
    "sinks4+win8": (O.SINKS, 8, 4, 0),
    "sinks4+win512": (O.SINKS, 512, 4, 0),
}


def oracle_mask(name, N, s=0):
    """Dense bool mask in the kernel's coordinates (permuted by residue s)."""
    M = O.dense_mask(*SPECS[name], N)
    if s:
        p = O.residue_perm(N, s)
        M = O.permuted_mask(M, p)
    return M
