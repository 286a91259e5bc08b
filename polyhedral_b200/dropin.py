"""Run one of the reference's gpu/ driver scripts (test_correctness.py,
exp0_gonogo.py, exp2_class_a.py, exp7_load_imbalance.py, ...) against this
library, unmodified:

    python -m polyhedral_b200.dropin <reference>/gpu/exp2_class_a.py [args ...]

The scripts import their path modules by bare name after putting their own
directory first on sys.path (``import blockindex, bench, masks_gpu, permute``,
``from triton_attn import block_sparse_attention``).  ``install`` registers this
package's modules under those names in ``sys.modules``, which an import consults
before sys.path, so the scripts run on this library while their remaining
helpers (``reference.py``, ``launchsweep.py``, ...) still come from their directory.
"""
import runpy
import sys

from . import blockindex, masks_gpu, permute, timing, triton_attn

# reference module name -> module of this package with the same API
MODULES = {
    "blockindex": blockindex,      # gpu/blockindex.py
    "masks_gpu": masks_gpu,        # gpu/masks_gpu.py
    "permute": permute,            # gpu/permute.py
    "triton_attn": triton_attn,    # gpu/triton_attn.py
    "bench": timing,               # gpu/bench.py (time_ms, paired_time, report)
}


def install():
    """Make ``import blockindex`` (etc.) resolve to this package, and keep the
    forward's work lists across calls with the same block index
    (``attention.set_plan_cache``): the drivers call the forward repeatedly with one
    index and never rewrite it."""
    from . import attention
    for name, mod in MODULES.items():
        sys.modules[name] = mod
    attention.set_plan_cache(True)


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv:
        raise SystemExit("usage: python -m polyhedral_b200.dropin <script.py> [args ...]")
    install()
    sys.argv = argv
    runpy.run_path(argv[0], run_name="__main__")


if __name__ == "__main__":
    main()
