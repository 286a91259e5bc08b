"""The driver runner resolves the reference's bare module names to this package
(CPU: only the import resolution is checked; the drivers themselves need a GPU)."""
import subprocess
import sys
import textwrap
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_style_imports_resolve_to_this_package(tmp_path):
    gpu = tmp_path / "gpu"
    gpu.mkdir()
    # a stand-in for a reference helper that must still come from the script's directory
    (gpu / "launchsweep.py").write_text("LAUNCH = ((4, 2),)\n")
    (gpu / "driver.py").write_text(textwrap.dedent("""
        import sys
        sys.path.insert(0, __file__.rsplit("/", 1)[0])
        import blockindex, bench, masks_gpu, permute
        from triton_attn import block_sparse_attention
        from launchsweep import LAUNCH
        assert blockindex.__name__ == "polyhedral_b200.blockindex"
        assert bench.__name__ == "polyhedral_b200.timing"
        assert masks_gpu.__name__ == "polyhedral_b200.masks_gpu"
        assert permute.__name__ == "polyhedral_b200.permute"
        assert block_sparse_attention.__module__ == "polyhedral_b200.attention"
        assert LAUNCH == ((4, 2),)
        import polyhedral_b200.attention as attention
        assert attention._plan_cache_on        # the drivers reuse one index per forward
        for name in ("time_ms", "paired_time", "report"):
            assert callable(getattr(bench, name))
        for name in ("build", "to_cuda"):
            assert callable(getattr(blockindex, name))
        for name in ("numpy_mask", "triton_params", "dense_bool", "flex_mask_mod",
                     "check_agreement"):
            assert callable(getattr(masks_gpu, name))
        for name in ("residue_perm", "identity_perm", "apply_perm", "invert",
                     "permutation_cost_ms"):
            assert callable(getattr(permute, name))
        print("ok", sys.argv[1:])
    """))
    r = subprocess.run([sys.executable, "-m", "polyhedral_b200.dropin", str(gpu / "driver.py"),
                        "--flag"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "ok ['--flag']" in r.stdout
