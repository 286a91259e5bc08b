"""Build ``libpolyattn_sm100.so`` in-tree from ``csrc/*.cu`` with nvcc for sm_100a.

    python -m polyhedral_b200.build [-v]

Objects go to ``polyhedral_b200/_build/``; the shared library lands next to this
file, where ``polyhedral_b200._lib`` loads it from.  Rebuilds only when a source,
header or these flags changed.
"""
import concurrent.futures
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libpolyattn_sm100.so"

SOURCES = ["capi_util.cu", "blockindex.cu", "permute.cu", "merge.cu", "attn.cu",
           "attn_k128.cu", "attn_k128r.cu", "attn_k64.cu", "attn_k64r.cu",
           "attn_k128m.cu", "attn_k128rm.cu", "attn_k64m.cu", "attn_k64rm.cu",
           "attn_db128.cu", "attn_db128r.cu", "attn_db64.cu", "attn_db64r.cu",
           "attn_k128g.cu", "attn_k64g.cu",
           "attn_k128p.cu", "attn_k128rp.cu", "attn_k64p.cu", "attn_k64rp.cu", "attn_noalloc.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]


def _nvcc():
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")
    return cand


def _digest():
    h = hashlib.sha256()
    h.update(" ".join(NVCC_FLAGS).encode())
    for p in sorted(list(CSRC.glob("*")) + list(INCLUDE.glob("*.h"))):
        if p.is_file():
            h.update(p.name.encode())
            h.update(p.read_bytes())
    return h.hexdigest()


def _compile(src, verbose):
    obj = BUILD / (Path(src).stem + ".o")
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c",
           str(CSRC / src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"--- {src}\n{r.stderr.strip()}", flush=True)
    return obj, r.stderr


def build(verbose=False, force=False):
    """Compile every CUDA source for sm_100a and link the shared library.
    Returns the library path."""
    BUILD.mkdir(exist_ok=True)
    stamp = BUILD / "stamp"
    digest = _digest()
    if not force and LIB.exists() and stamp.exists() and stamp.read_text() == digest:
        return LIB
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    objs = [str(o) for o, _ in results]
    (BUILD / "ptxas.txt").write_text("\n".join(e for _, e in results))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
           "-Xcompiler", "-fPIC", *objs, "-o", str(tmp)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    stamp.write_text(digest)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
