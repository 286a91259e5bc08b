"""Generate the golden fixtures that pin the CPU oracle to the reference itself.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py /path/to/polyhedral

It imports the reference's own Python (``gpu/blockindex.py``, ``gpu/permute.py``,
``gpu/masks_gpu.py``, ``gpu/reference.py``, ``src/polyattn``) and its kernel-math
test helpers (``tests/test_kernel_math.py``), evaluates them on seeded inputs and
writes the results next to this script:

* ``blockindex_small.npz``  -- full ``BlockIndex`` arrays, N <= 2048, every
  reference mask spec and the seven tile shapes of ``gpu/test_correctness.py:21``,
  plus residue-permuted masks built as ``M[p][:, p]`` (``gpu/test_correctness.py:71``).
* ``blockindex_configs.json`` -- SHA-256 of the ``BlockIndex`` arrays at the five
  benchmark configurations' full sizes (N = 1024 ... 32768), with elements/live.
* ``perm.json`` -- ``residue_perm`` / ``invert`` known answers.
* ``attention_small.npz`` -- ``attention_reference`` outputs on small seeded inputs.
* ``attention_c1.npz`` -- ``attention_reference`` on configuration 1 (window-128,
  B1 H4 N1024 D64, fp32, seed 0), plus the input checksums.
* ``kernel_math.npz`` -- the reference's float64 online-softmax simulation.
* ``counts.json`` -- ``live_count``, ``cost.cost`` and ``selector.costs`` values.

Nothing at test time reads the reference; tests read only these fixtures.
"""
import hashlib
import json
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def sha(a):
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.tobytes()).hexdigest()


class _Dense:
    """The reference's own adapter for an explicit boolean matrix
    (``gpu/test_correctness.py:90-95``)."""

    def __init__(self, M):
        self.M = M

    def row_cols(self, q, N):
        return self.M[q]


def main(ref_root):
    ref_root = Path(ref_root)
    sys.path.insert(0, str(ref_root / "gpu"))
    sys.path.insert(0, str(ref_root / "src"))
    sys.path.insert(0, str(ref_root / "tests"))
    import torch
    import blockindex
    import masks_gpu
    import permute
    import reference
    from polyattn import cost, masks, selector
    import test_kernel_math as tkm

    TILES = [(128, 128), (128, 32), (64, 64), (32, 32), (16, 16), (128, 16), (16, 128)]

    # the configuration masks the reference's SPECS lacks, built from its own classes
    extra = {
        "local64+str8": masks.LocalStrided(64, 8),
        "sinks4+win512": masks.SinksWindow(4, 512),
        "local1024+str16": masks.LocalStrided(1024, 16),
        "window-1024": masks.SlidingWindow(1024),
        "dilated-16": masks.Dilated(16),
    }

    def mask_of(name):
        if name in masks_gpu.SPECS:
            return masks_gpu.numpy_mask(name)
        return extra[name]

    def dense(m, N):
        return np.stack([m.row_cols(q, N) for q in range(N)])

    def far_mask(N, w=1024, s=16):
        """Part 2 of the configuration-5 split: the union minus the window part."""
        return dense(masks.LocalStrided(w, s), N) & ~dense(masks.SlidingWindow(w), N)

    # ------------------------------------------------------------ block index
    small = {}
    cases = []
    for name in list(masks_gpu.SPECS) + list(extra):
        for N in (512,):
            for BQ, A in TILES:
                cases.append((name, N, BQ, A, 0))
    for name, s in (("dilated-4", 4), ("dilated-8", 8), ("local64+str8", 8),
                    ("local256+str8", 8), ("dilated-16", 16), ("sinks4+win256", 4)):
        for BQ, A in ((16, 16), (128, 32), (64, 64), (128, 128), (32, 16)):
            cases.append((name, 1024, BQ, A, s))
    for BQ, A in TILES:
        cases.append(("window-128", 1024, BQ, A, 0))          # configuration 1
    for BQ, A in ((128, 32), (128, 128), (16, 16)):
        cases.append(("far1024+str16", 2048, BQ, A, 16))
        cases.append(("window-1024", 2048, BQ, A, 0))
    meta = []
    for idx, (name, N, BQ, A, s) in enumerate(cases):
        if name == "far1024+str16":
            M = far_mask(N)
        else:
            M = dense(mask_of(name), N)
        if s:
            p = permute.residue_perm(N, s)
            M = M[p][:, p]
        bi = blockindex.build(_Dense(M), N, BQ, A)
        key = f"c{idx}"
        small[key + "_kv_idx"] = bi.kv_idx
        small[key + "_kv_num"] = bi.kv_num
        small[key + "_kv_partial"] = bi.kv_partial
        meta.append(dict(key=key, name=name, N=N, BQ=BQ, A=A, s=s,
                         elements=int(bi.elements), live=int(bi.live)))
        if s == 0 and name != "far1024+str16":
            pred, _ = cost.cost(mask_of(name), N, BQ, A, exact_only=True)
            assert int(pred) == bi.elements, (name, N, BQ, A)
    small["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "blockindex_small.npz", **small)
    print(f"blockindex_small: {len(cases)} cases")

    # full-size configurations: hashes only
    big_cases = [
        ("c1", "window-128", 1024, 128, 32, 0),
        ("c1", "window-128", 1024, 128, 128, 0),
        ("c2", "dilated-4", 8192, 128, 32, 4),
        ("c2", "dilated-4", 8192, 128, 32, 0),
        ("c2", "dilated-4", 8192, 128, 128, 4),
        ("c3", "local64+str8", 16384, 16, 16, 8),
        ("c3", "local64+str8", 16384, 128, 32, 8),
        ("c3", "local64+str8", 16384, 128, 128, 8),
        ("c3", "local64+str8", 16384, 128, 32, 0),
        ("c4", "sinks4+win512", 8192, 128, 32, 0),
        ("c4", "sinks4+win512", 8192, 128, 128, 0),
        ("c5", "window-1024", 32768, 128, 128, 0),
        ("c5", "window-1024", 32768, 128, 32, 0),
        ("c5", "far1024+str16", 32768, 128, 32, 16),
        ("c5", "far1024+str16", 32768, 128, 128, 16),
    ]
    big = []
    for cfg, name, N, BQ, A, s in big_cases:
        t0 = time.time()
        M = far_mask(N) if name == "far1024+str16" else dense(mask_of(name), N)
        if s:
            p = permute.residue_perm(N, s)
            M = M[p][:, p]
        bi = blockindex.build(_Dense(M), N, BQ, A)
        del M
        big.append(dict(config=cfg, name=name, N=N, BQ=BQ, A=A, s=s,
                        elements=int(bi.elements), live=int(bi.live),
                        max_kv=int(bi.kv_idx.shape[1]),
                        kv_idx=sha(bi.kv_idx), kv_num=sha(bi.kv_num),
                        kv_partial=sha(bi.kv_partial),
                        kv_num_sum=int(bi.kv_num.sum()),
                        partial_sum=int(bi.kv_partial.sum())))
        print(f"  {cfg} {name} N={N} {BQ}x{A} s={s}: {time.time() - t0:.1f}s")
    (HERE / "blockindex_configs.json").write_text(json.dumps(big, indent=1))

    # ------------------------------------------------------------ permutation
    perms = []
    for N, s in ((16, 4), (10, 4), (17, 3), (1024, 8), (8192, 4), (16384, 8),
                 (32768, 16), (7, 1), (12, 12)):
        p = permute.residue_perm(N, s)
        inv = permute.invert(torch.from_numpy(p)).numpy()
        perms.append(dict(N=N, s=s,
                          perm=p.tolist() if N <= 64 else None,
                          perm_sha=sha(p.astype(np.int32)),
                          inv=inv.tolist() if N <= 64 else None,
                          inv_sha=sha(inv.astype(np.int32))))
    (HERE / "perm.json").write_text(json.dumps(perms, indent=1))

    # ------------------------------------------------------------ attention
    att = {}
    att_meta = []
    names = ["causal", "window-128", "dilated-8", "local256+str8", "twoband-1000",
             "sinks4+win8", "sinks4+win256", "dilated-4"]
    for i, name in enumerate(names):
        BH, N, D = 1, 256, 32
        g = torch.Generator().manual_seed(100 + i)
        q, k, v = (torch.randn(BH, N, D, generator=g) for _ in range(3))
        Mb = masks_gpu.dense_bool(name, N, device="cpu")
        o = reference.attention_reference(q, k, v, Mb)
        att[f"a{i}_o"] = o.numpy()
        att_meta.append(dict(key=f"a{i}", name=name, BH=BH, N=N, D=D, seed=100 + i,
                             q_sha=sha(q.numpy()), k_sha=sha(k.numpy()),
                             v_sha=sha(v.numpy())))
    # a dead row: the reference maps it to zeros (gpu/reference.py:12)
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(1, 64, 16, generator=g) for _ in range(3))
    Mb = masks_gpu.dense_bool("window-128", 64, device="cpu").clone()
    Mb[5] = False
    att["dead_o"] = reference.attention_reference(q, k, v, Mb).numpy()
    att_meta.append(dict(key="dead", name="window-128", dead_row=5, BH=1, N=64, D=16,
                         seed=7, q_sha=sha(q.numpy()), k_sha=sha(k.numpy()),
                         v_sha=sha(v.numpy())))
    att["meta"] = np.frombuffer(json.dumps(att_meta).encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "attention_small.npz", **att)

    # configuration 1, in full
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 4, 1024, 64, generator=g) for _ in range(3))
    q, k, v = (x.reshape(4, 1024, 64) for x in (q, k, v))
    Mb = masks_gpu.dense_bool("window-128", 1024, device="cpu")
    o = reference.attention_reference(q, k, v, Mb)
    np.savez_compressed(HERE / "attention_c1.npz", o=o.numpy(),
                        meta=np.frombuffer(json.dumps(dict(
                            q_sha=sha(q.numpy()), k_sha=sha(k.numpy()),
                            v_sha=sha(v.numpy()))).encode(), dtype=np.uint8))

    # ------------------------------------------------------------ kernel math
    km = {}
    rng = np.random.default_rng(0)
    qq, kk, vv = (rng.standard_normal((tkm.N, tkm.D)) for _ in range(3))
    for i, (m, BQ, A) in enumerate(tkm.CASES):
        M = np.stack([m.row_cols(r, tkm.N) for r in range(tkm.N)])
        km[f"k{i}"] = tkm._kernel_math(M, qq, kk, vv, BQ, A, -1e30)
    km["cases"] = np.frombuffer(json.dumps(
        [dict(name=m.name, BQ=BQ, A=A) for m, BQ, A in tkm.CASES]).encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "kernel_math.npz", **km)

    # ------------------------------------------------------------ counts
    counts = dict(live={}, cost={}, selector={}, select={})
    cfg_masks = {"c1": ("window-128", 1024), "c2": ("dilated-4", 8192),
                 "c3": ("local64+str8", 16384), "c4": ("sinks4+win512", 8192),
                 "c5": ("local1024+str16", 32768)}
    for cfg, (name, N) in cfg_masks.items():
        m = mask_of(name)
        counts["live"][f"{name}@{N}"] = int(m.live_count(N))
        for BQ, A in ((128, 128), (128, 32), (16, 16)):
            c, _ = cost.cost(m, N, BQ, A, exact_only=True)
            counts["cost"][f"{name}@{N}:{BQ}x{A}"] = int(c)
            cs = selector.costs(m, N, BQ, A)
            if cs is not None:
                counts["selector"][f"{name}@{N}:{BQ}x{A}"] = {k: int(v) for k, v in cs.items()}
            counts["select"][f"{name}@{N}:{BQ}x{A}"] = selector.select(m, N, BQ, A)
    for name in list(masks_gpu.SPECS) + list(extra):
        m = mask_of(name)
        for N in (512, 1024, 4096):
            counts["live"][f"{name}@{N}"] = int(m.live_count(N))
        for BQ, A in ((16, 16), (128, 32), (64, 64)):
            cs = selector.costs(m, 1024, BQ, A)
            counts["select"][f"{name}@1024:{BQ}x{A}"] = selector.select(m, 1024, BQ, A)
            if cs is not None:
                counts["selector"][f"{name}@1024:{BQ}x{A}"] = {k: int(v) for k, v in cs.items()}
    (HERE / "counts.json").write_text(json.dumps(counts, indent=1))
    print("done")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
