"""Parity of exactly what bench.py times, at every configuration's full size, on the
inputs BASELINE.json specifies.

Each case builds ``bench.Pipeline(workload)`` -- the same block indices, residue
bases, tile shapes, split parts and kernel options (``bench.SPLITS``,
``bench.KERNEL_OPTS``) the benchmark runs, so the tested shapes cannot drift from
the benched ones -- and runs its step on Q, K, V drawn on the CPU as the
configurations say: ``g = torch.Generator().manual_seed(seed)``, then
``randn(B, H, N, D, generator=g)`` for q, k and v in that order, cast to bf16 and
reshaped to [B*H, N, D].  The result is compared on sampled heads and rows --
including the first and last row blocks and the rows around the band / lattice
boundary (i - j in {w - 1, w}) -- against an fp64 evaluation of the reference's
dense masked attention (gpu/reference.py semantics) on the same bf16 values, within
2e-2 absolute + 1e-2 relative (the north star's tolerance); the LSE likewise, and a
row without live keys must give exactly O = 0, LSE = -inf.  This is the reference's
own gate (gpu/test_correctness.py:63-82: permuted path against the dense oracle) at
the benchmark's sizes.
"""
import numpy as np
import pytest
import torch

import bench
import oracle as O
from polyhedral_b200 import masks_gpu

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def _seeded_inputs(wl):
    B, H, N, D, *_, seed, _ = bench.WORKLOADS[wl]
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(3):                       # q, k, v in that order
        x = torch.randn(B, H, N, D, generator=g)
        out.append(x.to(torch.bfloat16).reshape(B * H, N, D).cuda())
        del x
    return out


def _rows(wl):
    B, H, N, D, name, *_ = bench.WORKLOADS[wl]
    spec = masks_gpu.triton_params(name)
    rng = np.random.default_rng(N)
    r = set(rng.choice(N, 40, replace=False).tolist())
    r |= {0, 1, 63, 64, 127, 128, 255, 256, N // 2, N - 129, N - 128, N - 2, N - 1}
    w = spec[1]                              # band width of the window / local masks
    if spec[0] in (O.WINDOW, O.LOCAL_STRIDED, O.SINKS) and w < N:
        r |= {w - 1, w, w + 1, 2 * w - 1, 2 * w}
    return np.array(sorted(x for x in r if 0 <= x < N))


def _oracle_rows(q, k, v, name, heads, rows):
    """fp64 dense masked attention for the given heads and original rows."""
    N, D = q.shape[1], q.shape[2]
    M = torch.from_numpy(O.dense_mask(*masks_gpu.triton_params(name), N, rows=rows))
    outs, lses = [], []
    for h in heads:
        s = (q[h, rows].double().cpu() @ k[h].double().cpu().T) * D ** -0.5
        s = s.masked_fill(~M, float("-inf"))
        p = torch.nan_to_num(torch.softmax(s, -1), nan=0.0)
        outs.append(p @ v[h].double().cpu())
        lses.append(torch.logsumexp(s, -1))
    return torch.stack(outs), torch.stack(lses)


@pytest.mark.parametrize("wl", sorted(bench.WORKLOADS))
def test_benched_step_full_size(wl):
    B, H, N, D, name, *_ = bench.WORKLOADS[wl]
    dev = torch.device("cuda:0")
    q, k, v = _seeded_inputs(wl)
    pipe = bench.Pipeline(wl, dev)
    if wl in bench.SPLITS:                     # the parts the bench runs, as it runs them
        got = [(p.BQ, p.A, p.stride, p.kv_rows) for p in pipe.split.parts]
        want = [(bq, a, s, o.get("kv_rows", 0)) for _, bq, a, s, o in bench.SPLITS[wl]]
        assert got == want
    o = torch.full((B * H, N, D), float("nan"), device=dev, dtype=torch.bfloat16)
    lse = torch.full((B * H, N), float("nan"), device=dev)
    pipe.step(q, k, v, o, lse)
    torch.cuda.synchronize()
    for plan in pipe.plans():
        assert plan.status() == 0
    assert not torch.isnan(o).any() and not torch.isnan(lse).any()
    heads = sorted({0, (B * H) // 2, B * H - 1})
    rows = _rows(wl)
    o_ref, lse_ref = _oracle_rows(q, k, v, name, heads, rows)
    og = o[heads][:, rows].double().cpu()
    lg = lse[heads][:, rows].double().cpu()
    err = (og - o_ref).abs()
    bad = err > ATOL + RTOL * o_ref.abs()
    assert not bad.any(), f"{wl}: O max abs err {err.max().item():.3e}"
    fin = torch.isfinite(lse_ref)
    assert torch.equal(torch.isfinite(lg), fin)
    assert (lg[~fin] == lse_ref[~fin]).all() and (og[~fin] == 0).all()
    d = (lg[fin] - lse_ref[fin]).abs()
    assert (d <= ATOL + RTOL * lse_ref[fin].abs()).all(), f"{wl}: LSE max err {d.max().item():.3e}"


def test_benched_c5_step_sharded_equals_whole():
    """The sharded forward (two contiguous head ranges run one after the other on one
    GPU, as two ranks would run them) is bit-identical to the whole forward."""
    from polyhedral_b200 import shard
    wl = "c5"
    B, H, N, D, *_ = bench.WORKLOADS[wl]
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(11)
    BH = 8                                     # a slice of c5's heads keeps this quick
    q, k, v = (torch.randn(BH, N, D, device=dev, generator=g).bfloat16() for _ in range(3))
    pipe = bench.Pipeline(wl, dev)
    o_all = torch.empty(BH, N, D, device=dev, dtype=torch.bfloat16)
    l_all = torch.empty(BH, N, device=dev)
    pipe.step(q, k, v, o_all, l_all)
    o_sh = torch.empty_like(o_all)
    l_sh = torch.empty_like(l_all)
    for r in range(3):                         # an uneven split: 3, 3, 2 heads
        sh = shard.shard_bh(BH, r, 3)
        sh.run(lambda q_, k_, v_, out, lse_out: pipe.step(q_, k_, v_, out, lse_out), q, k, v,
               out=o_sh, lse_out=l_sh)
    torch.cuda.synchronize()
    assert torch.equal(o_sh, o_all) and torch.equal(l_sh, l_all)
    # SplitPlan.run_shard gives the same rows
    for r in range(2):
        o_r, l_r = pipe.split.run_shard(q, k, v, r, 2)
        sh = shard.shard_bh(BH, r, 2)
        assert torch.equal(o_r, sh.slice(o_all)) and torch.equal(l_r, sh.slice(l_all))
