"""Benchmark of the block-sparse attention forward path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c1|c2|c3|c3-rp8|c4|c5] [--bh B]

Metric: effective TFLOP/s over LIVE mask elements,
4 * D * live * B * H per forward, with ms per forward.  Default workload c5
(configs[4], the largest configuration and the one quoted at 1/2/4/8 GPUs): the
union of a causal window of 1024 and a stride-16 lattice, B2 H64 N32768 D128 bf16,
computed as a disjoint split -- the window in the identity basis (128x128 tiles),
then the lattice beyond it in its residue-16 basis (128x64 tiles), whose epilogue
merges its result into the window part's O / LSE -- on ~N(0,1) synthetic inputs.

One step = one pass of the hot path over one batch resident in HBM, inputs and
outputs in original row order (residue permutations are applied inside the kernel by
its tensor maps and epilogue, so no copy of Q, K, V is made).  The explicit
permutation kernel (``permute``), the standalone LSE merge (``merge``) and the block
index build (``block_index``) are timed on their own.  The block index and the
forward's work lists depend on the mask only; they are built once per mask (as the
reference builds its BlockIndex offline) and their time is reported separately
(``index_ms``).

Multi-GPU (torchrun, one process per GPU): the configuration's B*H (batch, head)
pairs are split into contiguous ranges, one per rank (``polyhedral_b200.shard``),
with no data-path collective: strong scaling, the whole job is one forward of the
configuration, and its step time is the max over ranks of the CUDA-event time.  The
optional all-gather of every rank's O / LSE is timed separately (``allgather``).
``--impl reference`` times the CPU restatement of the reference's dense masked
attention (gpu/reference.py) on the host cores instead.
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "block-sparse attn fwd live-element TFLOP/s & ms/fwd at 1/2/4/8 B200; % bf16 peak"
DEFAULT_WORKLOAD = "c5"

WORKLOADS = {
    # name: (B, H, N, D, mask spec name, residue stride, BQ, A, seed, description)
    "c1": (1, 4, 1024, 64, "window-128", 0, 128, 32, 0,
           "c1: window-128, B1 H4 N1024 D64 (fp32 inputs cast to bf16), 128x32 tiles"),
    "c2": (1, 16, 8192, 128, "dilated-4", 4, 128, 32, 1,
           "c2: dilated-4 + residue-perm-4, 128x32 tiles, B1 H16 N8192 D128 bf16"),
    "c3": (2, 16, 16384, 128, "local64+str8", 8, 128, 64, 2,
           "c3: local64+str8 as window-64 (identity, 128x64, 64-row KV super-tiles) + far64+str8 "
           "(residue-perm-8, 128x64) split, LSE merge fused into the second part's epilogue, "
           "B2 H16 N16384 D128 bf16"),
    "c3-rp8": (2, 16, 16384, 128, "local64+str8", 8, 128, 32, 2,
               "c3 in one basis: local64+str8 + residue-perm-8, 128x32 tiles, "
               "B2 H16 N16384 D128 bf16"),
    "c4": (4, 32, 8192, 128, "sinks4+win512", 0, 128, 32, 3,
           "c4: sinks4+win512, 128x32 tiles, B4 H32 N8192 D128 bf16"),
    "c5": (2, 64, 32768, 128, "local1024+str16", 16, 128, 64, 4,
           "c5: window-1024 (identity, 128x128) + far1024+str16 (residue-perm-16, 128x64) "
           "split, LSE merge fused into the second part's epilogue, B2 H64 N32768 D128 bf16"),
}
# Attention kernel options per workload (``kv_rows``: KV rows per super-tile, 64 =
# S double-buffered; ``row_threads``: softmax threads per query row), chosen by
# interleaved measurement; the default kernel elsewhere.
KERNEL_OPTS = {"c2": {"row_threads": 2}, "c3-rp8": {"row_threads": 2},
               "c4": {"row_threads": 2}}
# Workloads computed as a disjoint split, part by part: (mask spec name, BQ, A,
# residue stride, KV rows per super-tile).  The first part writes O / LSE, the
# second merges into them in its epilogue.  Band + lattice unions split into the
# band in the identity basis and the lattice beyond it in its residue basis, where
# each is dense; in one residue basis the band is spread over every off-diagonal
# block (c3: 2x the tiles).
SPLITS = {
    "c3": [("window-64", 128, 64, 0, {"kv_rows": 64}), ("far64+str8", 128, 64, 8, {})],
    "c5": [("window-1024", 128, 128, 0, {}), ("far1024+str16", 128, 64, 16, {})],
}


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["bf16_tflops"], d.get("bf16_tflops_sustained"), d["hbm_gbs"], "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def _traffic_from_profiles(workload, part=None):
    """DRAM bytes per launch of the attention kernel (of one part of a split) on the
    full configuration, from the committed ncu summary."""
    p = ROOT / "profiles" / f"attn_fwd_{workload}.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
        except Exception:
            return None
        if part is not None:
            return (d.get("parts") or {}).get(part)
        return d.get("dram_bytes_per_launch")
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index, enabled=True):
        self.gpu = gpu_index
        self.enabled = enabled
        self.proc = None
        self.lines = []

    def __enter__(self):
        if not self.enabled:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln.strip() for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, val in zip(names, f[5:9]):
                if val.lower() in ("active", "1"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def max_over_ranks(x, device=None):
    """Max of a float over all ranks of the default process group (identity when
    there is none); CUDA tensor under NCCL, CPU tensor under gloo."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    dev = device if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([float(x)], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_tflops(flops_per_job, ms_per_step):
    """Whole-job throughput: the job's work per step over its step time (the slowest
    rank's)."""
    return flops_per_job / (ms_per_step * 1e-3) / 1e12


def config_of(wl, world):
    """The `config` object of the JSON line, the same for both arms."""
    B, H, N, D, name, s, BQ, A, seed, desc = WORKLOADS[wl]
    _, live = live_flops(B, H, N, D, name)
    return {"workload": desc, "global_batch": B * H, "seq_len": N, "head_dim": D,
            "parallelism": f"(batch, head) sharded over {world} GPU(s), contiguous ranges of "
                           f"{-(-B * H // world)} or fewer (b,h) per GPU, no data-path collective",
            "live_elements_per_head": live,
            "live_gflop_per_step": round(4.0 * D * live * B * H / 1e9, 3),
            "seed": seed,
            "l2": "inputs rotated over buffer sets of >= 2x L2 between steps (not flushed)"}


def live_flops(B, H, N, D, name):
    from polyhedral_b200 import masks_gpu
    live = masks_gpu.numpy_mask(name).live_count(N)
    return 4.0 * D * live * B * H, live


class Pipeline:
    """Mask-only preprocessing plus the per-batch step of one workload."""

    def __init__(self, wl, device, opts=None):
        import torch
        from polyhedral_b200 import attention, blockindex, masks_gpu, permute, split
        B, H, N, D, name, s, BQ, A, seed, _ = WORKLOADS[wl]
        self.opts = dict(KERNEL_OPTS.get(wl, {}) if opts is None else opts)
        self.wl, self.B, self.H, self.N, self.D = wl, B, H, N, D
        self.name, self.s, self.BQ, self.A = name, s, BQ, A
        self.device = device
        self.spec = masks_gpu.triton_params(name)
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        if wl in SPLITS:
            self.split_names = [pn for pn, *_ in SPLITS[wl]]
            parts = []
            for i, (pn, pbq, pa, ps, popts) in enumerate(SPLITS[wl]):
                o = dict(opts) if (i == 0 and opts is not None) else dict(popts)
                parts.append(split.SplitPart(masks_gpu.numpy_mask(pn), pbq, pa, ps,
                                             o.get("kv_rows", 0), o.get("row_threads", 0)))
            self.split = split.SplitPlan(parts, N, device)
            self.perm = None
            self.plan = None
        else:
            self.split = None
            self.perm = permute.residue_perm_device(N, s, device) if s else None
            dbi = blockindex.build_device(masks_gpu.numpy_mask(name), N, BQ, A,
                                          perm_q=self.perm, perm_kv=self.perm, device=device)
            self.plan = attention.make_plan(dbi.kv_idx, dbi.kv_num, dbi.kv_partial, N, BQ, A,
                                            residue_stride=s)
            self.dbi = dbi
        torch.cuda.synchronize(device)
        self.index_ms = (time.perf_counter() - t0) * 1e3

    def kernel_desc(self):
        """Attention kernel options of the step (per part for a split)."""
        if self.split is not None:
            return [{"part": n, "kv_rows": p.kv_rows or 128, "row_threads": p.row_threads or 1}
                    for n, p in zip(self.split_names, self.split.parts)]
        return {"kv_rows": self.opts.get("kv_rows") or 128,
                "row_threads": self.opts.get("row_threads") or 1}

    def plans(self):
        """The work lists the step runs on (their device status is checked)."""
        return list(self.split.plans) if self.split is not None else [self.plan]

    def launches_per_step(self):
        if self.split is not None:
            return 2                 # attention (window), attention (lattice, merging)
        return 1

    def step(self, q, k, v, o=None, lse=None):
        from polyhedral_b200 import attention
        if self.split is not None:
            return self.split.run(q, k, v, out=o, lse_out=lse)
        return attention.block_sparse_attention(
            q, k, v, None, None, None, *self.spec, self.BQ, self.A, residue_stride=self.s,
            plan=self.plan, return_lse=True, out=o, lse_out=lse, **self.opts)


def make_inputs(wl, device, sh, buf=0):
    """q, k, v of the (b,h) range of shard `sh`, buffer set `buf`: ~N(0,1) bf16, each
    head drawn from its own seeded generator, so the union over ranks is the same
    tensors whatever the number of ranks."""
    import torch
    B, H, N, D, _, _, _, _, seed, _ = WORKLOADS[wl]
    out = [torch.empty(sh.size, N, D, device=device, dtype=torch.bfloat16) for _ in range(3)]
    g = torch.Generator(device=device)
    for i, bh in enumerate(range(sh.start, sh.stop)):
        for t, x in enumerate(out):
            g.manual_seed(((seed * 1009 + buf) * 65537 + bh) * 3 + t)
            x[i].copy_(torch.randn(N, D, device=device, generator=g))
    return out


def run_ours(args, rank, world, device):
    import torch
    import torch.distributed as dist
    from polyhedral_b200 import shard as shard_mod
    wl = args.workload
    B, H, N, D, name, s, BQ, A, seed, desc = WORKLOADS[wl]
    BH = args.bh or B * H                   # --bh: a smaller case of the workload (profiling)
    flops_cfg, live = live_flops(B, H, N, D, name)
    flops_job = flops_cfg * BH / (B * H)
    sh = shard_mod.shard_bh(BH, rank, world)
    flops_rank = flops_cfg * sh.size / (B * H)
    pipe = Pipeline(wl, device, json.loads(args.kernel_opts) if args.kernel_opts else None)

    # inputs rotate over enough buffer sets that each step reads data not in L2
    props = torch.cuda.get_device_properties(device)
    l2 = getattr(props, "L2_cache_size", 0) or (126 << 20)
    step_bytes = 4 * sh.size * N * D * 2
    nbuf = max(2, -(-2 * l2 // step_bytes) + 1)
    bufs = [make_inputs(wl, device, sh, i) for i in range(nbuf)]
    outs = [(torch.empty(sh.size, N, D, device=device, dtype=torch.bfloat16),
             torch.empty(sh.size, N, device=device, dtype=torch.float32)) for _ in range(nbuf)]

    def do_step(i):
        q, k, v = bufs[i % nbuf]
        o, lse = outs[i % nbuf]
        return pipe.step(q, k, v, o, lse)

    for i in range(args.warmup):
        do_step(i)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    for plan in pipe.plans():
        st = plan.status()
        if st:
            raise RuntimeError(f"attention kernel reported device status {st} during warm-up")

    with ClockSampler(device.index if device.index is not None else 0,
                      enabled=not args.profile) as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for i in range(args.steps):
            do_step(i)
        ev1.record()
        torch.cuda.synchronize(device)
        t_ms = ev0.elapsed_time(ev1)
        # keep the same load running (untimed) so the sampler sees >= 1 s of it
        extra = 0 if args.profile else int(max(0.0, 1000.0 - t_ms) / max(t_ms / args.steps, 1e-3))
        for i in range(extra):
            do_step(i)
        torch.cuda.synchronize(device)
    t_ms = max_over_ranks(t_ms, device)
    if world > 1:
        dist.barrier()
    ms_per_step = t_ms / args.steps
    value = job_tflops(flops_job, ms_per_step)
    for plan in pipe.plans():
        st = plan.status()
        if st:
            raise RuntimeError(f"attention kernel reported device status {st} in the timed steps")

    # optional: every rank's O / LSE gathered onto every rank (NCCL all-gather over
    # NVLink), outside the step; every rank takes part
    ag_line = None
    if world > 1:
        o0, l0 = outs[0]
        for _ in range(2):
            shard_mod.gather(o0, l0, sh)
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        agreps = 5
        e0.record()
        for _ in range(agreps):
            shard_mod.gather(o0, l0, sh)
        e1.record()
        torch.cuda.synchronize(device)
        ag_ms = max_over_ranks(e0.elapsed_time(e1) / agreps, device)
        ag_bytes = BH * N * (D * 2 + 4)
        ag_line = {"collective": "all_gather_into_tensor of O and LSE (NCCL)", "ms": round(ag_ms, 4),
                   "bytes_gathered_per_rank": ag_bytes,
                   "bus_gbs": round(ag_bytes * (world - 1) / world / (ag_ms * 1e-3) / 1e9, 1),
                   "note": "optional, not part of the step"}

    # dominant kernel alone, CUDA events on the launching stream (for a split: each
    # part's launch alone, the one taking the most time reported, every part listed)
    kernel_flops, kernel_name, kernel_part = flops_rank, "attn_fwd_kernel", None
    reps = max(min(args.steps, 200), 20)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def time_alone(run):
        for i in range(3):
            run(i)
        e0.record()
        for i in range(reps):
            run(i)
        e1.record()
        torch.cuda.synchronize(device)
        return e0.elapsed_time(e1) / reps

    parts_line = None
    if pipe.split is not None:
        from polyhedral_b200 import masks_gpu
        part_flops = [4.0 * D * masks_gpu.numpy_mask(pn).live_count(N) * sh.size
                      for pn in pipe.split_names]
        part_ms = [time_alone(lambda i, k=k: pipe.split.run_part(k, *bufs[i % nbuf],
                                                                  *outs[i % nbuf]))
                   for k in range(len(part_flops))]
        dom = max(range(len(part_ms)), key=lambda i: part_ms[i])
        kernel_flops, kernel_ms, kernel_part = part_flops[dom], part_ms[dom], pipe.split_names[dom]
        kernel_name = f"attn_fwd_kernel ({kernel_part} part, merging)" if dom else \
            f"attn_fwd_kernel ({kernel_part} part)"
        peak0 = _peaks()[0]
        parts_line = [{"part": pn, "ms": round(ms, 5), "live_gflop": round(f / 1e9, 3),
                       "tflops": round(f / (ms * 1e-3) / 1e12, 2),
                       "frac": round(f / (ms * 1e-3) / 1e12 / peak0, 4),
                       "merging": k > 0}
                      for k, (pn, f, ms) in enumerate(zip(pipe.split_names, part_flops, part_ms))]
    else:
        kernel_ms = time_alone(lambda i: pipe.step(*bufs[i % nbuf], *outs[i % nbuf]))

    _, _, hbm_peak, hbm_kind = _peaks()
    # the explicit class A gather (Q, K, V in one launch), HBM-bound
    perm_line = None
    if s:
        from polyhedral_b200 import permute
        pv = permute.residue_perm_device(N, s, device)
        pouts = [permute.apply_perm_many(bufs[i], pv) for i in range(nbuf)]
        e0.record()
        for i in range(reps):
            permute._permute(list(bufs[i % nbuf]), pv, scatter=False, outs=pouts[i % nbuf])
        e1.record()
        torch.cuda.synchronize(device)
        pms = e0.elapsed_time(e1) / reps
        pbytes = 2 * 3 * sh.size * N * D * 2
        perm_line = {"kernel": "permute_rows_kernel (Q, K, V gather)", "ms": round(pms, 5),
                     "bytes": pbytes, "gbs": round(pbytes / (pms * 1e-3) / 1e9, 1),
                     "frac_of_hbm": round(pbytes / (pms * 1e-3) / 1e9 / hbm_peak, 4),
                     "peak_source": f"{hbm_kind} HBM copy"}
        del pouts

    # the block index (pa_block_index on the device, once per mask): integer work,
    # one classification per BQ x A tile; CUDA events over repeated builds
    from polyhedral_b200 import blockindex, masks_gpu
    bparts = ([(pn, pbq, pa, ps) for pn, pbq, pa, ps, _ in SPLITS[wl]] if pipe.split is not None
              else [(pipe.name, pipe.BQ, pipe.A, s)])
    bi_line = []
    for pn, pbq, pa, ps in bparts:
        bmask = masks_gpu.numpy_mask(pn)
        perm = pipe.perm if pipe.split is None else (
            pipe.split.perms[[x[0] for x in bparts].index(pn)])
        build = lambda: blockindex.build_device(bmask, N, pbq, pa, perm_q=perm, perm_kv=perm,
                                                device=device)
        for _ in range(3):
            build()
        e0.record()
        breps = 20
        for _ in range(breps):
            build()
        e1.record()
        torch.cuda.synchronize(device)
        bus = e0.elapsed_time(e1) / breps * 1e3
        tiles = (N // pbq) * (N // pa)
        bi_line.append({"kernel": "block_index_kernel (pa_block_index)", "mask": pn,
                        "basis": f"residue-{ps}" if ps else "identity", "tile": f"{pbq}x{pa}",
                        "us": round(bus, 2), "tiles": tiles,
                        "tiles_per_s": round(tiles / (bus * 1e-6), 1),
                        "note": "per build incl. output allocation; bit-exact vs the reference"})

    # the standalone LSE merge (pa_lse_merge), HBM-bound; a split step itself merges
    # in the attention epilogue instead
    merge_line = None
    if pipe.split is not None:
        from polyhedral_b200 import merge as merge_mod
        o1, l1 = outs[0]
        o2, l2_ = outs[1]
        for i in range(2):
            merge_mod.lse_merge(o1, l1, o2, l2_, out=o1, lse_out=l1)
        e0.record()
        mreps = max(3, min(reps, 20))
        for i in range(mreps):
            merge_mod.lse_merge(o1, l1, o2, l2_, out=o1, lse_out=l1)
        e1.record()
        torch.cuda.synchronize(device)
        mms = e0.elapsed_time(e1) / mreps
        mbytes = 3 * (sh.size * N * D * 2 + sh.size * N * 4)
        merge_line = {"kernel": "lse_merge_kernel (standalone pa_lse_merge)", "ms": round(mms, 5),
                      "bytes": mbytes, "gbs": round(mbytes / (mms * 1e-3) / 1e9, 1),
                      "frac_of_hbm": round(mbytes / (mms * 1e-3) / 1e9 / hbm_peak, 4),
                      "peak_source": f"{hbm_kind} HBM copy"}

    # End to end through the public API with host buffers.  Every step copies its
    # Q, K, V (this rank's heads) from pinned host memory and reads its O and LSE
    # back; the steps are pipelined over three streams (H2D of one step, compute of
    # the next older, D2H of the one before) with double-buffered device and host
    # tensors, as a serving loop would run them.
    e2e = None
    if not args.profile:
        hq = [x.cpu().pin_memory() for x in bufs[0]]
        ho = [torch.empty(sh.size, N, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        hl = [torch.empty(sh.size, N, dtype=torch.float32).pin_memory() for _ in range(2)]
        din = [[torch.empty_like(x, device=device) for x in bufs[0]] for _ in range(2)]
        dout = [(torch.empty(sh.size, N, D, device=device, dtype=torch.bfloat16),
                 torch.empty(sh.size, N, device=device, dtype=torch.float32)) for _ in range(2)]
        s_in, s_comp, s_out = (torch.cuda.Stream(device) for _ in range(3))
        ev = lambda: torch.cuda.Event()
        in_ready, comp_done, out_done = ([ev(), ev()] for _ in range(3))
        for x in comp_done + out_done:
            x.record(torch.cuda.current_stream(device))

        def e2e_step(i):
            b = i % 2
            with torch.cuda.stream(s_in):
                s_in.wait_event(comp_done[b])            # step i-2 has read din[b]
                for d_, h_ in zip(din[b], hq):
                    d_.copy_(h_, non_blocking=True)
                in_ready[b].record(s_in)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(in_ready[b])
                s_comp.wait_event(out_done[b])           # step i-2's O has left dout[b]
                pipe.step(*din[b], *dout[b])
                comp_done[b].record(s_comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(comp_done[b])
                ho[b].copy_(dout[b][0], non_blocking=True)
                hl[b].copy_(dout[b][1], non_blocking=True)
                out_done[b].record(s_out)

        e2e_steps = max(6, min(args.steps, 30))
        for i in range(4):
            e2e_step(i)
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s_in)
        for i in range(e2e_steps):
            e2e_step(i)
        e1.record(s_out)
        torch.cuda.synchronize(device)
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, device)
        e2e = {"value": round(job_tflops(flops_job, e2e_ms), 3), "unit": "TFLOP/s",
               "ms_per_step": round(e2e_ms, 4),
               "h2d_bytes_per_step": 3 * BH * N * D * 2,
               "d2h_bytes_per_step": BH * N * D * 2 + BH * N * 4,
               "bytes_note": "whole job; each rank copies its own heads' share",
               "pipelined": "H2D / compute / D2H of consecutive steps on three streams"}
        del hq, ho, hl, din, dout

    peak, peak_sus, hbm, peak_kind = _peaks()
    ach = kernel_flops / (kernel_ms * 1e-3) / 1e12
    traffic = _traffic_from_profiles(wl, kernel_part)
    if traffic is not None and args.bh:
        traffic = None          # the committed figure is for the full configuration
    elif traffic is not None:
        traffic = int(traffic * sh.size / BH)   # this rank's share of the (b,h)
    roof = {"bound": "tensor", "achieved": round(ach, 2), "peak": peak, "unit": "TFLOP/s",
            "frac": round(ach / peak, 4), "traffic": traffic,
            "kernel": kernel_name, "kernel_ms": round(kernel_ms, 5), "parts": parts_line,
            "kernel_live_gflop": round(kernel_flops / 1e9, 3),
            "peak_source": f"{peak_kind} bf16 dense (burst), of measured"
                           if peak_kind == "measured" else "fallback bf16 dense"}

    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu or args.profile):
        cpu = cpu_baseline(wl, budget_s=args.cpu_budget)

    if rank == 0:
        cfg = config_of(wl, world)
        if args.bh:
            cfg["global_batch"] = BH
            cfg["note"] = f"reduced case: first {BH} (b,h) of the configuration"
        line = {
            "metric": METRIC,
            "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic ~N(0,1), seeded per (b,h)",
            "config": cfg,
            "run": {"index_ms": round(pipe.index_ms, 3), "kernel": pipe.kernel_desc(),
                    "heads_per_rank": [shard_mod.shard_bh(BH, r, world).size for r in range(world)],
                    "buffer_sets": nbuf, "buffer_set_mib": step_bytes >> 20,
                    "step": "attention (O, LSE) over the residue permutation applied on the fly, "
                            "inputs/outputs in original order" if pipe.split is None else
                            f"window part + lattice part (residue-{s} on the fly) merging into "
                            "the window part's O / LSE in its epilogue"},
            "pct_bf16_peak": round(value / world / peak, 4),
            "gpu_launches": pipe.launches_per_step() * args.steps,
            "clocks": clk.summary(),
            "e2e": e2e,
            "roofline": roof,
            "allgather": ag_line,
            "permute": perm_line,
            "merge": merge_line,
            "block_index": bi_line,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)


def _cpu_rows(wl, rows_idx, g):
    """Oracle attention (CPU restatement of gpu/reference.py) for the query rows
    `rows_idx` of one head against all N keys, with the mask rows built for those
    rows only; returns (live elements, seconds of the attention itself)."""
    import torch
    import oracle as O
    from polyhedral_b200 import masks_gpu
    B, H, N, D, name, *_ = WORKLOADS[wl]
    q = torch.randn(1, len(rows_idx), D, generator=g)
    k, v = (torch.randn(1, N, D, generator=g) for _ in range(2))
    Mr = torch.from_numpy(O.dense_mask(*masks_gpu.triton_params(name), N, rows=rows_idx))
    t0 = time.perf_counter()
    O.attention(q, k, v, Mr)
    return int(Mr.sum()), time.perf_counter() - t0


def cpu_baseline(wl, budget_s=12.0, threads=None, rows=1024, start=0, pieces=None):
    """The oracle on the host cores, `rows` query rows per piece spread evenly over
    the sequence (so the live fraction is the workload's), until ~budget_s seconds of
    compute (or `pieces` pieces); TFLOP/s over the live elements done."""
    import numpy as np
    import torch
    B, H, N, D, name, _, _, _, seed, _ = WORKLOADS[wl]
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed + start)
    rows = min(rows, N)
    stride = N // rows
    live, dt, done = 0, 0.0, 0
    while True:
        idx = np.arange(rows) * stride + ((start + done) % stride)
        lv, t = _cpu_rows(wl, idx, g)
        live += lv
        dt += t
        done += 1
        if (pieces is not None and done >= pieces) or (pieces is None and dt >= budget_s) \
                or done >= stride * B * H:
            break
    val = 4.0 * D * live / dt / 1e12
    return {"value": round(val, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{done} x {rows} query rows (evenly spaced) x {N} keys of {wl}, fp32 "
                      f"dense masked attention (gpu/reference.py semantics), {dt:.2f} s",
            "live_elements": live, "seconds": round(dt, 3)}


def run_reference(args, rank, world):
    """The reference arm: the reference's own algorithm for the path, dense fp32 masked
    attention (gpu/reference.py, restated in oracle/), on the host cores.  Every step
    is one bounded sample of the workload (256 evenly spaced query rows of one head
    against all N keys), so ms_per_step is the time actually spent per step; the time
    of a whole forward at that rate is reported separately."""
    if rank != 0:
        return
    wl = args.workload
    B, H, N, D, name, *_ = WORKLOADS[wl]
    flops, live = live_flops(B, H, N, D, name)
    for i in range(args.warmup):
        cpu_baseline(wl, rows=256, start=i, pieces=1)
    tot_live, tot_s = 0, 0.0
    t0 = time.perf_counter()
    for i in range(args.steps):
        cb = cpu_baseline(wl, rows=256, start=args.warmup + i, pieces=1)
        tot_live += cb["live_elements"]
        tot_s += cb["seconds"]
    wall = time.perf_counter() - t0
    val = 4.0 * D * tot_live / tot_s / 1e12
    sample = (f"each step: 256 evenly spaced query rows x {N} keys of one head, dense fp32 "
              "masked attention (gpu/reference.py semantics)")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(val, 6), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(wall / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic ~N(0,1), seeded",
        "config": config_of(wl, world),
        "ms_per_forward_extrapolated": round(flops / (val * 1e12) * 1e3, 3),
        "cpu_baseline": {"value": round(val, 6), "unit": "TFLOP/s", "cores": os.cpu_count(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(val, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--bh", type=int, default=None,
                    help="run only the first BH (batch, head) pairs of the workload "
                         "(a smaller case for profiling)")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--kernel-opts", default=None,
                    help='attention kernel options replacing the workload\'s defaults '
                         '(the first part\'s, for a split), e.g. \'{"row_threads": 2}\'')
    ap.add_argument("--profile", action="store_true",
                    help="short run for ncu: no clock fill, no end-to-end leg, no CPU leg")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", device_id=device,
                                timeout=datetime.timedelta(seconds=120))
    try:
        run_ours(args, rank, world, device)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
