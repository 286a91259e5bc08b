"""CUDA-event timing with an L2 flush between repetitions (the methodology of
the reference's ``gpu/bench.py``, :11-74: medians, warm-up, flushed cache, and
interleaved A/B pairs for comparisons).  The flush buffer is sized from the
device's L2 (twice its size) rather than a fixed 64 MB."""
import statistics


def _flush_buffer(device=None):
    import torch
    props = torch.cuda.get_device_properties(device)
    l2 = getattr(props, "L2_cache_size", 0) or (128 << 20)
    return torch.empty(2 * l2 // 4, dtype=torch.int32, device=device)


def time_ms(fn, warmup=25, reps=100, flush_l2=True):
    """Median and stdev (ms) of ``fn()`` over ``reps`` CUDA-event-timed calls on
    the current stream."""
    import torch
    cache = _flush_buffer() if flush_l2 else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(reps):
        if cache is not None:
            cache.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e))
    return statistics.median(out), (statistics.stdev(out) if len(out) > 1 else 0.0)


def paired_time(fn_a, fn_b, warmup=25, reps=200, flush_l2=True):
    """Interleaved timing of two callables; returns (median_a, median_b,
    median of per-pair b/a ratios, stdev of the ratios)."""
    import torch
    cache = _flush_buffer() if flush_l2 else None
    for _ in range(warmup):
        fn_a()
        fn_b()
    torch.cuda.synchronize()
    a_s, b_s, ratios = [], [], []
    for _ in range(reps):
        pair = []
        for fn in (fn_a, fn_b):
            if cache is not None:
                cache.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            pair.append(s.elapsed_time(e))
        a_s.append(pair[0])
        b_s.append(pair[1])
        if pair[0] > 0:
            ratios.append(pair[1] / pair[0])
    return (statistics.median(a_s), statistics.median(b_s), statistics.median(ratios),
            statistics.stdev(ratios) if len(ratios) > 1 else 0.0)


def report(rows, cols, title=None, note=None):
    """Fixed-width table (gpu/bench.py:27-38)."""
    if title:
        print(f"\n{title}")
        print("-" * max(len(title), sum(w for _, w in cols)))
    print("".join(f"{h:>{w}}" for h, w in cols))
    for r in rows:
        print("".join(
            (f"{v:>{w}.{3 if isinstance(v, float) else 0}f}" if isinstance(v, (int, float))
             else f"{str(v):>{w}}")
            for v, (_, w) in zip(r, cols)))
    if note:
        print(f"\n{note}")
