"""Device timing for the reference's driver scripts, under the names they import
from their ``bench`` module (gpu/bench.py): ``time_ms``, ``paired_time``, ``report``.

Design: one ``_Timer`` owns an L2-sized scrub buffer and times single calls with a
pair of CUDA events on the current stream, synchronising after each call, so every
sample is one cold-L2 call.  ``time_ms`` summarises many samples of one callable;
``paired_time`` interleaves two callables, alternating which of the pair runs first
so neither always follows the other's cache state, and summarises the per-pair
ratios.  ``report`` prints a right-aligned fixed-width table.  The scrub buffer is
twice the device's L2 (126 MB on B200), not a fixed size.
"""
import statistics


class _Timer:
    """Times one call of a callable on the current CUDA stream."""

    def __init__(self, scrub_l2=True):
        import torch
        self._torch = torch
        self._scrub = None
        if scrub_l2:
            props = torch.cuda.get_device_properties(torch.cuda.current_device())
            l2 = getattr(props, "L2_cache_size", 0) or (128 << 20)
            self._scrub = torch.empty(2 * l2, dtype=torch.uint8, device="cuda")
        self._ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        self._tick = 0

    def __call__(self, fn):
        if self._scrub is not None:       # evict the previous call's data from L2
            self._tick = (self._tick + 1) & 0xFF
            self._scrub.fill_(self._tick)
        start, stop = self._ev
        start.record()
        fn()
        stop.record()
        stop.synchronize()
        return start.elapsed_time(stop)


def _spread(xs):
    return statistics.stdev(xs) if len(xs) > 1 else 0.0


def time_ms(fn, warmup=25, reps=100, flush_l2=True):
    """(median, standard deviation) in ms of ``reps`` single calls of ``fn`` after
    ``warmup`` untimed ones, L2 scrubbed before each timed call."""
    timer = _Timer(flush_l2)
    for _ in range(warmup):
        fn()
    samples = sorted(timer(fn) for _ in range(reps))
    return statistics.median(samples), _spread(samples)


def paired_time(fn_a, fn_b, warmup=25, reps=200, flush_l2=True):
    """Interleaved A/B timing: (median ms of a, median ms of b, median of the
    per-pair ratios b / a, their standard deviation).  Each pair runs both calls
    back to back, a first in even pairs and b first in odd ones."""
    timer = _Timer(flush_l2)
    for _ in range(warmup):
        fn_a()
        fn_b()
    ta, tb = [], []
    for i in range(reps):
        if i % 2 == 0:
            a = timer(fn_a)
            b = timer(fn_b)
        else:
            b = timer(fn_b)
            a = timer(fn_a)
        ta.append(a)
        tb.append(b)
    ratios = [b / a for a, b in zip(ta, tb) if a > 0]
    return statistics.median(ta), statistics.median(tb), statistics.median(ratios), _spread(ratios)


def _cell(value, width):
    """One right-aligned table cell: floats with three decimals, integers whole."""
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        return format(str(value), f">{width}")
    if isinstance(value, int):
        return format(value, f">{width}d")
    return format(value, f">{width}.3f")


def report(rows, cols, title=None, note=None):
    """Print `rows` as a table whose columns are ``cols = [(header, width), ...]``,
    under an optional title and its rule, followed by an optional note."""
    widths = [w for _, w in cols]
    lines = []
    if title:
        lines += ["", title, "-" * max(len(title), sum(widths))]
    lines.append("".join(_cell(h, w) for h, w in cols))
    lines += ["".join(_cell(v, w) for v, w in zip(r, widths)) for r in rows]
    if note:
        lines += ["", note]
    print("\n".join(lines))
