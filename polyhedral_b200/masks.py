"""Attention-mask predicates for the kernels, with the host-side views the
reference's mask objects expose (src/polyattn/masks.py:14-28): ``row_cols`` (live
columns of one query row), ``live_count`` (exact number of live (q, kv) pairs)
and ``dense``.

Every class here is a predicate on d = q - kv (plus the absolute kv index for
``SinksWindow``) and carries ``spec`` = (kind, p0, p1, p2), the form the CUDA
kernels evaluate (``include/polyattn.h``).  ``FarStrided`` is the one mask the
reference lacks: the lattice half (d >= w, d % s == 0) of the disjoint split of a
local+strided mask into its window and lattice parts.
"""
import numpy as np

CAUSAL, WINDOW, DILATED, LOCAL_STRIDED, TWOBAND, SINKS, FAR_STRIDED = range(7)


def _span(lo, hi, n):
    """Length of [lo, hi) intersected with [0, n), elementwise."""
    return np.maximum(0, np.minimum(hi, n) - np.maximum(lo, 0))


class Mask:
    spec = None
    name = "?"

    def row_cols(self, q, N):
        """bool[N]: live kv columns of query row q."""
        kv = np.arange(N, dtype=np.int64)
        return self._live(q - kv, kv)

    def dense(self, N):
        q = np.arange(N, dtype=np.int64)[:, None]
        kv = np.arange(N, dtype=np.int64)[None, :]
        return self._live(q - kv, kv)

    def live_count(self, N):
        raise NotImplementedError

    def _live(self, d, kv):
        raise NotImplementedError

    def __repr__(self):
        return f"{type(self).__name__}<{self.name}>"


class Causal(Mask):
    def __init__(self):
        self.name = "causal"
        self.spec = (CAUSAL, 0, 0, 0)

    def _live(self, d, kv):
        return d >= 0

    def live_count(self, N):
        return N * (N + 1) // 2


class SlidingWindow(Mask):
    def __init__(self, w):
        self.w = w
        self.name = f"window-{w}"
        self.spec = (WINDOW, w, 0, 0)

    def _live(self, d, kv):
        return (d >= 0) & (d < self.w)

    def live_count(self, N):
        q = np.arange(N, dtype=np.int64)
        return int(np.minimum(q + 1, self.w).sum())


class Dilated(Mask):
    def __init__(self, s):
        self.s = s
        self.name = f"dilated-{s}"
        self.spec = (DILATED, s, 0, 0)

    def _live(self, d, kv):
        return (d >= 0) & (d % self.s == 0)

    def live_count(self, N):
        q = np.arange(N, dtype=np.int64)
        return int((q // self.s + 1).sum())


class LocalStrided(Mask):
    def __init__(self, w, s):
        self.w, self.s = w, s
        self.name = f"local{w}+str{s}"
        self.spec = (LOCAL_STRIDED, w, s, 0)

    def _live(self, d, kv):
        return (d >= 0) & ((d < self.w) | (d % self.s == 0))

    def live_count(self, N):
        q = np.arange(N, dtype=np.int64)
        window = np.minimum(q + 1, self.w)
        # lattice offsets d = m*s with w <= d <= q
        first = -(-self.w // self.s)
        lattice = np.maximum(0, q // self.s - first + 1)
        return int((window + lattice).sum())


class FarStrided(Mask):
    """d >= w and d % s == 0: the lattice part of LocalStrided(w, s) with the
    window removed, so the two parts are disjoint and cover the union exactly."""

    def __init__(self, w, s):
        self.w, self.s = w, s
        self.name = f"far{w}+str{s}"
        self.spec = (FAR_STRIDED, w, s, 0)

    def _live(self, d, kv):
        return (d >= self.w) & (d >= 0) & (d % self.s == 0)

    def live_count(self, N):
        q = np.arange(N, dtype=np.int64)
        first = -(-max(self.w, 0) // self.s)
        return int(np.maximum(0, q // self.s - first + 1).sum())


class TwoBand(Mask):
    """Live on offsets [0, w1) and [off, off + w2)."""

    def __init__(self, w1, off, w2=None):
        self.w1, self.off, self.w2 = w1, off, w2 or w1
        self.name = f"twoband-{w1}+{off}"
        self.spec = (TWOBAND, w1, off, self.w2)

    def _live(self, d, kv):
        return (d >= 0) & ((d < self.w1) | ((d >= self.off) & (d < self.off + self.w2)))

    def live_count(self, N):
        n = np.arange(1, N + 1, dtype=np.int64)          # offsets 0 .. q available
        a = _span(0, self.w1, n)
        b = _span(self.off, self.off + self.w2, n)
        both = _span(max(0, self.off), min(self.w1, self.off + self.w2), n)
        return int((a + b - both).sum())


class SinksWindow(Mask):
    """g attention sinks (kv < g) plus a causal window of w."""

    def __init__(self, g, w):
        self.g, self.w = g, w
        self.name = f"sinks{g}+win{w}"
        self.spec = (SINKS, w, g, 0)

    def _live(self, d, kv):
        return (d >= 0) & ((d < self.w) | (kv < self.g))

    def live_count(self, N):
        q = np.arange(N, dtype=np.int64)
        sinks = np.minimum(q + 1, self.g)
        window = np.minimum(q + 1, self.w)
        both = np.maximum(0, np.minimum(self.g, q + 1) - np.maximum(0, q - self.w + 1))
        return int((sinks + window - both).sum())


def from_spec(kind, p0, p1, p2):
    """The mask object for a (kind, p0, p1, p2) spec."""
    if kind == CAUSAL:
        return Causal()
    if kind == WINDOW:
        return SlidingWindow(p0)
    if kind == DILATED:
        return Dilated(p0)
    if kind == LOCAL_STRIDED:
        return LocalStrided(p0, p1)
    if kind == TWOBAND:
        return TwoBand(p0, p1, p2)
    if kind == SINKS:
        return SinksWindow(p1, p0)
    if kind == FAR_STRIDED:
        return FarStrided(p0, p1)
    raise ValueError(f"unknown mask kind {kind}")
