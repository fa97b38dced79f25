"""Nano-batch splitting and the AIMD controller that picks the nano-batch count.

Reference: ``split_ranges`` phase6_two_gpu_overlap.py:73-87 (identical to
``split_into_n`` phase4_aimd.py:22-36) and ``AIMDController``
phase6b_real_aimd.py:59-123 (CPU twin phase4_aimd.py:150-215, Eq. (2) of the
tLoRA paper): alpha = 4, beta = 0.5, a stability margin tau, N clamped to
[1, max_n], one bootstrap observation followed by an additive probe.
"""

from __future__ import annotations

import math
from typing import List, Tuple


def split_ranges(total: int, n: int) -> List[Tuple[int, int]]:
    """N near-equal contiguous [start, end) ranges over ``total`` rows; N is
    clamped to [1, total] and the first ``total % N`` ranges are one longer."""
    if total <= 0:
        return [(0, 0)]
    n = min(max(1, int(n)), total)
    q, r = divmod(total, n)
    out = []
    s = 0
    for i in range(n):
        e = s + q + (1 if i < r else 0)
        out.append((s, e))
        s = e
    return out


split_into_n = split_ranges


def ramp_ranges(total: int, n: int, first: float = 0.5) -> List[Tuple[int, int]]:
    """N contiguous ranges over ``total`` units whose first range is ``first``
    times the size of the others (each at least one unit): a short first
    nano-batch starts the all-reduce chain earlier.  N is clamped as in
    split_ranges; with N = 1 the whole range."""
    if total <= 0:
        return [(0, 0)]
    n = min(max(1, int(n)), total)
    if n == 1:
        return [(0, total)]
    head = max(1, min(total - (n - 1), int(round(total * first / (first + n - 1)))))
    return [(0, head)] + [(head + s, head + e) for s, e in split_ranges(total - head, n - 1)]


class AIMDController:
    """Additive-increase / multiplicative-decrease control of the nano-batch
    count N from measured iteration times.

    observe(T): the first call records T and probes N + alpha; afterwards
    N <- N + alpha when T <= T_prev - tau, else N <- max(1, floor(beta N)),
    clamped to [1, max_n].  ``best_n`` / ``best_ms`` track the fastest
    observation.  Times are in milliseconds (tau_ms likewise)."""

    def __init__(self, start_n: int = 1, alpha: int = 4, beta: float = 0.5, tau_ms: float = 0.05,
                 max_n: int = 64):
        self.n = max(1, int(start_n))
        self.alpha = int(alpha)
        self.beta = float(beta)
        self.tau_ms = float(tau_ms)
        self.max_n = max(1, int(max_n))
        self.prev_ms = None
        self.best_n = self.n
        self.best_ms = float("inf")
        self.history: List[Tuple[int, float, str, int]] = []

    def observe(self, current_ms: float) -> Tuple[int, str]:
        t = float(current_ms)
        used = self.n
        if t < self.best_ms:
            self.best_ms, self.best_n = t, used
        if self.prev_ms is None:
            self.prev_ms = t
            self.n = min(self.max_n, self.n + self.alpha)
            decision = "bootstrap additive probe"
        else:
            if t <= self.prev_ms - self.tau_ms:
                nxt, decision = self.n + self.alpha, "additive increase"
            else:
                nxt, decision = max(1, math.floor(self.beta * self.n)), "multiplicative decrease"
            self.prev_ms = t
            self.n = max(1, min(self.max_n, nxt))
        self.history.append((used, t, decision, self.n))
        return self.n, decision
