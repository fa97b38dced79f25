"""CPU oracle for the heterogeneous multi-LoRA linear (numpy restatement).

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this module:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` use it, and only as the checker or
as the timed CPU baseline.

It restates, in plain numpy, the reference algorithm of
GOPIKA-SUSHAMA/mini-tlora-reproduction for the one hot path this repository
accelerates:

* ``LoRAAdapter.forward``          tlora/multi_lora_linear.py:28-31
* ``MultiLoRALinear.forward``      tlora/multi_lora_linear.py:92-118
* autograd of that forward (dX incl. the frozen backbone term, dA, dB; no dW,
  the backbone is frozen at tlora/multi_lora_linear.py:78-80), written out as
  the analytic formulas of phase5d_triton_training.py:287-312
* one isolated SGD step            phase5d_triton_training.py:554-559
                                   (torch.optim.SGD, phase3_nano_batch.py:90-97)
* ``split_ranges``/``split_into_n`` phase6_two_gpu_overlap.py:73-87,
                                   phase4_aimd.py:22-36
* ``nano_forward_by_count``        phase4_aimd.py:39-80
* ``AIMDController``               phase6b_real_aimd.py:59-123
                                   (CPU twin phase4_aimd.py:150-215)
* ``synthetic_iteration_time``     phase4_aimd.py:218-230

Parity is pinned: ``tests/test_oracle_golden.py`` checks this module against
golden vectors produced by running the reference's own ``tlora`` package
(``tests/golden/make_golden.py``) and against the AIMD known-answer trace
captured in the reference's ``results/phase4_aimd.txt:26-38``.

Arrays use the reference's layouts: x ``[rows, in]``, W ``[out, in]``,
bias ``[out]``, A ``[rank, in]``, B ``[out, rank]``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np


@dataclass
class OracleAdapter:
    """One LoRA branch (tlora/multi_lora_linear.py:9-31)."""

    A: np.ndarray  # [rank, in]
    B: np.ndarray  # [out, rank]
    scaling: float  # alpha / rank (multi_lora_linear.py:19)

    @property
    def rank(self) -> int:
        return int(self.A.shape[0])


def adapter_delta(x: np.ndarray, ad: OracleAdapter) -> np.ndarray:
    """delta(x) = scaling * (x @ A^T) @ B^T  (multi_lora_linear.py:28-31)."""
    hidden = x @ ad.A.T
    return (hidden @ ad.B.T) * ad.scaling


def _check_inputs(x: np.ndarray, ids: np.ndarray) -> None:
    # multi_lora_linear.py:100-103
    if x.ndim != 2:
        raise ValueError("Phase 1 expects x shaped [batch, in_features]")
    if ids.ndim != 1 or ids.shape[0] != x.shape[0]:
        raise ValueError("adapter_ids must be [batch] and match x.shape[0]")


def multi_lora_forward(
    x: np.ndarray,
    ids: np.ndarray,
    W: np.ndarray,
    bias: Optional[np.ndarray],
    adapters: Dict[int, OracleAdapter],
) -> np.ndarray:
    """Y = X W^T (+b), then Y[mask_s] += delta_s(X[mask_s]) per adapter.

    Follows multi_lora_linear.py:105-118: the backbone runs once over all
    rows, then a boolean-mask loop over the adapters in insertion order adds
    each adapter's delta to the rows routed to it.  Rows whose id names no
    adapter receive only the backbone output.
    """
    _check_inputs(x, ids)
    out = x @ W.T
    if bias is not None:
        out = out + bias
    result = out.copy()
    for aid, ad in adapters.items():
        mask = ids == aid
        if mask.any():
            result[mask] = result[mask] + adapter_delta(x[mask], ad)
    return result


def multi_lora_backward(
    x: np.ndarray,
    ids: np.ndarray,
    W: np.ndarray,
    adapters: Dict[int, OracleAdapter],
    dY: np.ndarray,
) -> Tuple[np.ndarray, Dict[int, Optional[np.ndarray]], Dict[int, Optional[np.ndarray]]]:
    """Analytic gradients of ``multi_lora_forward`` for upstream grad dY.

    dX = dY W + sum_s scatter_s(dz_s A_s)   (the backbone term is what autograd
    of ``self.base(x)`` at multi_lora_linear.py:106 contributes; W and b are
    frozen so there is no dW, :78-80).  Per adapter, on its masked rows
    (phase5d_triton_training.py:287-312):
        z  = x A^T
        dB = s * g^T z
        dz = s * g B
        dA = dz^T x
        dx = dz A
    Adapters that receive no rows get ``None`` gradients, as autograd leaves
    their ``.grad`` unset (the mask loop never calls them, :115).
    """
    _check_inputs(x, ids)
    dX = dY @ W
    dA: Dict[int, Optional[np.ndarray]] = {}
    dB: Dict[int, Optional[np.ndarray]] = {}
    for aid, ad in adapters.items():
        mask = ids == aid
        if not mask.any():
            dA[aid] = None
            dB[aid] = None
            continue
        xs = x[mask]
        g = dY[mask]
        z = xs @ ad.A.T
        dB[aid] = ad.scaling * (g.T @ z)
        dz = ad.scaling * (g @ ad.B)
        dA[aid] = dz.T @ xs
        dX[mask] = dX[mask] + dz @ ad.A
    return dX, dA, dB


def grad_projections(
    x: np.ndarray,
    ids: np.ndarray,
    adapters: Dict[int, OracleAdapter],
    dY: np.ndarray,
    probes: Dict[int, Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]],
) -> Dict[int, Tuple[np.ndarray, np.ndarray]]:
    """Bilinear probes of the adapter gradients of ``multi_lora_backward``
    without forming them, for checks at sizes where the full gradients are too
    costly on a CPU: for adapter a and probe vectors (uA [k, r], vA [k, d_in],
    uB [k, d_out], vB [k, r]) returns (uA_i^T dA vA_i, uB_i^T dB vB_i) for
    i < k.  With the per-adapter formulas of phase5d_triton_training.py:287-312
    (z = x A^T, dB = s g^T z, dz = s g B, dA = dz^T x):
        u^T dA v = s (g (B u))^T (x v),   u^T dB v = s (g u)^T (x (A^T v)),
    matrix-vector products only.  Adapters without rows are left out."""
    _check_inputs(x, ids)
    out: Dict[int, Tuple[np.ndarray, np.ndarray]] = {}
    for aid, (uA, vA, uB, vB) in probes.items():
        ad = adapters[aid]
        mask = ids == aid
        if not mask.any():
            continue
        xs = np.asarray(x[mask], dtype=np.float64)
        g = np.asarray(dY[mask], dtype=np.float64)
        # all k probes in one pass over g and x: column i is probe i
        pa = ad.scaling * np.einsum("ni,ni->i", g @ (ad.B @ uA.T), xs @ vA.T)
        pb = ad.scaling * np.einsum("ni,ni->i", g @ uB.T, xs @ (ad.A.T @ vB.T))
        out[aid] = (pa, pb)
    return out


def sgd_step(param: np.ndarray, grad: Optional[np.ndarray], lr: float) -> np.ndarray:
    """Plain SGD, P <- P - lr * dP (phase5d_triton_training.py:554-559).

    torch.optim.SGD with no momentum/weight decay skips parameters whose grad
    is None, which is what keeps absent adapters bit-identical
    (tests/test_equivalence.py:137-141).
    """
    if grad is None:
        return param.copy()
    return param - lr * grad


def split_ranges(total: int, n: int) -> List[Tuple[int, int]]:
    """N near-equal contiguous [start, end) ranges; the first ``total % N``
    ranges get one extra row; N is clamped to [1, total]
    (phase6_two_gpu_overlap.py:73-87, phase4_aimd.py:22-36)."""
    n = min(max(1, int(n)), total)
    q, r = divmod(total, n)
    out = []
    start = 0
    for i in range(n):
        size = q + (1 if i < r else 0)
        out.append((start, start + size))
        start += size
    return out


def nano_forward_by_count(
    x: np.ndarray,
    W: np.ndarray,
    bias: Optional[np.ndarray],
    adapters: Dict[int, OracleAdapter],
    spans: Dict[int, Tuple[int, int]],
    n_nano: int,
) -> np.ndarray:
    """Per nano-batch: backbone plus only the adapter segments overlapping it,
    with segments straddling nano-batch boundaries split (phase4_aimd.py:39-80)."""
    outs = []
    for ns, ne in split_ranges(x.shape[0], n_nano):
        xn = x[ns:ne]
        res = xn @ W.T
        if bias is not None:
            res = res + bias
        for aid, (js, je) in spans.items():
            os_, oe = max(ns, js), min(ne, je)
            if os_ >= oe:
                continue
            res[os_ - ns:oe - ns] += adapter_delta(x[os_:oe], adapters[aid])
        outs.append(res)
    return np.concatenate(outs, axis=0)


class AIMDController:
    """AIMD nano-batch count controller (phase6b_real_aimd.py:59-123).

    N_{t+1} = N_t + alpha            if T_t <= T_{t-1} - tau
    N_{t+1} = max(1, floor(beta N_t)) otherwise
    Bootstrap: the first observation only records T and probes N + alpha.
    N is clamped to [1, max_n]; the best (N, T) seen is tracked.
    """

    def __init__(self, start_n=1, alpha=4, beta=0.5, tau=0.05, max_n=64):
        self.n = max(1, int(start_n))
        self.alpha = int(alpha)
        self.beta = float(beta)
        self.tau = float(tau)
        self.max_n = max(1, int(max_n))
        self.prev = None
        self.best_n = self.n
        self.best = float("inf")

    def observe(self, t: float) -> Tuple[int, str]:
        t = float(t)
        if t < self.best:
            self.best = t
            self.best_n = self.n
        if self.prev is None:
            self.prev = t
            self.n = min(self.max_n, self.n + self.alpha)
            return self.n, "bootstrap additive probe"
        if t <= self.prev - self.tau:
            nxt, why = self.n + self.alpha, "additive increase"
        else:
            nxt, why = max(1, math.floor(self.beta * self.n)), "multiplicative decrease"
        self.prev = t
        self.n = max(1, min(self.max_n, nxt))
        return self.n, why


def synthetic_iteration_time(n: int) -> float:
    """Toy U-shaped landscape in seconds (phase4_aimd.py:218-230)."""
    base_ms = 5.0
    overlap_gain_ms = 2.2 * (1.0 - math.exp(-n / 5.0))
    overhead_ms = 0.035 * n
    return (base_ms - overlap_gain_ms + overhead_ms) / 1000.0


def aimd_trace(horizons: int, tau_seconds: float, max_n: int = 60) -> List[Tuple[int, float, str, int]]:
    """The synthetic controller demo of phase4_aimd.py:233-261: returns
    (N used, time in ms, decision, next N) per horizon."""
    c = AIMDController(start_n=1, alpha=4, beta=0.5, tau=tau_seconds, max_n=max_n)
    rows = []
    for _ in range(horizons):
        used = c.n
        t = synthetic_iteration_time(used)
        nxt, why = c.observe(t)
        rows.append((used, t * 1000.0, why, nxt))
    return rows


def relative_l2(a: np.ndarray, b: np.ndarray) -> float:
    """||a-b|| / max(||b||, 1e-12) (phase5d_triton_training.py:355-369)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-12))


def training_step(
    x: np.ndarray,
    ids: np.ndarray,
    W: np.ndarray,
    bias: Optional[np.ndarray],
    adapters: Dict[int, OracleAdapter],
    dY: np.ndarray,
    lr: float,
):
    """Forward, analytic backward and one isolated SGD step.  Returns
    (Y, dX, dA, dB, A_next, B_next) with per-adapter dicts."""
    Y = multi_lora_forward(x, ids, W, bias, adapters)
    dX, dA, dB = multi_lora_backward(x, ids, W, adapters, dY)
    A_next = {a: sgd_step(ad.A, dA[a], lr) for a, ad in adapters.items()}
    B_next = {a: sgd_step(ad.B, dB[a], lr) for a, ad in adapters.items()}
    return Y, dX, dA, dB, A_next, B_next


def segments_from_ids(ids: Sequence[int]) -> List[Tuple[int, int, int]]:
    """Maximal runs (start, end, id) of equal ids in row order."""
    ids = list(ids)
    out = []
    s = 0
    for i in range(1, len(ids) + 1):
        if i == len(ids) or ids[i] != ids[s]:
            out.append((s, i, int(ids[s])))
            s = i
    return out
