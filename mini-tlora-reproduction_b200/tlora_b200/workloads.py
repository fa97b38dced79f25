"""Seeded synthetic workloads of the five benchmark configurations.

No dataset is involved: every input is synthetic, with the shapes, rank and
token-count distributions and initialisation scales of each configuration.

  c0  CPU fp32 MultiLoRALinear: d_in = d_out = 1024, W ~ N(0, 1/1024), zero
      bias, 4 adapters ranks 4/8/16/32, alpha = 2r (scaling 2),
      A ~ U(-1/32, 1/32), B ~ N(0, 0.02), contiguous segments 64/128/192/256,
      X ~ N(0, 1), seed 0; fwd, bwd and one SGD step, lr 1e-3
  c1  bf16 forward: d = 4096, W ~ N(0, 1/4096), 16 adapters ranks uniform
      on {8, 16, 32, 64}, tokens per adapter uniform on [256, 2048], A/B as
      c0 scaled to d (A ~ U(-1/64, 1/64)), seed 1
  c2  bf16 training step on an MLP up-projection: 4096 -> 11008, 8 adapters
      ranks alternating 16/64, 4 sequences x 2048 tokens each (65,536 rows),
      fwd + bwd + isolated SGD, seed 2
  c3  multi-GPU: 8192 x 8192, 32 jobs ranks on {8, 16, 32, 64}, tokens
      uniform on [512, 2048], seed 3
  c4  stress: 8192 x 8192, 64 adapters ranks uniform on [1, 128], Zipf(1.2)
      token counts normalised to 65,536 rows with empty and 1-token
      segments, seed 4
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List

import numpy as np
import torch

from .multi_lora_linear import MultiLoRALinear


@dataclass
class WorkloadSpec:
    name: str
    d_in: int
    d_out: int
    ranks: List[int]
    counts: List[int]   # rows per adapter, adapter order = segment order
    seed: int
    dtype: torch.dtype
    lr: float = 1e-3
    train: bool = True  # fwd + bwd (+ SGD) vs forward only

    @property
    def rows(self) -> int:
        return int(sum(self.counts))

    def flops(self) -> float:
        """Algorithmic FLOPs of one step: forward 2 d_in d_out + 2 r (d_in + d_out)
        per row; backward (dX incl. backbone, dZ, dA, dB) 2 d_in d_out + 4 r (d_in + d_out)."""
        rsum = float(sum(r * n for r, n in zip(self.ranks, self.counts)))
        fwd = 2.0 * self.d_in * self.d_out * self.rows + 2.0 * rsum * (self.d_in + self.d_out)
        if not self.train:
            return fwd
        return fwd + 2.0 * self.d_in * self.d_out * self.rows + 4.0 * rsum * (self.d_in + self.d_out)


def _zipf_counts(rng: np.random.Generator, n: int, total: int, s: float, n_empty: int, n_one: int) -> List[int]:
    w = 1.0 / np.arange(1, n + 1) ** s
    counts = np.floor(w / w.sum() * total).astype(np.int64)
    order = rng.permutation(n)
    counts = counts[order]
    small = rng.choice(n, size=n_empty + n_one, replace=False)
    counts[small[:n_empty]] = 0
    counts[small[n_empty:]] = 1
    counts[int(np.argmax(counts))] += total - int(counts.sum())
    return [int(c) for c in counts]


def spec(name: str, scale: float = 1.0, rows_scale: float = 1.0) -> WorkloadSpec:
    """The named configuration.  ``scale`` < 1 shrinks rows and features
    (rounded to multiples of 64) for parity tests the oracle can finish;
    ``rows_scale`` shrinks the rows only (same layer shape)."""

    def d(v):
        return max(64, int(round(v * scale / 64)) * 64)

    def rows(v):
        return max(1, int(round(v * scale * rows_scale)))

    if name == "c0":
        return WorkloadSpec("c0", d(1024), d(1024), [4, 8, 16, 32], [rows(c) for c in (64, 128, 192, 256)],
                            0, torch.float32)
    if name == "c1":
        rng = np.random.default_rng(1)
        ranks = [int(x) for x in rng.choice([8, 16, 32, 64], size=16)]
        counts = [rows(int(x)) for x in rng.integers(256, 2049, size=16)]
        return WorkloadSpec("c1", d(4096), d(4096), ranks, counts, 1, torch.bfloat16, train=False)
    if name == "c2":
        ranks = [16 if i % 2 == 0 else 64 for i in range(8)]
        return WorkloadSpec("c2", d(4096), d(11008), ranks, [rows(4 * 2048)] * 8, 2, torch.bfloat16)
    if name == "c3":
        rng = np.random.default_rng(3)
        ranks = [int(x) for x in rng.choice([8, 16, 32, 64], size=32)]
        counts = [rows(int(x)) for x in rng.integers(512, 2049, size=32)]
        return WorkloadSpec("c3", d(8192), d(8192), ranks, counts, 3, torch.bfloat16)
    if name == "c4":
        rng = np.random.default_rng(4)
        ranks = [int(x) for x in rng.integers(1, 129, size=64)]
        counts = _zipf_counts(rng, 64, rows(65536), 1.2, n_empty=3, n_one=3)
        return WorkloadSpec("c4", d(8192), d(8192), ranks, counts, 4, torch.bfloat16)
    raise ValueError(f"unknown workload {name}")


@dataclass
class Workload:
    spec: WorkloadSpec
    model: MultiLoRALinear
    x: torch.Tensor
    ids: torch.Tensor
    dy: torch.Tensor  # upstream gradient of Y (the gradient the layer above hands back), N(0, 1) / rows


def build(sp: WorkloadSpec, device="cuda", dtype=None) -> Workload:
    """Random-init module and seeded inputs of ``sp`` on ``device``."""
    dtype = dtype or sp.dtype
    g = torch.Generator(device="cpu").manual_seed(sp.seed)
    ranks = {i: r for i, r in enumerate(sp.ranks)}
    torch.manual_seed(sp.seed)
    m = MultiLoRALinear(sp.d_in, sp.d_out, ranks, bias=True)
    a_bound = 1.0 / np.sqrt(sp.d_in)
    with torch.no_grad():
        m.base.weight.normal_(0.0, 1.0 / np.sqrt(sp.d_in), generator=g)
        m.base.bias.zero_()
        for i, r in ranks.items():
            ad = m.adapters[str(i)]
            ad.alpha = 2.0 * r
            ad.scaling = 2.0
            ad.A.uniform_(-a_bound, a_bound, generator=g)
            ad.B.normal_(0.0, 0.02, generator=g)
    m = m.to(device=device, dtype=dtype)
    dev = torch.device(device)
    gd = torch.Generator(device=dev).manual_seed(sp.seed + 1000)
    x = torch.randn(sp.rows, sp.d_in, generator=gd, device=dev, dtype=torch.float32).to(dtype)
    # the upstream gradient of a loss averaged over the rows (N(0, 1) / rows),
    # so that repeated SGD steps with it stay bounded
    dy = (torch.randn(sp.rows, sp.d_out, generator=gd, device=dev, dtype=torch.float32) / max(1, sp.rows)).to(dtype)
    ids = torch.cat([torch.full((c,), i, dtype=torch.int64) for i, c in enumerate(sp.counts)]).to(dev)
    return Workload(sp, m, x, ids, dy)
