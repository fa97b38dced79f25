"""CUDA-graph replay of a training step with fixed routing.

A step of the fused layer is a handful of kernel launches plus host work
(routing, plan building, argument packing).  When the job mix of a batch does
not change between steps, the whole step — fused forward, analytic backward
against the upstream gradient, isolated SGD — can be captured once into a
CUDA graph and replayed: the routing plan is uploaded once into a resident
workspace (MultiLoRALinear.make_resident, MLORA_PLAN_RESIDENT), every kernel
and the per-call reset of the work counters become graph nodes, and a replay
costs one launch.

    step = GraphedTrainStep(model, x, adapter_ids, dy, lr=1e-3)
    for batch in batches:          # same rows per adapter each step
        y = step(batch.x, batch.dy)

Inputs are copied into the graph's static buffers before each replay; the
returned Y, the adapters' .grad and the updated weights live in the graph's
memory and are overwritten by the next replay.
"""

from __future__ import annotations

from typing import Optional

import torch

from .multi_lora_linear import MultiLoRALinear


class GraphedTrainStep:
    def __init__(self, model: MultiLoRALinear, x: torch.Tensor, adapter_ids: torch.Tensor, dy: torch.Tensor,
                 lr: float, warmup: int = 3, need_dx: bool = True):
        if x.device.type != "cuda":
            raise RuntimeError("CUDA graphs need CUDA tensors")
        self.model = model
        self.lr = float(lr)
        self.plan = model.route(adapter_ids.cpu(), device=x.device)
        model.make_resident(self.plan)
        self.ids = adapter_ids.cpu()
        self.x = x.detach().clone().requires_grad_(need_dx)
        self.dy = dy.detach().clone()
        side = torch.cuda.Stream(x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):  # warm-up off the default stream, as capture requires
            for _ in range(max(1, warmup)):
                self._step()
        torch.cuda.current_stream(x.device).wait_stream(side)
        torch.cuda.synchronize(x.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.y = self._step()

    def _step(self) -> torch.Tensor:
        m = self.model
        for ad in m.adapters.values():
            ad.A.grad = None
            ad.B.grad = None
        self.x.grad = None
        y = m(self.x, self.ids, plan=self.plan)
        y.backward(self.dy)
        m.sgd_step(self.lr)
        return y

    def __call__(self, x: Optional[torch.Tensor] = None, dy: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Copy new inputs (same shapes) into the static buffers and replay
        the captured step; returns Y (graph memory)."""
        if x is not None:
            self.x.detach().copy_(x, non_blocking=True)
        if dy is not None:
            self.dy.copy_(dy, non_blocking=True)
        self.graph.replay()
        return self.y

    @property
    def dx(self) -> Optional[torch.Tensor]:
        return self.x.grad
