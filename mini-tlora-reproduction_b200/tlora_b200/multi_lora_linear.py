"""Drop-in replacement of the reference's ``tlora/multi_lora_linear.py``.

Same classes, constructor signatures, attributes, ``state_dict`` keys
(``base.weight``, ``base.bias``, ``adapters.<id>.A``, ``adapters.<id>.B``),
``adapter_parameters`` and ``ValueError``s; the same random initialisation
sequence, so a seeded construction yields the same weights as the reference.
Forward and backward run in the native sm_100a library (tcgen05 tensor-core
kernels for bf16, CUDA-core fp32 kernels for fp32) on CUDA tensors; there is
no CPU path and no PyTorch fallback for the computation.

Storage: every adapter's ``A`` [rank, in] and ``B`` [out, rank] is a view into
two packed buffers per module, ``A_pack`` [r_pack, in] and ``B_pack``
[out, r_pack], with each adapter's rank padded to a multiple of 64
(zeros).  The kernels read the packs directly, optimizers update the views in
place, and gradients come back as views of packed gradient buffers.
"""

from __future__ import annotations

import math
from typing import Dict, Iterable, Optional

import numpy as np
import torch
import torch.nn as nn

from . import ops


class LoRAAdapter(nn.Module):
    """A minimal LoRA branch: delta(x) = scaling * (x @ A^T) @ B^T.

    tlora/multi_lora_linear.py:9-31: A [rank, in] kaiming-uniform(a=sqrt(5)),
    B [out, rank] zeros, alpha defaults to rank, scaling = alpha / rank."""

    def __init__(self, in_features: int, out_features: int, rank: int, alpha: float | None = None):
        super().__init__()
        if rank <= 0:
            raise ValueError("rank must be > 0")
        self.rank = rank
        self.alpha = float(alpha if alpha is not None else rank)
        self.scaling = self.alpha / self.rank
        self.A = nn.Parameter(torch.empty(rank, in_features))
        self.B = nn.Parameter(torch.zeros(out_features, rank))
        nn.init.kaiming_uniform_(self.A, a=math.sqrt(5))
        self.in_features = in_features
        self.out_features = out_features

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """The adapter's delta alone (no backbone), through the native
        delta-only kernel path (the reference kernel's ADD_BASE=False)."""
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        ids = torch.zeros(x2.shape[0], dtype=torch.int64)
        packed = self.__dict__.get("_packed")
        if packed is None or not packed.owns({"0": self}):
            packed = _PackedAdapters({"0": self})
            self.__dict__["_packed"] = packed
        y = packed.apply(x2, ids, None, None, impl="auto")
        return y.reshape(*lead, self.out_features)


class IndependentLoRALinear(nn.Module):
    """One LoRA job on its own frozen backbone (tlora/multi_lora_linear.py:34-56)."""

    def __init__(self, in_features: int, out_features: int, rank: int, bias: bool = True,
                 alpha: float | None = None):
        super().__init__()
        self.base = nn.Linear(in_features, out_features, bias=bias)
        for p in self.base.parameters():
            p.requires_grad_(False)
        self.adapter = LoRAAdapter(in_features, out_features, rank, alpha)
        self._packed = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        ids = torch.zeros(x2.shape[0], dtype=torch.int64)
        if self._packed is None or not self._packed.owns({"0": self.adapter}):
            self._packed = _PackedAdapters({"0": self.adapter})
        y = self._packed.apply(x2, ids, self.base.weight, self.base.bias, impl="auto")
        return y.reshape(*lead, self.base.out_features)


class _PackedAdapters:
    """Packed storage of a set of adapters and the call into the native op.

    The packs are (re)built when the adapters' parameters no longer view them
    (first call, ``.to()``/``.cuda()``, a replaced Parameter); otherwise the
    parameters already live in the packs and nothing is copied."""

    def __init__(self, adapters: Dict[str, LoRAAdapter]):
        self.keys = list(adapters.keys())
        self.adapters = [adapters[k] for k in self.keys]
        self.table = ops.AdapterTable.build([int(k) for k in self.keys], [a.rank for a in self.adapters])
        self.A_pack: Optional[torch.Tensor] = None
        self.B_pack: Optional[torch.Tensor] = None
        self._views = None

    def owns(self, adapters: Dict[str, LoRAAdapter]) -> bool:
        return list(adapters.keys()) == self.keys and all(
            a is b for a, b in zip((adapters[k] for k in self.keys), self.adapters))

    def _in_sync(self) -> bool:
        if self._views is None:
            return False
        for ad, (pa, pb) in zip(self.adapters, self._views):
            if ad.A.data_ptr() != pa or ad.B.data_ptr() != pb:
                return False
            if ad.A.device != self.A_pack.device or ad.A.dtype != self.A_pack.dtype:
                return False
            if ad.B.device != self.A_pack.device or ad.B.dtype != self.A_pack.dtype:
                return False
        return True

    def sync(self):
        if self._in_sync():
            return
        ref = self.adapters[0].A
        dev, dt = ref.device, ref.dtype
        d_in = ref.shape[1]
        d_out = self.adapters[0].B.shape[0]
        R = self.table.r_pack
        A_pack = torch.zeros(R, d_in, device=dev, dtype=dt)
        B_pack = torch.zeros(d_out, R, device=dev, dtype=dt)
        views = []
        with torch.no_grad():
            for i, ad in enumerate(self.adapters):
                if ad.A.device != dev or ad.B.device != dev or ad.A.dtype != dt or ad.B.dtype != dt:
                    raise RuntimeError("all adapters of a module must share one device and dtype")
                o, r = int(self.table.pack_off[i]), int(self.table.rank[i])
                A_pack[o:o + r].copy_(ad.A)
                B_pack[:, o:o + r].copy_(ad.B)
                ad.A.data = A_pack[o:o + r]
                ad.B.data = B_pack[:, o:o + r]
                views.append((ad.A.data_ptr(), ad.B.data_ptr()))
        self.A_pack, self.B_pack, self._views = A_pack, B_pack, views

    def scaling(self) -> np.ndarray:
        return np.array([float(a.scaling) for a in self.adapters], dtype=np.float32)

    def apply(self, x, ids, W, bias, impl="auto", plan: Optional[ops.RoutePlan] = None):
        if x.device.type != "cuda":
            raise RuntimeError(
                "tlora_b200 computes on CUDA devices only (sm_100a); move the module and inputs to a "
                "B200 with .cuda() -- there is no CPU path")
        self.sync()
        if self.A_pack.device != x.device:
            raise RuntimeError(f"input on {x.device} but adapters on {self.A_pack.device}")
        if x.dtype != self.A_pack.dtype or (W is not None and W.dtype != x.dtype):
            raise RuntimeError(f"dtype mismatch: input {x.dtype}, weights {self.A_pack.dtype}")
        if W is not None and W.requires_grad and torch.is_grad_enabled():
            raise NotImplementedError("the backbone is frozen: no dW (tlora/multi_lora_linear.py:78-80)")
        x = x.contiguous()
        if plan is None:
            plan = ops.route(ids, self.table, x.device)
        st = ops.LayerState(self.table, self.scaling(), plan, self.A_pack, self.B_pack, impl)
        params = []
        for ad in self.adapters:
            params += [ad.A, ad.B]
        Wc = W.contiguous() if W is not None else None
        bc = bias.contiguous() if bias is not None else None
        with torch.cuda.device(x.device):
            return ops.MultiLoRAFunction.apply(x, Wc, bc, st, *params)


class MultiLoRALinear(nn.Module):
    """Shared frozen backbone + heterogeneous-rank adapters, one per job.

    tlora/multi_lora_linear.py:59-118.  ``forward(x, adapter_ids)`` takes
    ``x`` [batch, in_features] and per-row adapter ids [batch] in any order;
    rows whose id names no adapter get the backbone output only.  ``impl``
    selects the kernel family: "auto" (tcgen05 for bf16, SIMT otherwise),
    "tc" or "simt"."""

    def __init__(self, in_features: int, out_features: int, adapter_ranks: Dict[int, int], bias: bool = True):
        super().__init__()
        if not adapter_ranks:
            raise ValueError("adapter_ranks cannot be empty")
        self.base = nn.Linear(in_features, out_features, bias=bias)
        for p in self.base.parameters():
            p.requires_grad_(False)
        self.adapters = nn.ModuleDict(
            {str(adapter_id): LoRAAdapter(in_features, out_features, rank)
             for adapter_id, rank in adapter_ranks.items()})
        self.impl = "auto"
        self._packed: Optional[_PackedAdapters] = None

    def adapter_parameters(self, adapter_id: int) -> Iterable[nn.Parameter]:
        return self.adapters[str(adapter_id)].parameters()

    def _pack(self) -> _PackedAdapters:
        ads = dict(self.adapters.items())
        if self._packed is None or not self._packed.owns(ads):
            self._packed = _PackedAdapters(ads)
        return self._packed

    @property
    def adapter_table(self) -> ops.AdapterTable:
        return self._pack().table

    def route(self, adapter_ids: torch.Tensor, device=None) -> ops.RoutePlan:
        """Routing plan of ``adapter_ids``; pass it back as ``plan=`` to reuse
        it across calls with the same ids."""
        dev = torch.device(device) if device is not None else self.base.weight.device
        return ops.route(adapter_ids, self._pack().table, dev)

    def make_resident(self, plan: ops.RoutePlan) -> None:
        """Upload the routing ``plan`` once into a device workspace kept on the
        plan; calls with ``plan=plan`` then issue no host-to-device copy, so a
        training step with fixed routing can be captured into a CUDA graph
        (tlora_b200.graphs.GraphedTrainStep).  The adapters' ranks and
        scalings must not change afterwards."""
        pk = self._pack()
        pk.sync()
        st = ops.LayerState(pk.table, pk.scaling(), plan, pk.A_pack, pk.B_pack, self.impl)
        w = self.base.weight
        ops.make_resident(st, plan.rows, self.base.in_features, self.base.out_features, w.dtype, w.device)

    def packed(self):
        """(A_pack, B_pack, AdapterTable): the packed adapter storage."""
        p = self._pack()
        p.sync()
        return p.A_pack, p.B_pack, p.table

    def forward(self, x: torch.Tensor, adapter_ids: torch.Tensor, plan: Optional[ops.RoutePlan] = None,
                add_base: bool = True) -> torch.Tensor:
        if x.ndim != 2:
            raise ValueError("Phase 1 expects x shaped [batch, in_features]")
        if adapter_ids.ndim != 1 or adapter_ids.shape[0] != x.shape[0]:
            raise ValueError("adapter_ids must be [batch] and match x.shape[0]")
        W = self.base.weight if add_base else None
        b = self.base.bias if add_base else None
        return self._pack().apply(x, adapter_ids, W, b, impl=self.impl, plan=plan)

    @torch.no_grad()
    def sgd_step(self, lr: float, adapter_ids: Optional[Iterable[int]] = None) -> int:
        """Isolated SGD over the adapters listed (all by default), one native
        launch: P <- P - lr * P.grad for each listed adapter whose grads are
        set; every other adapter is neither read nor written.  Equivalent to
        one ``torch.optim.SGD(model.adapter_parameters(id), lr)`` step per
        listed adapter (phase3_nano_batch.py:90-107).  Returns the number of
        tensors updated."""
        keys = [str(a) for a in adapter_ids] if adapter_ids is not None else list(self.adapters.keys())
        pairs = []
        for k in keys:
            ad = self.adapters[k]
            for p in (ad.A, ad.B):
                if p.grad is not None:
                    pairs.append((p, p.grad))
        return ops.sgd_step_(pairs, lr)
