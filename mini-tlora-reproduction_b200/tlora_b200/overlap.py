"""K-sharded multi-LoRA layer across the ranks of one node, with the
nano-batch compute / all-reduce overlap steered by AIMD.

Rebuild of phase6_two_gpu_overlap.py (split_ranges :73-87, run_serial
:220-244, run_pipelined :247-280, measure_distributed :283-343) and
phase6b_real_aimd.py (controller loop :245-302) for 1-8 GPUs, with the
semantics the reference's microbenchmark leaves out: the ranks hold shards of
ONE layer instead of unrelated replicas.

Partitioning (rank p of P): columns [k0, k1) of d_in.  Rank p holds
W[:, k0:k1], A_pack[:, k0:k1] and X[:, k0:k1]; B_pack is replicated.  Its
forward partial is Y_p = X_p W_p^T (+ bias and the LoRA expand on rank 0
only), Z_p = s X_p A_p^T; since both are linear in X_p, sum_p Y_p = Y and
sum_p Z_p = Z.  Per step:

  1. shrink: Z_p over all tiles, then an async SUM all-reduce of Z (small:
     128 x 64 bf16 per tile x rank chunk);
  2. for each of N nano-batches (N near-equal ranges of 128-row tiles):
     the fused mainloop over its tiles, then an async SUM all-reduce of its
     rows of Y; nano-batch i+1's mainloop overlaps nano-batch i's all-reduce;
  3. backward with the replicated dY: dX_p = dY W_p + dZ A_p and
     dA_p = dZ^T X_p are local; dB = dY^T Z uses the all-reduced Z (computed
     identically on every rank, no exchange); then the isolated SGD step.

Nano-batch boundaries are rounded to 128-row tiles (the reference splits rows
exactly); N still counts nano-batches.
"""

from __future__ import annotations

import os
import statistics
import time
from typing import List, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist

from . import ops
from ._lib import TILE_ROWS
from .nano import AIMDController, split_ranges


def shard_columns(d_in: int, rank: int, world: int, align: int = 64) -> Tuple[int, int]:
    """Contiguous column range of d_in owned by ``rank``: near-equal blocks of
    ``align`` columns (keeps every shard's row pitch 16-byte aligned)."""
    blocks = (d_in + align - 1) // align
    s, e = split_ranges(blocks, world)[rank] if blocks >= world else (rank, rank + 1)
    return min(d_in, s * align), min(d_in, e * align)


class NativeCompute:
    """The native kernels (tcgen05 for bf16) behind the sharded layer.
    ``comm_sms`` SMs are left out of the nano-batch mainloops so the NCCL
    all-reduce of the previous nano-batch has SMs to run on."""

    def __init__(self, impl: str = "auto", comm_sms: int = 16):
        self.impl = impl
        self.comm_sms = int(comm_sms)
        self._sms = None

    def _main_ctas(self, device):
        if self.comm_sms <= 0:
            return 0
        if self._sms is None:
            self._sms = torch.cuda.get_device_properties(device).multi_processor_count
        return max(1, self._sms - self.comm_sms)

    def begin(self, layer, x_p, plan):
        st = ops.LayerState(layer.table, layer.scaling, plan, layer.A_pack, layer.B_pack, self.impl)
        fw = ops.StagedForward(x_p, layer.W, layer.bias, st)
        zbytes = ops._CallArgs(x_p.shape[0], x_p.shape[1], layer.B_pack.shape[0], ops.mlora_dtype(x_p.dtype),
                               self.impl, plan, layer.table, layer.scaling).sizes()[0]
        zview = fw.z[:zbytes].view(x_p.dtype) if zbytes else None
        return {"fw": fw, "st": st, "z": zview, "y": fw.y, "n_tiles": fw.n_tiles}

    def shrink(self, ctx):
        ctx["fw"].shrink()

    def main(self, ctx, t0, t1, expand, add_bias):
        ctx["fw"].main(t0, t1, expand=expand, add_bias=add_bias, max_ctas=self._main_ctas(ctx["fw"].x.device))

    def backward(self, ctx, layer, x_p, dy, overlapped=False):
        st = ctx["st"]
        if overlapped:  # leave SMs to the all-reduces still in flight
            st = ops.LayerState(st.table, st.scaling, st.plan, st.A_pack, st.B_pack, st.impl,
                                self._main_ctas(x_p.device))
        return ops.backward_raw(dy, x_p, layer.W, ctx["fw"].z, st, True, True, True)

    def sgd(self, layer, plan, dA_p, dB, lr):
        pairs = []
        for i in range(layer.table.n):
            if not plan.active[i]:
                continue
            o, r = int(layer.table.pack_off[i]), int(layer.table.rank[i])
            pairs.append((layer.A_pack[o:o + r], dA_p[o:o + r]))
            pairs.append((layer.B_pack[:, o:o + r], dB[:, o:o + r]))
        return ops.sgd_step_(pairs, lr)


class ShardedLayer:
    """Rank ``rank``'s K-shard of a MultiLoRALinear (see module docstring)."""

    def __init__(self, model, rank: int, world: int, compute=None, group=None):
        self.rank, self.world, self.group = rank, world, group
        A_pack, B_pack, table = model.packed()
        d_in = model.base.in_features
        self.k0, self.k1 = shard_columns(d_in, rank, world)
        with torch.no_grad():
            self.W = model.base.weight[:, self.k0:self.k1].contiguous()
            self.A_pack = A_pack[:, self.k0:self.k1].contiguous()
            self.B_pack = B_pack.clone()
            self.bias = model.base.bias.detach().clone() if (rank == 0 and model.base.bias is not None) else None
        self.table = table
        self.scaling = np.array([float(a.scaling) for a in model.adapters.values()], dtype=np.float32)
        self.compute = compute or NativeCompute(getattr(model, "impl", "auto"))

    def shard_input(self, x: torch.Tensor) -> torch.Tensor:
        return x[:, self.k0:self.k1].contiguous()

    def forward(self, x_p, plan, n_nano: int, pipelined: bool = True, comm: bool = True):
        """Pipelined forward; returns (Y, ctx) with every collective complete.
        ``comm=False`` skips the collectives (compute-only timing)."""
        y, ctx, works, hz = self.forward_async(x_p, plan, n_nano, pipelined, comm)
        for w in works:
            w.wait()
        if hz is not None:
            hz.wait()
        return y, ctx

    def forward_async(self, x_p, plan, n_nano: int, pipelined: bool = True, comm: bool = True):
        """Pipelined forward that returns with the nano-batch all-reduces still
        in flight: (Y, ctx, Y work handles, Z work handle or None)."""
        c = self.compute
        ctx = c.begin(self, x_p, plan)
        c.shrink(ctx)
        hz = None
        if comm and ctx["z"] is not None:
            hz = dist.all_reduce(ctx["z"], op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        owner = self.rank == 0
        if owner and hz is not None:
            hz.wait()
            hz = None
        rows = x_p.shape[0]
        works = []
        for t0, t1 in split_ranges(ctx["n_tiles"], n_nano):
            c.main(ctx, t0, t1, expand=owner, add_bias=owner)
            if not comm:
                continue
            seg = ctx["y"][t0 * TILE_ROWS:min(t1 * TILE_ROWS, rows)]
            if pipelined:
                works.append(dist.all_reduce(seg, op=dist.ReduceOp.SUM, group=self.group, async_op=True))
            else:
                dist.all_reduce(seg, op=dist.ReduceOp.SUM, group=self.group)
        return ctx["y"], ctx, works, hz

    def backward(self, ctx, x_p, dy, overlapped=False):
        return self.compute.backward(ctx, self, x_p, dy, overlapped)

    def step(self, x_p, plan, dy, n_nano: int, lr: float, pipelined: bool = True, comm: bool = True):
        """Forward, backward and isolated SGD on this rank's shard.  Returns
        (Y, dX_p).  With ``pipelined`` the nano-batch all-reduces of Y overlap
        the following nano-batches AND the backward: dY is the upstream
        gradient, so the backward needs only the (small) all-reduced Z; the
        Y all-reduces are waited for at the end of the step."""
        y, ctx, works, hz = self.forward_async(x_p, plan, n_nano, pipelined, comm)
        if hz is not None:
            hz.wait()  # dB = dY^T Z needs the summed Z
        dx_p, dA_p, dB = self.backward(ctx, x_p, dy, overlapped=bool(works))
        self.compute.sgd(self, plan, dA_p, dB, lr)
        for w in works:
            w.wait()
        return y, dx_p


def comm_only(layer: ShardedLayer, y: torch.Tensor, z: Optional[torch.Tensor], n_tiles: int, n_nano: int):
    """The step's collectives alone (for the overlap fraction)."""
    works = []
    if z is not None:
        works.append(dist.all_reduce(z, op=dist.ReduceOp.SUM, group=layer.group, async_op=True))
    rows = y.shape[0]
    for t0, t1 in split_ranges(n_tiles, n_nano):
        seg = y[t0 * TILE_ROWS:min(t1 * TILE_ROWS, rows)]
        works.append(dist.all_reduce(seg, op=dist.ReduceOp.SUM, group=layer.group, async_op=True))
    for w in works:
        w.wait()


# ---------------------------------------------------------------------------
# benchmark driver (bench.py --gpus N)
# ---------------------------------------------------------------------------

def _timed(fn, iters: int, device) -> float:
    """Mean device ms per call, max over ranks (phase6_two_gpu_overlap.py:283-343)."""
    dist.barrier()
    torch.cuda.synchronize(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize(device)
    t = torch.tensor([e0.elapsed_time(e1) / iters], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def bench_multi(args, peaks_d, peaks_kind, metric, unit):
    import datetime

    from . import _lib, workloads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    # SMs the mainloops leave to NCCL while all-reduces are in flight
    # (MLORA_COMM_SMS), and optionally NCCL's channel (CTA) count
    # (MLORA_NCCL_CHANNELS, fixed before the communicator exists)
    comm_sms = int(os.environ.get("MLORA_COMM_SMS", "16"))
    if os.environ.get("MLORA_NCCL_CHANNELS"):
        os.environ.setdefault("NCCL_MAX_NCHANNELS", os.environ["MLORA_NCCL_CHANNELS"])
        os.environ.setdefault("NCCL_MIN_NCHANNELS", os.environ["MLORA_NCCL_CHANNELS"])
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        sp = workloads.spec(args.workload)
        w = workloads.build(sp, device=dev)
        layer = ShardedLayer(w.model, rank, world, compute=NativeCompute(comm_sms=comm_sms))
        x_p = layer.shard_input(w.x)
        plan = ops.route(w.ids, layer.table, dev)
        lr = sp.lr
        dy = w.dy
        n_tiles = (sp.rows + TILE_ROWS - 1) // TILE_ROWS

        def stepper(n, pipelined=True, comm=True):
            return lambda: layer.step(x_p, plan, dy, n, lr, pipelined, comm)

        for _ in range(max(3, args.warmup)):
            stepper(4)()
        torch.cuda.synchronize(dev)

        # AIMD over the real pipelined step (phase6b_real_aimd.py:245-302)
        ctl = AIMDController(start_n=1, alpha=4, beta=0.5, tau_ms=0.05, max_n=min(32, n_tiles))
        horizons = []
        for _ in range(8):
            n = ctl.n
            t = _timed(stepper(n), 3, dev)
            nxt, why = ctl.observe(t)
            horizons.append({"n": n, "ms": round(t, 4), "decision": why, "next_n": nxt})
        best_n = ctl.best_n

        # SMs left to NCCL during the nano-batch mainloops (the persistent
        # mainloop would otherwise hold every SM and serialise the all-reduce)
        sm_sweep = {}
        for k in sorted({0, comm_sms // 2, comm_sms, comm_sms + comm_sms // 2}):
            layer.compute.comm_sms = k
            sm_sweep[k] = _timed(stepper(best_n), 3, dev)
        best_k = min(sm_sweep, key=sm_sweep.get)
        layer.compute.comm_sms = best_k

        # overlap accounting at the chosen N
        t_pipe = _timed(stepper(best_n), 3, dev)
        t_serial = _timed(stepper(best_n, pipelined=False), 3, dev)
        t_compute = _timed(stepper(best_n, comm=False), 3, dev)
        y_buf, ctx = layer.forward(x_p, plan, best_n)
        t_comm = _timed(lambda: comm_only(layer, y_buf, ctx["z"], n_tiles, best_n), 3, dev)
        hidden = 1.0 - max(0.0, t_pipe - t_compute) / t_comm if t_comm > 0 else 0.0

        # timed region
        launches0 = _lib.launch_count()
        ms = _timed(stepper(best_n), args.steps, dev)
        launches = _lib.launch_count() - launches0

        # end to end: every step copies its X shard from pinned host memory
        # (copy stream, double-buffered: step i+1's copy overlaps step i) and
        # reads a probe of the updated adapter weights back to the host
        x_host = x_p.detach().cpu().pin_memory()
        bufs = [torch.empty_like(x_p) for _ in range(2)]
        copied = [torch.cuda.Event() for _ in range(2)]
        consumed = [torch.cuda.Event() for _ in range(2)]
        copy_stream = torch.cuda.Stream(dev)
        compute = torch.cuda.current_stream(dev)
        probe = torch.empty(64, dtype=x_p.dtype).pin_memory()
        counter = [0]

        def issue_copy(i):
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(consumed[i % 2])
                bufs[i % 2].copy_(x_host, non_blocking=True)
                copied[i % 2].record(copy_stream)

        def e2e():
            i = counter[0]
            counter[0] += 1
            compute.wait_event(copied[i % 2])
            issue_copy(i + 1)
            layer.step(bufs[i % 2], plan, dy, best_n, lr)
            consumed[i % 2].record(compute)
            probe.copy_(layer.A_pack[0, :64], non_blocking=True)
            compute.synchronize()

        for ev in consumed:
            ev.record(compute)
        issue_copy(0)
        e2e()
        e2e_ms = _timed(e2e, max(3, args.steps // 2), dev)
        torch.cuda.synchronize(dev)

        if rank != 0:
            return None
        step_flops = sp.flops()
        return {
            "metric": metric, "value": round(sp.rows / (ms / 1000.0), 1), "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; random-init weights)",
            "config": {"workload": f"{sp.name}: fwd+bwd+isolated SGD d_in={sp.d_in} d_out={sp.d_out}, "
                                   f"backbone K-sharded over {world} GPUs, nano-batch all-reduce overlap",
                       "rows": sp.rows, "global_batch": sp.rows, "seq_len": None,
                       "parallelism": f"K-shard x{world} + nano-batch pipeline (AIMD N={best_n})",
                       "l2": "per-step traffic (Y all-reduce, 1.4 GiB) larger than L2"},
            "step_tflops": round(step_flops / (ms / 1000.0) / 1e12, 1),
            "overlap": {"n": best_n, "comm_sms": best_k, "nccl_channels": os.environ.get("NCCL_MAX_NCHANNELS"),
                        "comm_sms_sweep_ms": {str(k): round(v, 4) for k, v in sm_sweep.items()},
                        "pipelined_ms": round(t_pipe, 4), "serial_ms": round(t_serial, 4),
                        "compute_only_ms": round(t_compute, 4), "comm_only_ms": round(t_comm, 4),
                        "comm_hidden_frac": round(hidden, 4)},
            "aimd": horizons,
            "e2e": {"value": round(sp.rows / (e2e_ms / 1000.0), 1), "unit": unit, "ms_per_step": round(e2e_ms, 3),
                    "h2d_bytes_per_step": int(x_p.numel() * x_p.element_size()),
                    "d2h_bytes_per_step": int(probe.numel() * probe.element_size())},
            "gpu_launches": int(launches),
        }
    finally:
        dist.barrier()
        dist.destroy_process_group()
