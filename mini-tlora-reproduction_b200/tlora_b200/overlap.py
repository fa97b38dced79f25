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
     256 x 64 bf16 per tile x rank chunk);
  2. for each of N nano-batches (N near-equal ranges of 256-row plan tiles):
     the fused mainloop over its tiles, then an async SUM all-reduce of its
     rows of Y; nano-batch i+1's mainloop overlaps nano-batch i's all-reduce;
  3. backward with the replicated dY, overlapping the Y all-reduces still in
     flight: dZ = s dY B is split by tiles and dB = dY^T Z by 128-row blocks
     of d_out across the ranks, each summed with a small all-reduce on a
     second communicator (so it does not queue behind the Y traffic);
     dX_p = dY W_p + dZ A_p and dA_p = dZ^T X_p are local; then the isolated
     SGD step.

Nano-batch boundaries are rounded to 256-row plan tiles (the reference splits rows
exactly); N still counts nano-batches.

The Y all-reduce of step 2 has two implementations (``ShardedLayer.comm``):
"nccl" (an async SUM all-reduce per nano-batch, as the reference) and "peer"
(peer.PeerAllReduce: the mainloop's epilogue writes each partial tile straight
into its owner rank's receive buffer over NVLink, and a small owner kernel on
a side stream adds the partials of its tiles and writes the sums into every
rank's Y while the next nano-batch's mainloop runs).  The routing plan must
keep the rows in their order (adapter-sorted ids).
"""

from __future__ import annotations

import os
import statistics
import time
from typing import List, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist

from . import ops, peer
from ._lib import TILE_ROWS
from .nano import AIMDController, split_ranges


class _Range:
    """NVTX range (visible in Nsight timelines) around a phase of the step;
    a no-op without CUDA."""

    def __init__(self, name: str):
        self.name = name
        self.on = torch.cuda.is_available()

    def __enter__(self):
        if self.on:
            torch.cuda.nvtx.range_push(self.name)

    def __exit__(self, *exc):
        if self.on:
            torch.cuda.nvtx.range_pop()
        return False


def shard_columns(d_in: int, rank: int, world: int, align: int = 64) -> Tuple[int, int]:
    """Contiguous column range of d_in owned by ``rank``: near-equal blocks of
    ``align`` columns (keeps every shard's row pitch 16-byte aligned)."""
    blocks = (d_in + align - 1) // align
    s, e = split_ranges(blocks, world)[rank] if blocks >= world else (rank, rank + 1)
    return min(d_in, s * align), min(d_in, e * align)


def _share(total: int, rank: int, world: int) -> Tuple[int, int]:
    """Rank ``rank``'s contiguous share of ``total`` items (empty when there
    are fewer items than ranks and this rank gets none)."""
    if total <= 0:
        return 0, 0
    spans = split_ranges(total, world)
    return spans[rank] if rank < len(spans) else (total, total)


class NativeCompute:
    """The native kernels (tcgen05 for bf16) behind the sharded layer.
    ``comm_sms`` SMs can be left out of the mainloops that run beside the
    NCCL all-reduces.  The kernels hand out work items dynamically, so CTAs
    that find their SM taken by NCCL simply start later and take fewer items;
    0 (no reservation) is the measured best on B200."""

    def __init__(self, impl: str = "auto", comm_sms: int = 0):
        self.impl = impl
        self.comm_sms = int(comm_sms)
        self._sms = None

    def _main_ctas(self, device):
        if self.comm_sms <= 0:
            return 0
        if self._sms is None:
            self._sms = torch.cuda.get_device_properties(device).multi_processor_count
        return max(1, self._sms - self.comm_sms)

    def begin(self, layer, x_p, plan, y=None):
        st = ops.LayerState(layer.table, layer.scaling, plan, layer.A_pack, layer.B_pack, self.impl)
        fw = ops.StagedForward(x_p, layer.W, layer.bias, st, y=y)
        zbytes = ops._CallArgs(x_p.shape[0], x_p.shape[1], layer.B_pack.shape[0], ops.mlora_dtype(x_p.dtype),
                               self.impl, plan, layer.table, layer.scaling).sizes()[0]
        zview = fw.z[:zbytes].view(x_p.dtype) if zbytes else None
        return {"fw": fw, "st": st, "z": zview, "y": fw.y, "n_tiles": fw.n_tiles}

    def shrink(self, ctx):
        ctx["fw"].shrink()

    def main(self, ctx, t0, t1, expand, add_bias):
        ctx["fw"].main(t0, t1, expand=expand, add_bias=add_bias, max_ctas=self._main_ctas(ctx["fw"].x.device))

    def push(self, ctx, ar, t0, t1, expand, add_bias):
        ctx["fw"].push(ar, t0, t1, expand=expand, add_bias=add_bias)

    def bwd_begin(self, ctx, layer, x_p, dy, overlapped=False):
        st = ctx["st"]
        if overlapped:  # leave SMs to the all-reduces still in flight
            st = ops.LayerState(st.table, st.scaling, st.plan, st.A_pack, st.B_pack, st.impl,
                                self._main_ctas(x_p.device))
        bw = ops.StagedBackward(dy, x_p, layer.W, ctx["fw"].z, st)
        return {"bw": bw, "dz": bw.dz_view(), "dx": bw.dx, "dA": bw.dA, "dB": bw.dB,
                "n_tiles": bw.n_tiles, "n_db": bw.n_db}

    def bwd_dz(self, b, t0, t1):
        b["bw"].run_dz(t0, t1)

    def bwd_dx_da(self, b):
        b["bw"].run_dx()
        b["bw"].run_da()

    def bwd_db(self, b, b0, b1):
        b["bw"].run_db(b0, b1)

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

    def __init__(self, model, rank: int, world: int, compute=None, group=None, bwd_group=None,
                 comm: str = "nccl"):
        # `bwd_group`: a second communicator for the backward's small
        # all-reduces (dZ, dB), so they do not queue behind the large Y
        # all-reduces still in flight on `group`
        if comm not in ("nccl", "peer"):
            raise ValueError(f"comm must be 'nccl' or 'peer', not {comm!r}")
        self.rank, self.world, self.group = rank, world, group
        self.comm = comm
        self._ar = None
        self._last_done = None
        self._pending = None  # the peer all-reduce's last finish, until launched
        # set to a list to record a timeline of the next steps: (phase, CUDA
        # event on the stream that runs it); read with timeline_ms()
        self.timeline = None
        self.bwd_group = bwd_group if bwd_group is not None else group
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

    def _mark(self, name: str, stream=None) -> None:
        if self.timeline is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            self.timeline.append((name, ev))

    def timeline_ms(self) -> dict:
        """Milliseconds from the first recorded phase to the end of each
        recorded phase (waits for the device)."""
        if not self.timeline:
            return {}
        torch.cuda.synchronize()
        t0 = self.timeline[0][1]
        return {name: round(t0.elapsed_time(ev), 4) for name, ev in self.timeline}

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

    def forward_async(self, x_p, plan, n_nano: int, pipelined: bool = True, comm: bool = True,
                      defer_finish: bool = False):
        """Pipelined forward that returns with the nano-batch all-reduces still
        in flight: (Y, ctx, Y work handles, Z work handle or None).  With the
        peer all-reduce and ``defer_finish``, the last nano-batch's finish is
        launched by the returned handle's ``launch()`` (or its ``wait()``), so
        that the caller can queue it beside work of its choice."""
        if comm and pipelined and self.comm == "peer" and self.world > 1:
            return self._forward_peer(x_p, plan, n_nano, defer_finish)
        c = self.compute
        self._mark("start")
        ctx = c.begin(self, x_p, plan)
        with _Range("mlora.shrink"):
            c.shrink(ctx)
        self._mark("shrink")
        hz = None
        if comm and ctx["z"] is not None:
            hz = dist.all_reduce(ctx["z"], op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        owner = self.rank == 0
        if owner and hz is not None:
            hz.wait()
            hz = None
        rows = x_p.shape[0]
        works = []
        for i, (t0, t1) in enumerate(split_ranges(ctx["n_tiles"], n_nano)):
            with _Range(f"mlora.nano{i}"):
                c.main(ctx, t0, t1, expand=owner, add_bias=owner)
                self._mark(f"main{i}")
                if not comm:
                    continue
                seg = ctx["y"][t0 * TILE_ROWS:min(t1 * TILE_ROWS, rows)]
                if pipelined:
                    works.append(dist.all_reduce(seg, op=dist.ReduceOp.SUM, group=self.group, async_op=True))
                else:
                    dist.all_reduce(seg, op=dist.ReduceOp.SUM, group=self.group)
        return ctx["y"], ctx, works, hz

    def peer_buffers(self, rows: int, dtype, device) -> "peer.PeerAllReduce":
        """This rank's peer all-reduce buffers for ``rows`` rows (collective
        on first use or when the row count or dtype changes)."""
        if self._ar is None or self._ar.rows != rows or self._ar.dtype != dtype:
            self.close()  # no rank still uses the old buffers; every rank unmaps before any frees
            d_out = self.B_pack.shape[0]
            self._ar = peer.PeerAllReduce.over_group(rows, d_out, dtype, device, self.group)
            self._one = torch.zeros(1, dtype=torch.float32, device=device)
            self._side = torch.cuda.Stream(device)
        return self._ar

    def _forward_peer(self, x_p, plan, n_nano: int, defer_finish: bool = False):
        """forward_async with the Y all-reduce issued from the forward epilogue
        (peer.PeerAllReduce); the returned work handle makes the caller's
        stream wait until every row of Y holds the sum.  Y is the peer buffer
        and is overwritten by this layer's next forward."""
        if plan.perm is not None:
            raise ValueError("the peer all-reduce needs a routing plan that keeps the row order")
        c = self.compute
        dev = x_p.device
        rows = x_p.shape[0]
        ar = self.peer_buffers(rows, x_p.dtype, dev)
        if self._pending is not None:
            self._pending.launch()  # a previous call's deferred finish that nobody launched
        cur = torch.cuda.current_stream(dev)
        if self._last_done is not None:
            cur.wait_event(self._last_done)  # this rank's previous call is finished with the buffers
        self._mark("start")
        ar.reset(cur)
        # every rank's counters are zero before any rank pushes (and every
        # rank's previous call has finished with the buffers)
        dist.all_reduce(self._one, op=dist.ReduceOp.SUM, group=self.group)
        self._mark("barrier")
        ctx = c.begin(self, x_p, plan, y=ar.y)
        with _Range("mlora.shrink"):
            c.shrink(ctx)
        self._mark("shrink")
        hz = None
        if ctx["z"] is not None:
            hz = dist.all_reduce(ctx["z"], op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        owner = self.rank == 0
        if owner and hz is not None:
            hz.wait()
            hz = None
        side = self._side
        ranges = split_ranges(ctx["n_tiles"], n_nano)
        for i, (t0, t1) in enumerate(ranges):
            with _Range(f"mlora.nano{i}"):
                c.push(ctx, ar, t0, t1, expand=owner, add_bias=owner)
                self._mark(f"push{i}", cur)
                if i + 1 < len(ranges):
                    ev = torch.cuda.Event()
                    ev.record(cur)
                    side.wait_event(ev)
                    ar.finish(t0, t1, side)
                    self._mark(f"finish{i}", side)
        last = _PeerFinish(self, ar, ranges[-1], len(ranges) - 1, dev)
        self._pending = last
        if not defer_finish:
            last.launch()
        return ar.y, ctx, [last], hz

    def close(self) -> None:
        """Release the peer buffers (collective: every rank calls it after its
        device work; each rank unmaps its peers' buffers before any rank frees
        its own)."""
        if self._ar is None:
            return
        torch.cuda.synchronize(self._ar.device)
        dist.barrier(group=self.group)
        self._ar.close_peers()
        dist.barrier(group=self.group)
        self._ar.close()
        self._ar = None
        self._last_done = None
        self._pending = None

    def backward(self, ctx, x_p, dy, overlapped=False, after_dz=None):
        """Backward on this rank's shard.  dZ (needs all of dY and B) and dB
        (needs all of dY and Z) are split across ranks — dZ by tiles, dB by
        128-row blocks of d_out — and summed with two small all-reduces;
        dX_p and dA_p are local.  Returns (dX_p, dA_p, dB)."""
        c = self.compute
        b = c.bwd_begin(ctx, self, x_p, dy, overlapped)
        t0, t1 = _share(b["n_tiles"], self.rank, self.world)
        c.bwd_dz(b, t0, t1)
        self._mark("bwd_dz")
        if b["dz"] is not None and self.world > 1:
            dist.all_reduce(b["dz"], op=dist.ReduceOp.SUM, group=self.bwd_group)
            self._mark("bwd_dz_allreduce")
        if after_dz is not None:
            after_dz()
        c.bwd_dx_da(b)
        self._mark("bwd_dx_da")
        b0, b1 = _share(b["n_db"], self.rank, self.world)
        c.bwd_db(b, b0, b1)
        if self.world > 1:
            dist.all_reduce(b["dB"], op=dist.ReduceOp.SUM, group=self.bwd_group)
        self._mark("bwd_db")
        return b["dx"], b["dA"], b["dB"]

    def step(self, x_p, plan, dy, n_nano: int, lr: float, pipelined: bool = True, comm: bool = True):
        """Forward, backward and isolated SGD on this rank's shard.  Returns
        (Y, dX_p).  With ``pipelined`` the nano-batch all-reduces of Y overlap
        the following nano-batches AND the backward: dY is the upstream
        gradient, so the backward needs only the (small) all-reduced Z; the
        Y all-reduces are waited for at the end of the step."""
        y, ctx, works, hz = self.forward_async(x_p, plan, n_nano, pipelined, comm, defer_finish=True)
        if hz is not None:
            hz.wait()  # dB = dY^T Z needs the summed Z

        def after_dz():
            # the peer all-reduce's last finish (HBM-bound) runs beside the
            # tensor-bound dX mainloop rather than beside the HBM-bound dZ pass
            for w in works:
                if isinstance(w, _PeerFinish):
                    w.launch()

        with _Range("mlora.backward"):
            dx_p, dA_p, dB = self.backward(ctx, x_p, dy, overlapped=bool(works), after_dz=after_dz)
        with _Range("mlora.sgd"):
            self.compute.sgd(self, plan, dA_p, dB, lr)
        self._mark("sgd")
        for w in works:
            w.wait()
        self._mark("end")
        return y, dx_p


class _PeerFinish:
    """Work handle of the peer all-reduce: the last nano-batch's finish and
    the completion wait, queued on the layer's side stream by ``launch()``
    (after the work queued so far on the current stream), and ``wait()``,
    which launches them if that has not happened and makes the current stream
    wait for them (as an NCCL work handle's wait() does for its collective)."""

    def __init__(self, layer: "ShardedLayer", ar, rng, index: int, device):
        self.layer, self.ar, self.rng, self.index, self.device = layer, ar, rng, index, device
        self.done = None

    def launch(self):
        if self.done is not None:
            return
        L, side = self.layer, self.layer._side
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        side.wait_event(ev)
        self.ar.finish(self.rng[0], self.rng[1], side)
        L._mark(f"finish{self.index}", side)
        self.ar.wait(side)
        L._mark("ar_wait", side)
        self.done = torch.cuda.Event()
        self.done.record(side)
        L._last_done = self.done
        if L._pending is self:
            L._pending = None

    def wait(self):
        self.launch()
        torch.cuda.current_stream(self.device).wait_event(self.done)


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


def _timed_med(fn, iters: int, device, reps: int = 3) -> float:
    """Median of ``reps`` _timed measurements: the collectives' speed varies
    from one measurement to the next on a shared node."""
    return float(statistics.median(_timed(fn, iters, device) for _ in range(reps)))


def _job_parallel(args, rank, world, dev, metric, unit):
    """Weak scaling without any collective on the data path: every rank trains
    its own set of jobs (same layer shape, its own adapters and rows, seeded
    by rank) on its own replica of the frozen backbone.  Returns the per-step
    device time (max over ranks) of the timed region and the e2e time."""
    from . import _lib, workloads
    from .nano import AIMDController  # noqa: F401  (kept for symmetry of imports)

    sp = workloads.spec(args.workload, rows_scale=getattr(args, "rows_scale", 1.0))
    sp.seed = sp.seed + 7919 * rank
    w = workloads.build(sp, device=dev)
    m = w.model
    x = w.x.requires_grad_(True)
    ids_host = w.ids.cpu()

    def step(xi=None):
        for ad in m.adapters.values():
            ad.A.grad = None
            ad.B.grad = None
        xx = x if xi is None else xi
        xx.grad = None
        y = m(xx, ids_host)
        y.backward(w.dy)
        m.sgd_step(sp.lr)

    for _ in range(max(3, args.warmup)):
        step()
    launches0 = _lib.launch_count()
    ms = _timed(step, args.steps, dev)
    launches = _lib.launch_count() - launches0
    # e2e: prefetched pinned H2D of this rank's X, probe read back every step
    # (waited for one step later; the last one before the closing event)
    x_host = w.x.detach().cpu().pin_memory()
    bufs = [torch.empty_like(w.x.detach()) for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    copy_stream = torch.cuda.Stream(dev)
    compute = torch.cuda.current_stream(dev)
    probes = [torch.empty(64, dtype=w.x.dtype).pin_memory() for _ in range(2)]
    read = [torch.cuda.Event() for _ in range(2)]
    a0 = m.adapters["0"].A
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
        step(bufs[i % 2].detach().requires_grad_(True))
        consumed[i % 2].record(compute)
        probes[i % 2].copy_(a0.detach()[0, :64], non_blocking=True)
        read[i % 2].record(compute)
        if i > 0:  # the previous step's result, one step late as a training loop logs it
            read[(i - 1) % 2].synchronize()

    for ev in consumed:
        ev.record(compute)
    issue_copy(0)
    e2e()
    e2e_ms = _timed(e2e, max(3, args.steps // 2), dev)
    torch.cuda.synchronize(dev)
    out = {"sp": sp, "ms": ms, "e2e_ms": e2e_ms, "launches": launches,
           "h2d": int(w.x.numel() * w.x.element_size()), "d2h": int(probes[0].numel() * probes[0].element_size())}
    del w, m, x, bufs
    torch.cuda.empty_cache()
    return out


def bench_multi(args, peaks_d, peaks_kind, metric, unit):
    """bench.py --gpus N (N > 1).  Primary value: job-parallel weak scaling
    (the jobs are independent and the backbone is frozen, so no collective
    is needed).  Also measured in the same run and reported as `ksharded`:
    one layer K-sharded across the ranks with the nano-batch all-reduce
    overlap steered by AIMD (the rebuilt phase6 pipeline)."""
    import datetime

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    comm_sms = int(os.environ.get("MLORA_COMM_SMS", "16"))
    if os.environ.get("MLORA_NCCL_CHANNELS"):
        os.environ.setdefault("NCCL_MAX_NCHANNELS", os.environ["MLORA_NCCL_CHANNELS"])
        os.environ.setdefault("NCCL_MIN_NCHANNELS", os.environ["MLORA_NCCL_CHANNELS"])
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        jp = _job_parallel(args, rank, world, dev, metric, unit)
        ks = _ksharded(args, rank, world, dev, comm_sms, peaks_d)
        if rank != 0:
            return None
        sp = jp["sp"]
        ms = jp["ms"]
        step_flops = sp.flops() * world
        return {
            "metric": metric, "value": round(world * sp.rows / (ms / 1000.0), 1), "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded per rank; random-init weights)",
            "config": {"workload": f"{sp.name}: fwd+bwd+isolated SGD d_in={sp.d_in} d_out={sp.d_out} per GPU, "
                                   "job-parallel (each GPU trains its own adapters on a frozen-backbone replica)",
                       "rows": sp.rows * world, "global_batch": sp.rows * world, "seq_len": None,
                       "parallelism": f"job-parallel x{world} (no collective on the data path)",
                       "l2": "inputs larger than L2 (X 512 MiB per GPU)"},
            "step_tflops": round(step_flops / (ms / 1000.0) / 1e12, 1),
            "e2e": {"value": round(world * sp.rows / (jp["e2e_ms"] / 1000.0), 1), "unit": unit,
                    "ms_per_step": round(jp["e2e_ms"], 3), "h2d_bytes_per_step": jp["h2d"] * world,
                    "d2h_bytes_per_step": jp["d2h"] * world},
            "gpu_launches": int(jp["launches"]),
            "ksharded": ks,
        }
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _one_timeline(layer: ShardedLayer, step, device) -> dict:
    """One step with the layer's phase timeline on: milliseconds from the
    step's start to the end of each phase on this rank."""
    torch.cuda.synchronize(device)
    layer.timeline = []
    try:
        step()
        try:
            return layer.timeline_ms()
        except Exception as e:  # a timing record only: never fail the bench over it
            return {"error": f"{type(e).__name__}: {e}"[:200]}
    finally:
        layer.timeline = None


def _ksharded(args, rank, world, dev, comm_sms, peaks_d=None):
    """The K-sharded layer with the nano-batch all-reduce pipeline: AIMD over
    the nano-batch count, the SM reservation sweep, overlap accounting, timed
    steps and the prefetched e2e loop.  Returns the summary (rank 0)."""
    from . import _lib, workloads

    sp = workloads.spec(getattr(args, "ksharded_workload", "c3"), rows_scale=getattr(args, "rows_scale", 1.0))
    w = workloads.build(sp, device=dev)
    bwd_group = dist.new_group(list(range(world)))
    layer = ShardedLayer(w.model, rank, world, compute=NativeCompute(comm_sms=comm_sms), bwd_group=bwd_group)
    x_p = layer.shard_input(w.x)
    plan = ops.route(w.ids.cpu(), layer.table, dev)
    lr = sp.lr
    dy = w.dy
    n_tiles = (sp.rows + TILE_ROWS - 1) // TILE_ROWS

    def stepper(n, pipelined=True, comm=True):
        return lambda: layer.step(x_p, plan, dy, n, lr, pipelined, comm)

    for _ in range(max(3, args.warmup)):
        stepper(4)()
    torch.cuda.synchronize(dev)

    # fixed nano-batch counts (the multi-GPU configuration's sweep N = 1, 2, 4, 8, 16)
    n_sweep = {}
    for n in (1, 2, 4, 8, 16):
        if n <= n_tiles:
            n_sweep[n] = _timed_med(stepper(n), 3, dev)

    # AIMD over the real pipelined step (phase6b_real_aimd.py:245-302)
    ctl = AIMDController(start_n=1, alpha=4, beta=0.5, tau_ms=0.05, max_n=min(32, n_tiles))
    horizons = []
    for _ in range(8):
        n = ctl.n
        t = _timed(stepper(n), 3, dev)
        nxt, why = ctl.observe(t)
        horizons.append({"n": n, "ms": round(t, 4), "decision": why, "next_n": nxt})
    best_n = ctl.best_n

    sm_sweep = {}
    for k in sorted({0, comm_sms // 2, comm_sms, comm_sms + comm_sms // 2}):
        layer.compute.comm_sms = k
        sm_sweep[k] = _timed_med(stepper(best_n), 3, dev)
    best_k = min(sm_sweep, key=sm_sweep.get)
    layer.compute.comm_sms = best_k

    t_pipe = _timed_med(stepper(best_n), 3, dev)
    t_serial = _timed_med(stepper(best_n, pipelined=False), 3, dev)
    t_compute = _timed_med(stepper(best_n, comm=False), 3, dev)
    y_buf, ctx = layer.forward(x_p, plan, best_n)
    t_comm = _timed_med(lambda: comm_only(layer, y_buf, ctx["z"], n_tiles, best_n), 3, dev)
    hidden = 1.0 - max(0.0, t_pipe - t_compute) / t_comm if t_comm > 0 else 0.0
    ms = _timed_med(stepper(best_n), args.steps, dev)
    timeline = _one_timeline(layer, stepper(best_n), dev)

    # the same pipeline with the Y all-reduce issued from the forward epilogue
    # over peer memory (peer.PeerAllReduce) instead of NCCL
    peer_res = None
    if world > 1 and getattr(args, "ksharded_comm", "both") == "both":
        try:
            layer.comm = "peer"
            layer.compute.comm_sms = 0
            for _ in range(3):
                stepper(best_n)()
            torch.cuda.synchronize(dev)
            p_sweep = {n: _timed_med(stepper(n), 3, dev) for n in (1, 2, 4, 8, 16) if n <= n_tiles}
            pn = min(p_sweep, key=p_sweep.get)
            p_ms = _timed_med(stepper(pn), args.steps, dev)
            p_timeline = _one_timeline(layer, stepper(pn), dev)
            err = _lib.device_error()
            # roofline of the fused compute + collective step: the slower of the
            # rank's FLOPs at the measured sustained GEMM peak and the bytes each
            # GPU sends over NVLink in each direction (partials to the owners,
            # then the owners' sums: 2 (P-1)/P M d_out 2 bytes) at the measured
            # peer-copy bandwidth of 770 GB/s per direction
            peak_tf = float((peaks_d or {}).get("bf16_tflops_sustained", 1370.6))
            link_gbs = 770.0
            nvl_bytes = 2.0 * (world - 1) / world * sp.rows * sp.d_out * 2
            t_tc = sp.flops() / world / (peak_tf * 1e12) * 1e3
            t_nvl = nvl_bytes / (link_gbs * 1e9) * 1e3
            target = max(t_tc, t_nvl)
            peer_res = {"n": pn, "value": round(sp.rows / (p_ms / 1000.0), 1), "ms_per_step": round(p_ms, 4),
                        "roofline": {"bound": "tensor" if t_tc >= t_nvl else "nvlink", "target_ms": round(target, 4),
                                     "tensor_ms": round(t_tc, 4), "nvlink_ms": round(t_nvl, 4),
                                     "nvlink_bytes_per_direction": int(nvl_bytes), "frac": round(target / p_ms, 4),
                                     "peaks": f"{peak_tf} TFLOP/s bf16 sustained (measured), {link_gbs} GB/s "
                                              "peer copy per direction (measured on the pool)"},
                        "step_tflops": round(sp.flops() / (p_ms / 1000.0) / 1e12, 1),
                        "exposed_over_compute_ms": round(p_ms - t_compute, 4),
                        "n_sweep_ms": {str(k): round(v, 4) for k, v in p_sweep.items()},
                        "timeline_ms": p_timeline,
                        "device_error": int(err)}
        except Exception as e:  # reported beside the NCCL numbers, which stand
            peer_res = {"error": f"{type(e).__name__}: {e}"[:300]}
        finally:
            layer.comm = "nccl"
            layer.compute.comm_sms = best_k
            layer.close()
    del w
    if rank != 0:
        return None
    peak_tf = float((peaks_d or {}).get("bf16_tflops_sustained", 1370.6))
    t_tc = sp.flops() / world / (peak_tf * 1e12) * 1e3
    return {"value": round(sp.rows / (ms / 1000.0), 1), "ms_per_step": round(ms, 4), "scaling": "strong",
            "tensor_bound_ms": round(t_tc, 4), "frac_of_tensor_bound": round(t_tc / ms, 4),
            "workload": f"{sp.name} one layer, backbone K-sharded over {world} GPUs",
            "rows": sp.rows, "step_tflops": round(sp.flops() / (ms / 1000.0) / 1e12, 1),
            "overlap": {"n": best_n, "comm_sms": best_k, "nccl_channels": os.environ.get("NCCL_MAX_NCHANNELS"),
                        "comm_sms_sweep_ms": {str(k): round(v, 4) for k, v in sm_sweep.items()},
                        "pipelined_ms": round(t_pipe, 4), "serial_ms": round(t_serial, 4),
                        "compute_only_ms": round(t_compute, 4), "comm_only_ms": round(t_comm, 4),
                        "comm_hidden_frac": round(hidden, 4)},
            "n_sweep_ms": {str(k): round(v, 4) for k, v in n_sweep.items()},
            "aimd": horizons,
            "timeline_ms": timeline,
            "peer_allreduce": peer_res}
