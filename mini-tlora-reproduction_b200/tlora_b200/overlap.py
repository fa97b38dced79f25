"""K-sharded multi-LoRA layer across the ranks of one node, with the
nano-batch compute / all-reduce overlap steered by AIMD.

Rebuild of phase6_two_gpu_overlap.py (split_ranges :73-87, run_serial
:220-244, run_pipelined :247-280, measure_distributed :283-343) and
phase6b_real_aimd.py (controller loop :245-302) for 1-8 GPUs, with the
semantics the reference's microbenchmark leaves out: the ranks hold shards of
ONE layer instead of unrelated replicas.

Partitioning (rank p of P): columns [k0, k1) of d_in.  Rank p holds
W[:, k0:k1], A_pack[:, k0:k1] and X[:, k0:k1]; B_pack is replicated.  Its
forward partial is Y_p = X_p W_p^T (+ bias and the LoRA expand on the rank
that owns them for the nano-batch), Z_p = s X_p A_p^T; since both are linear
in X_p, sum_p Y_p = Y and sum_p Z_p = Z.  Per step:

  1. shrink: Z_p over all tiles, then an async SUM all-reduce of Z (small:
     256 x 64 bf16 per tile x rank chunk);
  2. for each of N nano-batches (N near-equal ranges of 256-row plan tiles):
     the fused mainloop over its tiles, then the SUM all-reduce of its rows of
     Y, which overlaps the next nano-batch's mainloop.  Nano-batch i's bias
     and LoRA expand are added by rank i % P only, so that the P ranks share
     that work and every other rank starts its mainloops without waiting for
     the Z all-reduce;
  3. backward with the replicated dY, overlapping the Y all-reduces still in
     flight: dZ = s dY B is split by tiles and dB = dY^T Z by 128-row blocks
     of d_out across the ranks, each summed with an async all-reduce on a
     second communicator (so it does not queue behind the Y traffic); dB's
     runs beside the dX mainloop.  dX_p = dY W_p + dZ A_p and dA_p = dZ^T X_p
     are local; then the isolated SGD step.

With one rank there is no collective at all: the same pipeline runs the whole
layer (the one-GPU point of the scaling curve).

Nano-batch boundaries are rounded to 256-row plan tiles (the reference splits rows
exactly); N still counts nano-batches.

The Y all-reduce of step 2 has three implementations (``ShardedLayer.comm``):
"nccl" (an async SUM all-reduce per nano-batch on NCCL's stream, as the
reference), "peer" (peer.PeerAllReduce: the mainloop's epilogue writes each
partial tile straight into its owner rank's receive buffer over NVLink, and a
small owner kernel on a side stream adds the partials of its tiles and writes
the sums into every rank's Y while the next nano-batch's mainloop runs) and
"mc" (peer.MulticastAllReduce: the mainloop writes the partial rows into a
buffer bound to an NVLink multicast object, and a kernel on a side stream sums
each rank's share of the rows in the switch with multimem.ld_reduce and writes
the sums into every rank's Y with multimem.st).  The peer and mc paths need a
routing plan that keeps the rows in their order (adapter-sorted ids), and
their Y is the all-reduce buffer, overwritten by the layer's next forward.
"""

from __future__ import annotations

from typing import Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist

from . import _lib, ops, peer
from ._lib import TILE_ROWS
from .nano import ramp_ranges, split_ranges

COMMS = ("nccl", "peer", "mc")


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
    """The native kernels (tcgen05 for bf16) behind the sharded layer.  The
    isolated SGD step of A (and, with one rank, of B) is fused into the
    gradient reduction's epilogue (``fused_sgd``).  The
    staged forward / backward objects (call arguments, buffers, the routing
    plan kept resident in a device workspace) are built once per input
    buffer and plan and reused by every later step, so a step's host work is
    the kernel launches.  ``comm_sms`` SMs can be left out of the mainloops
    that run beside the all-reduces; the kernels hand out work items
    dynamically, so CTAs that find their SM taken simply start later and take
    fewer items, and 0 (no reservation) is the measured best on B200."""

    fused_sgd = True

    def __init__(self, impl: str = "auto", comm_sms: int = 0):
        self.impl = impl
        self.comm_sms = int(comm_sms)
        self._sms = None
        self._fw = None
        self._bw = None

    def _main_ctas(self, device):
        if self.comm_sms <= 0:
            return 0
        if self._sms is None:
            self._sms = torch.cuda.get_device_properties(device).multi_processor_count
        return max(1, self._sms - self.comm_sms)

    def begin(self, layer, x_p, plan, y=None):
        # keyed by everything but X itself: a step on another input buffer of
        # the same shape reuses the objects with the new X
        key = (tuple(x_p.shape), x_p.dtype, id(plan), None if y is None else y.data_ptr(),
               layer.A_pack.data_ptr(), id(layer.err_word))
        c = self._fw
        if c is not None and c["key"] == key:
            c["fw"].rebind(x_p)
            return c
        self._bw = None
        st = ops.LayerState(layer.table, layer.scaling, plan, layer.A_pack, layer.B_pack, self.impl,
                            err_word=layer.err_word)
        ops.make_resident(st, x_p.shape[0], x_p.shape[1], layer.B_pack.shape[0], x_p.dtype, x_p.device)
        fw = ops.StagedForward(x_p, layer.W, layer.bias, st, y=y)
        zbytes = fw.args.sizes()[0]
        zview = fw.z[:zbytes].view(x_p.dtype) if zbytes else None
        # the plan object is held so that its id() stays unique while cached
        self._fw = {"key": key, "plan": plan, "fw": fw, "st": st, "z": zview, "y": fw.y, "n_tiles": fw.n_tiles}
        return self._fw

    def shrink(self, ctx):
        ctx["fw"].shrink()

    def shrink_main(self, ctx):
        ctx["fw"].shrink_main()

    def main(self, ctx, t0, t1, expand, add_bias):
        ctx["fw"].main(t0, t1, expand=expand, add_bias=add_bias, max_ctas=self._main_ctas(ctx["fw"].x.device))

    def push(self, ctx, ar, t0, t1, expand, add_bias):
        ctx["fw"].push(ar, t0, t1, expand=expand, add_bias=add_bias)

    def bwd_begin(self, ctx, layer, x_p, dy, overlapped=False, partial=True):
        """The staged backward of this forward; ``partial``: dZ and dB are
        written only in part (a rank's share) and summed across the ranks, so
        they start at zero."""
        max_ctas = self._main_ctas(x_p.device) if overlapped else 0
        c = self._bw
        if c is None or c["max_ctas"] != max_ctas or c["dy_shape"] != tuple(dy.shape):
            st = ctx["st"]
            st = ops.LayerState(st.table, st.scaling, st.plan, st.A_pack, st.B_pack, st.impl, max_ctas,
                                err_word=st.err_word)
            bw = ops.StagedBackward(dy, x_p, layer.W, ctx["fw"].z, st)
            c = self._bw = {"bw": bw, "max_ctas": max_ctas, "dy_shape": tuple(dy.shape), "dz": bw.dz_view(),
                            "dx": bw.dx, "dA": bw.dA, "dB": bw.dB, "n_tiles": bw.n_tiles, "n_db": bw.n_db}
        c["bw"].rebind(dy, x_p, ctx["fw"].z)
        if partial:
            c["bw"].zero_partials()
        return c

    def bwd_dz(self, b, t0, t1):
        b["bw"].run_dz(t0, t1)

    def bwd_dx(self, b):
        b["bw"].run_dx()

    def bwd_da(self, b, sgd_lr=None):
        if sgd_lr is None:
            b["bw"].run_da()
        else:
            b["bw"].run_da_sgd(sgd_lr)

    def bwd_db(self, b, b0, b1):
        b["bw"].run_db(b0, b1)

    def bwd_dadb(self, b):
        b["bw"].run_dadb()

    def bwd_all(self, b, sgd_lr=None):
        b["bw"].run_all(sgd_lr)

    def sgd(self, layer, plan, dA_p, dB, lr, which=("A", "B")):
        """Isolated SGD of the plan's active adapters (their A and / or B, as
        ``which`` lists), one launch; the item list (pointers into the layer's
        weights and the reused gradient buffers) is built once per plan and
        buffers."""
        which = tuple(which)
        if not which:
            return 0
        key = (id(plan), which, layer.A_pack.data_ptr(), layer.B_pack.data_ptr(), dA_p.data_ptr(), dB.data_ptr())
        c = getattr(self, "_sgd", None)
        if c is None or c[0] != key:
            pairs = []
            for i in range(layer.table.n):
                if not plan.active[i]:
                    continue
                o, r = int(layer.table.pack_off[i]), int(layer.table.rank[i])
                if "A" in which:
                    pairs.append((layer.A_pack[o:o + r], dA_p[o:o + r]))
                if "B" in which:
                    pairs.append((layer.B_pack[:, o:o + r], dB[:, o:o + r]))
            c = self._sgd = (key, ops.SgdItems(pairs), plan)
        return c[1].step(lr)


class ShardedLayer:
    """Rank ``rank``'s K-shard of a MultiLoRALinear (see module docstring).

    ``err_word``: an optional CUDA int32 tensor that receives the device-side
    flags of every kernel the layer launches (bounds bit 0, timeout bit 1);
    by default they go to the library-wide word.  ``check()`` reads the word
    (a device synchronisation) and raises if a flag is set, e.g. when an
    all-reduce wait ran out and rows of Y hold no sum."""

    def __init__(self, model, rank: int, world: int, compute=None, group=None, bwd_group=None,
                 comm: str = "nccl", err_word: Optional[torch.Tensor] = None, dz: str = "split"):
        # `bwd_group`: a second communicator for the backward's small
        # all-reduces (dZ, dB), so they do not queue behind the large Y
        # all-reduces still in flight on `group`.
        # `dz`: "split" = each rank computes dZ = s dY B for its share of the
        # tiles and the shares are summed with an all-reduce; "replicated" =
        # every rank computes all of dZ (dY and B_pack are replicated), no
        # all-reduce
        if comm not in COMMS:
            raise ValueError(f"comm must be one of {COMMS}, not {comm!r}")
        if dz not in ("split", "replicated"):
            raise ValueError(f"dz must be 'split' or 'replicated', not {dz!r}")
        self.dz = dz
        # nano-batch ranges over the plan tiles: "even" (the reference's
        # split_ranges) or "ramp" (the first nano-batch half as long, so that
        # the all-reduce chain starts earlier)
        self.split = "even"
        self.rank, self.world, self.group = rank, world, group
        self.comm = comm
        self.err_word = err_word
        self._ar = None  # peer.PeerAllReduce of the "peer" path
        self._mc = None  # peer.MulticastAllReduce of the "mc" path
        self._side = None
        self._one = None
        self._last_done = None
        self._pending = None  # the peer / mc all-reduce's last stage, until launched
        # set to a list to record a timeline of the next steps: (phase, CUDA
        # event on the stream that runs it); read with timeline_ms()
        self.timeline = None
        # gradients of the last step() (views of reused buffers)
        self.last_grads = None
        self.bwd_group = bwd_group if bwd_group is not None else group
        A_pack, B_pack, table = model.packed()
        d_in = model.base.in_features
        self.k0, self.k1 = shard_columns(d_in, rank, world)
        with torch.no_grad():
            # copies (also with one rank, where the slice is the whole tensor):
            # the layer's SGD steps update its own adapter shards, not the model's
            self.W = model.base.weight[:, self.k0:self.k1].clone(memory_format=torch.contiguous_format)
            self.A_pack = A_pack[:, self.k0:self.k1].clone(memory_format=torch.contiguous_format)
            self.B_pack = B_pack.clone()
            # every rank keeps the bias: the rank that owns a nano-batch adds it
            self.bias = model.base.bias.detach().clone() if model.base.bias is not None else None
        self.table = table
        self.scaling = np.array([float(a.scaling) for a in model.adapters.values()], dtype=np.float32)
        self.compute = compute or NativeCompute(getattr(model, "impl", "auto"))

    # -- bookkeeping -----------------------------------------------------------
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

    def ranges(self, n_tiles: int, n_nano: int):
        """The nano-batches' plan-tile ranges (see ``split``; "ramp:<f>" sets
        the first nano-batch's length relative to the others, 0.5 for
        "ramp")."""
        if self.split == "even":
            return split_ranges(n_tiles, n_nano)
        if self.split == "ramp" or self.split.startswith("ramp:"):
            first = float(self.split[5:]) if ":" in self.split else 0.5
            if not first > 0:
                raise ValueError(f"the first nano-batch's relative length must be > 0: {self.split!r}")
            return ramp_ranges(n_tiles, n_nano, first)
        raise ValueError(f"split must be 'even', 'ramp' or 'ramp:<fraction>', not {self.split!r}")

    def check(self) -> None:
        """Raise if a kernel of this layer flagged a device-side check (reads
        the status word: a device synchronisation)."""
        if self.err_word is not None:
            v = int(self.err_word.item())
        else:
            torch.cuda.synchronize()
            v = _lib.device_error()
        if v:
            what = " and ".join(n for b, n in ((1, "a bounds check fired"), (2, "a bounded wait timed out")) if v & b)
            raise RuntimeError(f"K-sharded layer, rank {self.rank}: {what} (status word {v}); "
                               "rows of Y or the gradients may be incomplete")

    def shard_input(self, x: torch.Tensor) -> torch.Tensor:
        return x[:, self.k0:self.k1].contiguous()

    def _collective(self, comm: bool) -> bool:
        return comm and self.world > 1

    def _owner(self, i: int) -> bool:
        """This rank adds nano-batch i's bias and LoRA expand."""
        return i % self.world == self.rank

    # -- forward ---------------------------------------------------------------
    def forward(self, x_p, plan, n_nano: int, pipelined: bool = True, comm: bool = True):
        """Pipelined forward; returns (Y, ctx) with every collective complete.
        ``comm=False`` skips the collectives (compute-only timing).  Y is a
        buffer of the layer, overwritten by its next forward."""
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
        peer or mc all-reduce and ``defer_finish``, the last nano-batch's
        all-reduce is launched by the returned handle's ``launch()`` (or its
        ``wait()``), so that the caller can queue it beside work of its
        choice."""
        if self._collective(comm) and pipelined and self.comm in ("peer", "mc"):
            return self._forward_device_ar(x_p, plan, n_nano, defer_finish)
        c = self.compute
        collective = self._collective(comm)
        self._mark("start")
        ctx = c.begin(self, x_p, plan)
        if self.world == 1 and n_nano <= 1 and hasattr(c, "shrink_main"):
            # one rank, one nano-batch: the shrink and the mainloop in one call
            with _Range("mlora.forward"):
                c.shrink_main(ctx)
            self._mark("main0")
            return ctx["y"], ctx, [], None
        with _Range("mlora.shrink"):
            c.shrink(ctx)
        self._mark("shrink")
        hz = None
        if collective and ctx["z"] is not None:
            hz = dist.all_reduce(ctx["z"], op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        rows = x_p.shape[0]
        works = []
        for i, (t0, t1) in enumerate(self.ranges(ctx["n_tiles"], n_nano)):
            own = self._owner(i)
            if own and hz is not None:
                hz.wait()  # the expand reads the summed Z
                hz = None
            with _Range(f"mlora.nano{i}"):
                c.main(ctx, t0, t1, expand=own, add_bias=own)
                self._mark(f"main{i}")
                if not collective:
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
            if self.err_word is not None:
                self._ar.set_err_word(self.err_word)
            self._one = torch.zeros(1, dtype=torch.float32, device=device)
            self._side = torch.cuda.Stream(device)
        return self._ar

    def mc_buffers(self, rows: int, dtype, device) -> "peer.MulticastAllReduce":
        """This rank's multicast all-reduce buffers for ``rows`` rows
        (collective on first use or when the row count or dtype changes)."""
        if self._mc is None or self._mc.rows != rows or self._mc.dtype != dtype:
            self.close()
            self._mc = peer.MulticastAllReduce(rows, self.B_pack.shape[0], dtype, device, self.group)
            if self.err_word is not None:
                self._mc.set_err_word(self.err_word)
            self._side = torch.cuda.Stream(device)
        return self._mc

    def _forward_device_ar(self, x_p, plan, n_nano: int, defer_finish: bool = False):
        """forward_async with the Y all-reduce done by this library's kernels
        (the peer path: pushes from the epilogue and owner finishes; the mc
        path: switch reductions of each nano-batch's rows).  The returned work
        handle makes the caller's stream wait until every row of Y holds the
        sum.  Y is the all-reduce buffer, overwritten by the next forward."""
        if plan.perm is not None:
            raise ValueError("the peer and mc all-reduces need a routing plan that keeps the row order")
        c = self.compute
        dev = x_p.device
        rows = x_p.shape[0]
        mc = self.comm == "mc"
        ar = self.mc_buffers(rows, x_p.dtype, dev) if mc else self.peer_buffers(rows, x_p.dtype, dev)
        if self._pending is not None:
            self._pending.launch()  # a previous call's deferred stage that nobody launched
        cur = torch.cuda.current_stream(dev)
        if self._last_done is not None:
            cur.wait_event(self._last_done)  # this rank's previous call is finished with the buffers
        self._mark("start")
        if not mc:
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
        side = self._side
        ranges = self.ranges(ctx["n_tiles"], n_nano)
        for i, (t0, t1) in enumerate(ranges):
            own = self._owner(i)
            if own and hz is not None:
                hz.wait()
                hz = None
            with _Range(f"mlora.nano{i}"):
                if mc:
                    c.main(ctx, t0, t1, expand=own, add_bias=own)
                    self._mark(f"main{i}", cur)
                else:
                    c.push(ctx, ar, t0, t1, expand=own, add_bias=own)
                    self._mark(f"push{i}", cur)
                if i + 1 < len(ranges):
                    ev = torch.cuda.Event()
                    ev.record(cur)
                    side.wait_event(ev)
                    if mc:
                        ar.reduce(t0 * TILE_ROWS, min(t1 * TILE_ROWS, rows), i, side)
                        self._mark(f"reduce{i}", side)
                    else:
                        ar.finish(t0, t1, side)
                        self._mark(f"finish{i}", side)
        last = _DeviceArStage(self, ar, ranges, dev, mc)
        self._pending = last
        if not defer_finish:
            last.launch()
        return ar.y, ctx, [last], hz

    def close(self) -> None:
        """Release the peer / multicast buffers (collective: every rank calls
        it after its device work; each rank unmaps its peers' buffers before
        any rank frees its own)."""
        if self._ar is not None:
            torch.cuda.synchronize(self._ar.device)
            dist.barrier(group=self.group)
            self._ar.close_peers()
            dist.barrier(group=self.group)
            self._ar.close()
            self._ar = None
        if self._mc is not None:
            self._mc.close()
            self._mc = None
        self._last_done = None
        self._pending = None

    # -- backward and the step ---------------------------------------------------
    def backward(self, ctx, x_p, dy, overlapped=False, after_dz=None, lr=None):
        """Backward on this rank's shard.  dZ (needs all of dY and B) and dB
        (needs all of dY and Z) are split across ranks — dZ by tiles, dB by
        128-row blocks of d_out — and summed with two small async all-reduces:
        dZ's runs beside this rank's dB share, dB's beside the dX mainloop.
        dX_p and dA_p are local.  With ``lr`` and a compute that fuses the SGD
        step, the reductions also update the weights whose gradients are
        complete on this rank (A_p; with one rank also B).  Returns (dX_p,
        dA_p, dB, dB work handle or None: wait for it before reading dB, the
        weights already updated: a subset of {"A", "B"})."""
        c = self.compute
        coll = self.world > 1
        fused = lr if (lr is not None and getattr(c, "fused_sgd", False)) else None
        b = c.bwd_begin(ctx, self, x_p, dy, overlapped, partial=coll)
        if not coll:
            if after_dz is not None:
                after_dz()
            if hasattr(c, "bwd_all"):
                # dZ, dX (overlapping dZ's tail), dA and dB in one call, the
                # SGD step in the reduction's epilogue
                c.bwd_all(b, sgd_lr=fused)
                applied = ("A", "B") if fused is not None else ()
            else:
                c.bwd_dz(b, 0, b["n_tiles"])
                c.bwd_dx(b)
                c.bwd_dadb(b)
                applied = ()
            self._mark("bwd")
            return b["dx"], b["dA"], b["dB"], None, applied
        hdz = None
        if self.dz == "replicated":
            c.bwd_dz(b, 0, b["n_tiles"])
            self._mark("bwd_dz")
        else:
            t0, t1 = _share(b["n_tiles"], self.rank, self.world)
            c.bwd_dz(b, t0, t1)
            self._mark("bwd_dz")
            if b["dz"] is not None:
                hdz = dist.all_reduce(b["dz"], op=dist.ReduceOp.SUM, group=self.bwd_group, async_op=True)
        b0, b1 = _share(b["n_db"], self.rank, self.world)
        c.bwd_db(b, b0, b1)  # reads Z and dY only: runs while dZ is being summed
        hdb = dist.all_reduce(b["dB"], op=dist.ReduceOp.SUM, group=self.bwd_group, async_op=True)
        self._mark("bwd_db")
        if hdz is not None:
            hdz.wait()
        self._mark("bwd_dz_allreduce")
        if after_dz is not None:
            after_dz()
        c.bwd_dx(b)
        self._mark("bwd_dx")
        if fused is not None:
            c.bwd_da(b, sgd_lr=fused)  # dA_p is complete on this rank: its SGD step in the epilogue
            applied = ("A",)
        else:
            c.bwd_da(b)
            applied = ()
        self._mark("bwd_da")
        return b["dx"], b["dA"], b["dB"], hdb, applied

    def step(self, x_p, plan, dy, n_nano: int, lr: float, pipelined: bool = True, comm: bool = True):
        """Forward, backward and isolated SGD on this rank's shard.  Returns
        (Y, dX_p).  With ``pipelined`` the nano-batch all-reduces of Y overlap
        the following nano-batches AND the backward: dY is the upstream
        gradient, so the backward needs only the (small) all-reduced Z; the
        Y all-reduces are waited for at the end of the step.  The gradients
        (dA_p, dB) stay in ``last_grads`` until the next step."""
        y, ctx, works, hz = self.forward_async(x_p, plan, n_nano, pipelined, comm, defer_finish=True)
        if hz is not None:
            hz.wait()  # dB = dY^T Z needs the summed Z

        def after_dz():
            # the device all-reduce's last stage runs beside the tensor-bound
            # dX mainloop rather than beside the HBM-bound dZ pass
            for w in works:
                if isinstance(w, _DeviceArStage):
                    w.launch()

        with _Range("mlora.backward"):
            dx_p, dA_p, dB, hdb, applied = self.backward(ctx, x_p, dy, overlapped=bool(works), after_dz=after_dz,
                                                         lr=lr)
        if hdb is not None:
            hdb.wait()
        self._mark("bwd_db_allreduce")
        rest = tuple(w for w in ("A", "B") if w not in applied)
        if rest:
            with _Range("mlora.sgd"):
                self.compute.sgd(self, plan, dA_p, dB, lr, which=rest)
            self._mark("sgd")
        for w in works:
            w.wait()
        self._mark("end")
        self.last_grads = (dA_p, dB)
        return y, dx_p


class _DeviceArStage:
    """Work handle of the peer / mc all-reduce: the last nano-batch's finish
    (or switch reduction) and the completion wait, queued on the layer's side
    stream by ``launch()`` (after the work queued so far on the current
    stream), and ``wait()``, which launches them if that has not happened and
    makes the current stream wait for them (as an NCCL work handle's wait()
    does for its collective)."""

    def __init__(self, layer: "ShardedLayer", ar, ranges, device, mc: bool):
        self.layer, self.ar, self.ranges, self.device, self.mc = layer, ar, ranges, device, mc
        self.done = None

    def launch(self):
        if self.done is not None:
            return
        L, side = self.layer, self.layer._side
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        side.wait_event(ev)
        i = len(self.ranges) - 1
        t0, t1 = self.ranges[-1]
        if self.mc:
            self.ar.reduce(t0 * TILE_ROWS, min(t1 * TILE_ROWS, self.ar.rows), i, side)
            L._mark(f"reduce{i}", side)
            self.ar.wait(len(self.ranges), side)
        else:
            self.ar.finish(t0, t1, side)
            L._mark(f"finish{i}", side)
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
    """The step's forward collectives alone, through the layer's all-reduce
    path (for the overlap fraction): the Z all-reduce and one Y all-reduce
    per nano-batch.  The peer path's all-reduce lives in the mainloop's
    epilogue and cannot run without it, so it is timed as NCCL's."""
    works = []
    if z is not None:
        works.append(dist.all_reduce(z, op=dist.ReduceOp.SUM, group=layer.group, async_op=True))
    rows = y.shape[0]
    ranges = layer.ranges(n_tiles, n_nano)
    if layer.comm == "mc" and layer._mc is not None and y.data_ptr() == layer._mc.y.data_ptr():
        mc = layer._mc
        cur = torch.cuda.current_stream(y.device)
        for i, (t0, t1) in enumerate(ranges):
            mc.reduce(t0 * TILE_ROWS, min(t1 * TILE_ROWS, rows), i, cur)
        mc.wait(len(ranges), cur)
    else:
        for t0, t1 in ranges:
            seg = y[t0 * TILE_ROWS:min(t1 * TILE_ROWS, rows)]
            works.append(dist.all_reduce(seg, op=dist.ReduceOp.SUM, group=layer.group, async_op=True))
    for w in works:
        w.wait()


class GraphedShardedStep:
    """CUDA-graph replay of ``ShardedLayer.step`` for fixed routing, input
    buffers and nano-batch count: every kernel, every all-reduce (NCCL's
    collectives, or the peer / multicast kernels on their side stream) and
    the stream forks and joins of one step are captured once and replayed with
    one launch, so a step costs no host work.  Every rank of the layer's group
    builds its graph at the same point (capture runs one eager step on each
    rank first).  ``x_p`` and ``dy`` are the graph's input buffers: copy new
    inputs into them before a replay; Y, dX_p and the gradients live in the
    layer's buffers and are overwritten by the next replay."""

    def __init__(self, layer: "ShardedLayer", x_p, plan, dy, n_nano: int, lr: float, warmup: int = 2,
                 pipelined: bool = True, comm: bool = True):
        dev = x_p.device
        self.layer, self.x, self.plan, self.dy, self.n, self.lr = layer, x_p, plan, dy, int(n_nano), float(lr)
        kw = {"pipelined": pipelined, "comm": comm}
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # warm-up off the default stream, as capture requires
            for _ in range(max(1, warmup)):
                layer.step(x_p, plan, dy, self.n, self.lr, **kw)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        # the captured step must not wait on events recorded outside the capture
        layer._last_done = None
        layer._pending = None
        if layer.world > 1:
            dist.barrier(group=layer.group)
        self.graph = torch.cuda.CUDAGraph()
        launches0 = _lib.launch_count()
        # thread-local capture: other threads of the process (NCCL's watchdog)
        # keep making CUDA calls while this one captures
        with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            self.y, self.dx = layer.step(x_p, plan, dy, self.n, self.lr, **kw)
        self.kernels = _lib.launch_count() - launches0  # this library's kernels in one replay
        layer._last_done = None
        layer._pending = None
        self.grads = layer.last_grads
        # Every buffer the captured kernels and collectives read or write
        # must live as long as the graph, also after the layer replaces its
        # cached objects (a later step with comm off, other inputs or another
        # plan builds new call arguments, workspaces, gradient buffers and SGD
        # item lists; without these references the old ones would go back to
        # the allocator while the graph still points at them).  close() of the
        # layer releases the peer / multicast buffers and ends the graph's use.
        c = layer.compute
        self._keep = (getattr(c, "_fw", None), getattr(c, "_bw", None), getattr(c, "_sgd", None),
                      layer._one, layer._ar, layer._mc, layer._side, plan, x_p, dy)

    def __call__(self):
        """Replay one step on the current stream; returns (Y, dX_p)."""
        self.graph.replay()
        return self.y, self.dx
