"""One-GPU timing of the K-sharded forward with the peer all-reduce issued
from the epilogue (peer.PeerAllReduce), with ``--world`` ranks emulated on
one GPU: each emulated rank runs its K-shard's forward mainloop with the push
epilogue on the main stream, and the owners' finish kernels run on a side
stream, beside the next nano-batch's mainloops.  Every finish starts after
all the pushes it waits for, so no kernel waits on a kernel running beside it.

Prints one JSON line: per nano-batch count N, the device milliseconds of the
plain mainloops (writing a local Y, no all-reduce), of the pushes alone, of
pushes + finishes in sequence, and of pushes + finishes overlapped; and of one
finish of all tiles alone.  The emulated GPU does the work of every rank, so
the times are ``world`` times a rank's share.

    python -m tlora_b200.peer_bench --workload c3 --world 2 --rows-scale 1.0
"""
from __future__ import annotations

import argparse
import json

import torch

from . import _lib, ops, peer, workloads
from .nano import split_ranges
from .overlap import NativeCompute, ShardedLayer


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--workload", default="c3", choices=["c2", "c3", "c4"])
    p.add_argument("--world", type=int, default=2)
    p.add_argument("--rows-scale", type=float, default=1.0)
    p.add_argument("--nano", default="1,2,4", help="nano-batch counts to time")
    p.add_argument("--iters", type=int, default=10)
    args = p.parse_args()

    dev = torch.device("cuda")
    w = workloads.build(workloads.spec(args.workload, rows_scale=args.rows_scale), device=dev)
    world = args.world
    rows, d_out = w.x.shape[0], w.model.base.weight.shape[0]
    layers = [ShardedLayer(w.model, r, world, compute=NativeCompute("auto")) for r in range(world)]
    plan = ops.route(w.ids.cpu(), layers[0].table, dev)
    xs = [L.shard_input(w.x) for L in layers]
    ars = peer.PeerAllReduce.emulated(world, rows, d_out, w.x.dtype, dev)
    ctxs = [L.compute.begin(L, x, plan, y=ars[r].y) for r, (L, x) in enumerate(zip(layers, xs))]
    for L, c in zip(layers, ctxs):
        L.compute.shrink(c)
    n_tiles = ctxs[0]["n_tiles"]
    main_s = torch.cuda.current_stream()
    side = torch.cuda.Stream()

    ys = [torch.empty(rows, d_out, dtype=w.x.dtype, device=dev) for _ in range(world)]

    def run(n, mode):
        if mode == "main_only":
            for t0, t1 in split_ranges(n_tiles, n):
                for r, (L, c) in enumerate(zip(layers, ctxs)):
                    c["fw"].y = ys[r]
                    L.compute.main(c, t0, t1, expand=r == 0, add_bias=r == 0)
            return
        for a in ars:
            a.reset(main_s)
        for t0, t1 in split_ranges(n_tiles, n):
            for r, (L, c) in enumerate(zip(layers, ctxs)):
                L.compute.push(c, ars[r], t0, t1, expand=r == 0, add_bias=r == 0)
            if mode == "serial":
                for a in ars:
                    a.finish(t0, t1, main_s)
            elif mode == "overlap":
                ev = torch.cuda.Event()
                ev.record(main_s)
                side.wait_event(ev)
                for a in ars:
                    a.finish(t0, t1, side)
        if mode == "serial":
            for a in ars:
                a.wait(main_s)
        elif mode == "overlap":
            for a in ars:
                a.wait(side)
            ev = torch.cuda.Event()
            ev.record(side)
            main_s.wait_event(ev)

    def timed(fn, iters):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(main_s)
        for _ in range(iters):
            fn()
        e1.record(main_s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    _lib.clear_device_error()
    out = {"workload": f"{w.spec.name} rows={rows} d_out={d_out}, {world} ranks emulated on one GPU", "ms": {}}
    for n in (int(v) for v in args.nano.split(",")):
        out["ms"][str(n)] = {m: round(timed(lambda: run(n, m), args.iters), 4)
                             for m in ("main_only", "push_only", "serial", "overlap")}

    # one finish of all tiles by every rank, its pushes complete
    run(1, "push_only")
    torch.cuda.synchronize()

    def finish_all():
        for a in ars:
            a.finish(0, n_tiles, main_s)

    for a in ars:
        a.reset(main_s)
    for r, (L, c) in enumerate(zip(layers, ctxs)):
        L.compute.push(c, ars[r], 0, n_tiles, expand=r == 0, add_bias=r == 0)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main_s)
    finish_all()
    e1.record(main_s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    # bytes of all finishes: every rank reads `world` partials of its rows and
    # writes their sum into `world` copies of Y
    nbytes = 2.0 * world * rows * d_out * 2
    out["finish_all_ms"] = round(ms, 4)
    out["finish_all_gbs"] = round(nbytes / (ms / 1e3) / 1e9, 1)
    out["device_error"] = _lib.device_error()
    print(json.dumps(out), flush=True)
    for a in ars:
        a.close()


if __name__ == "__main__":
    main()
