"""GPU parity of the K-sharded training step (tlora_b200.overlap.ShardedLayer)
against the fp64 oracle of the unsharded layer: Y, dX (gathered from the
ranks' d_in shards), dA (gathered), dB and the one-step SGD update of every
adapter, within the bf16 bound of 2e-2 relative L2 (fp32 accumulation), and
the SGD update elementwise (bf16 rounding of P - lr G).

Reference semantics: the reference's nano-batch pipeline sums each
nano-batch's partial rows with a SUM all-reduce (phase6_two_gpu_overlap.py:
247-280) and checks its GPU path's forward, gradients and SGD step against a
PyTorch reference (phase5d_triton_training.py:420-589).

Runs on ONE GPU: one rank with no collective (the pipeline's one-GPU point),
and two or three ranks as separate processes sharing the GPU, their
collectives over gloo (the NCCL path's choreography: Z, each nano-batch's Y,
dZ and dB all-reduces).  No kernel of one process waits on another process's
kernel, so sharing the GPU is safe.  The all-reduce paths that need one GPU
per rank (NCCL, peer stores, multicast) are covered by
test_gpu_peer_multi.py on two GPUs."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _spec():
    from tlora_b200 import workloads
    # c3 at 1/8 of its features and rows: 1024 x 1024, 32 jobs, ~5k rows
    return workloads.spec("c3", scale=0.125)


def run_rank(rank, world, n_nano, dev, steps=1, split="even", dz="split"):
    """One rank's training step(s); returns numpy Y, this rank's dX shard,
    dA shard, dB, the updated A shard and B, and the shard's columns."""
    from tlora_b200 import _lib, ops, workloads
    from tlora_b200.overlap import ShardedLayer

    w = workloads.build(_spec(), device=dev)
    group = dist.new_group(list(range(world))) if world > 1 else None
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    layer = ShardedLayer(w.model, rank, world, bwd_group=group, err_word=err, dz=dz)
    layer.split = split
    plan = ops.route(w.ids.cpu(), layer.table, dev)
    x_p = layer.shard_input(w.x)
    for _ in range(steps):
        y, dx_p = layer.step(x_p, plan, w.dy, n_nano, lr=w.spec.lr)
    torch.cuda.synchronize(dev)
    layer.check()
    dA_p, dB = layer.last_grads

    def f64(t):
        return t.detach().float().cpu().numpy().astype(np.float64)

    out = {"y": f64(y), "dx": f64(dx_p), "dA": f64(dA_p), "dB": f64(dB), "A": f64(layer.A_pack),
           "B": f64(layer.B_pack), "cols": (layer.k0, layer.k1), "err": int(err.item()),
           "lib_err": _lib.device_error()}
    return out


def check_against_oracle(parts, steps=1):
    """parts: per-rank results of run_rank; compares the assembled layer with
    the fp64 oracle of the unsharded layer."""
    import mlora_oracle as orc
    from _util import oracle_params, to_np
    from tlora_b200 import workloads

    w = workloads.build(_spec(), device="cuda")
    W, b, ads = oracle_params(w.model)
    A_pack0, B_pack0, table = w.model.packed()
    x, dy, ids = to_np(w.x), to_np(w.dy), w.ids.cpu().numpy()
    lr = w.spec.lr
    Y = orc.multi_lora_forward(x, ids, W, b, ads)
    dX, dA, dB = orc.multi_lora_backward(x, ids, W, ads, dy)
    order = sorted(parts, key=lambda p: p["cols"][0])
    got_y = parts[0]["y"]
    got_dx = np.concatenate([p["dx"] for p in order], axis=1)
    got_dA = np.concatenate([p["dA"] for p in order], axis=1)
    got_A = np.concatenate([p["A"] for p in order], axis=1)
    errs = {"Y": orc.relative_l2(got_y, Y), "dX": orc.relative_l2(got_dx, dX)}
    for p in parts:
        assert p["err"] == 0 and p["lib_err"] == 0, "a device-side check fired"
        # every rank holds the same summed Y and dB
        assert np.array_equal(p["y"], got_y)
        assert np.array_equal(p["dB"], parts[0]["dB"])
    A_prev, B_prev = to_np(A_pack0), to_np(B_pack0)
    for i, a in enumerate(table.ids):
        o, r = int(table.pack_off[i]), int(table.rank[i])
        errs[f"dA{a}"] = orc.relative_l2(got_dA[o:o + r], dA[a])
        errs[f"dB{a}"] = orc.relative_l2(parts[0]["dB"][:, o:o + r], dB[a])
        if steps == 1:
            errs[f"A{a}"] = orc.relative_l2(got_A[o:o + r], orc.sgd_step(ads[a].A, dA[a], lr))
            errs[f"B{a}"] = orc.relative_l2(parts[0]["B"][:, o:o + r], orc.sgd_step(ads[a].B, dB[a], lr))
            # elementwise: the update of the gradients the layer produced, rounded once to bf16
            for got, P, G in ((got_A[o:o + r], A_prev[o:o + r], got_dA[o:o + r]),
                              (parts[0]["B"][:, o:o + r], B_prev[:, o:o + r], parts[0]["dB"][:, o:o + r])):
                want = P - lr * G
                bound = 2.0 ** -8 * np.abs(want) + 1e-6 * (np.abs(P) + lr * np.abs(G)) + 1e-30
                assert np.all(np.abs(got - want) <= bound), f"SGD update of adapter {a}"
    bad = {k: v for k, v in errs.items() if not v <= BF16_TOL}
    assert not bad, f"relative L2 above {BF16_TOL}: {bad}"
    return errs


@pytest.mark.parametrize("n_nano,split", [(1, "even"), (3, "even"), (3, "ramp")])
def test_one_rank_pipeline_matches_oracle(n_nano, split):
    """The pipeline's one-GPU point: no collective at all; even nano-batches
    or a short first one."""
    res = run_rank(0, 1, n_nano, torch.device("cuda", 0), split=split)
    check_against_oracle([res])


@pytest.mark.parametrize("n_nano", [1, 3])
def test_graphed_step_matches_eager_step(n_nano):
    """GraphedShardedStep (the whole step captured once, replayed) gives the
    eager step's Y, dX, gradients and updated weights bit for bit, replay
    after replay (one rank: no collective, deterministic kernels)."""
    from tlora_b200 import ops, workloads
    from tlora_b200.overlap import GraphedShardedStep, ShardedLayer

    dev = torch.device("cuda", 0)
    w = workloads.build(_spec(), device=dev)
    layer = ShardedLayer(w.model, 0, 1)
    plan = ops.route(w.ids.cpu(), layer.table, dev)
    x_p = layer.shard_input(w.x)
    A0, B0 = layer.A_pack.clone(), layer.B_pack.clone()
    g = GraphedShardedStep(layer, x_p, plan, w.dy, n_nano, w.spec.lr)
    for _ in range(2):
        with torch.no_grad():
            layer.A_pack.copy_(A0)
            layer.B_pack.copy_(B0)
        y, dx = layer.step(x_p, plan, w.dy, n_nano, w.spec.lr)
        want = [t.clone() for t in (y, dx, *layer.last_grads, layer.A_pack, layer.B_pack)]
        with torch.no_grad():
            layer.A_pack.copy_(A0)
            layer.B_pack.copy_(B0)
        y, dx = g()
        got = [t.clone() for t in (y, dx, *g.grads, layer.A_pack, layer.B_pack)]
        torch.cuda.synchronize(dev)
        for name, a, b in zip(("Y", "dX", "dA", "dB", "A", "B"), got, want):
            assert torch.equal(a, b), name
    assert g.kernels > 0


def test_graph_outlives_the_layers_cached_buffers():
    """A captured step keeps its buffers after the layer rebuilds its cached
    call objects (here: a step with another plan object) and their old
    memory is handed out again: replays still give the eager step's results
    bit for bit."""
    from tlora_b200 import ops, workloads
    from tlora_b200.overlap import GraphedShardedStep, ShardedLayer

    dev = torch.device("cuda", 0)
    w = workloads.build(_spec(), device=dev)
    layer = ShardedLayer(w.model, 0, 1)
    plan = ops.route(w.ids.cpu(), layer.table, dev)
    x_p = layer.shard_input(w.x)
    A0, B0 = layer.A_pack.clone(), layer.B_pack.clone()
    g = GraphedShardedStep(layer, x_p, plan, w.dy, 3, w.spec.lr)

    def reset():
        with torch.no_grad():
            layer.A_pack.copy_(A0)
            layer.B_pack.copy_(B0)

    reset()
    y, dx = layer.step(x_p, plan, w.dy, 3, w.spec.lr)
    want = [t.clone() for t in (y, dx, *layer.last_grads, layer.A_pack, layer.B_pack)]
    # another plan object: the layer builds new call objects and buffers
    plan2 = ops.route(w.ids.cpu(), layer.table, dev)
    reset()
    layer.step(x_p, plan2, w.dy, 3, w.spec.lr)
    torch.cuda.synchronize(dev)
    # take back whatever the allocator has free and scribble on it
    junk = [torch.full((1 << 20,), 7, dtype=torch.int32, device=dev) for _ in range(64)]
    reset()
    y, dx = g()
    got = [t.clone() for t in (y, dx, *g.grads, layer.A_pack, layer.B_pack)]
    torch.cuda.synchronize(dev)
    del junk
    for name, a, b in zip(("Y", "dX", "dA", "dB", "A", "B"), got, want):
        assert torch.equal(a, b), name


def _worker(rank, world, port, n_nano, q, split="even", dz="split"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        q.put((rank, run_rank(rank, world, n_nano, dev, split=split, dz=dz)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_nano,split,dz", [(2, 1, "even", "split"), (2, 3, "even", "split"),
                                                   (3, 4, "even", "split"), (2, 3, "ramp", "replicated")])
def test_sharded_ranks_on_one_gpu_match_oracle(world, n_nano, split, dz):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_nano, q, split, dz)) for r in range(world)]
    for p in procs:
        p.start()
    parts = {}
    try:
        for _ in range(world):
            r, res = q.get(timeout=600)
            parts[r] = res
    finally:
        for p in procs:
            p.join(timeout=120)
    for p in procs:
        assert p.exitcode == 0
    check_against_oracle(list(parts.values()))


def _mc_worker(port, q):
    """One rank: the multicast all-reduce over a one-GPU multicast object
    (the sum over one rank is the value itself), several slots and uses."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from tlora_b200 import _lib, peer
        try:
            mc = peer.MulticastAllReduce(1000, 264, torch.bfloat16, dev)
        except RuntimeError as e:
            q.put({"unsupported": str(e)})
            return
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        mc.set_err_word(err)
        ok = True
        for it in range(3):
            want = torch.randn(1000, 264, device=dev).to(torch.bfloat16)
            mc.y.copy_(want)
            side = torch.cuda.Stream(dev)
            ev = torch.cuda.Event()
            ev.record()
            side.wait_event(ev)
            for i, (r0, r1) in enumerate(((0, 256), (256, 700), (700, 1000))):
                mc.reduce(r0, r1, i, side)
            mc.wait(3, side)
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            ok = ok and torch.equal(mc.y, want)
        uses = mc.buf[-4 * _lib.MC_FLAG_WORDS:].view(torch.int32)[3 * _lib.MC_SLOTS:3 * _lib.MC_SLOTS + 3]
        q.put({"ok": ok, "err": int(err.item()), "lib_err": _lib.device_error(), "uses": uses.tolist()})
        mc.close()
    finally:
        dist.destroy_process_group()


def test_multicast_allreduce_one_gpu():
    """mlora_mc_allreduce / mlora_mc_wait on a multicast object of one GPU:
    every row comes back unchanged (a sum over one rank), the flag counters
    of three slots advance over three uses without a reset, and no bounded
    wait runs out.  Skipped where the GPU offers no multicast object."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_mc_worker, args=(_free_port(), q))
    p.start()
    try:
        res = q.get(timeout=300)
    finally:
        p.join(timeout=120)
    if "unsupported" in res:
        pytest.skip(res["unsupported"])
    assert p.exitcode == 0
    assert res["ok"] and res["err"] == 0 and res["lib_err"] == 0 and res["uses"] == [3, 3, 3]
