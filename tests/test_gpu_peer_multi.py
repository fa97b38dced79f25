"""The K-sharded training step across real GPUs, one process per GPU (NCCL for
the plumbing), with each of the three all-reduce paths of the partial Y:
NCCL's all-reduce of each nano-batch (the reference's
phase6_two_gpu_overlap.py:247-280), the all-reduce issued from the forward
epilogue over peer memory (CUDA IPC), and the one through the NVSwitch's
multicast objects (torch symmetric memory).  For each path, one full
training step (forward, backward, isolated SGD) must match the fp64 oracle of
the unsharded layer within 2e-2 (Y, dX and dA gathered from the ranks'
shards, dB, the updated weights) with the SGD update elementwise, as the
reference checks its GPU training path (phase5d_triton_training.py:420-589);
the peer and multicast forwards must equal NCCL's up to the rounding of the
bf16 sum.  Each path is also checked replayed from a CUDA graph of the whole
step (GraphedShardedStep), replayed twice.  Needs >= 2 GPUs; NVLink multicast objects are used only by the
multicast case, whose ranks all finish their device work before any exits."""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

COMMS = ("nccl", "peer", "mc")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from test_gpu_ksharded import run_rank, _spec
        from tlora_b200 import ops, workloads
        from tlora_b200.overlap import ShardedLayer

        out = {}
        for comm in COMMS:
            for graphed in (False, True):
                try:
                    res = run_rank_comm(rank, world, comm, dev, graphed)
                except RuntimeError as e:
                    if comm == "mc" and "multicast" in str(e):
                        res = {"unsupported": str(e)}
                    else:
                        raise
                out[(comm, graphed)] = res
        # forwards of the three paths on the same inputs
        w = workloads.build(_spec(), device=dev)
        fw = {}
        for comm in COMMS:
            if "unsupported" in out.get((comm, False), {}):
                continue
            layer = ShardedLayer(w.model, rank, world, comm=comm)
            plan = ops.route(w.ids.cpu(), layer.table, dev)
            y, _ = layer.forward(layer.shard_input(w.x), plan, 3)
            torch.cuda.synchronize(dev)
            fw[comm] = y.float().cpu().numpy()
            layer.close()
        out["forwards"] = fw
        q.put((rank, out))
    finally:
        torch.cuda.synchronize(dev)
        dist.barrier()
        dist.destroy_process_group()


def run_rank_comm(rank, world, comm, dev, graphed=False):
    """run_rank of test_gpu_ksharded with the given all-reduce path (one
    step, 3 nano-batches) on the default NCCL group; with ``graphed`` the
    step is replayed from a CUDA graph (GraphedShardedStep) after the
    weights are reset to the model's."""
    from test_gpu_ksharded import _spec
    import numpy as np  # noqa: F811
    from tlora_b200 import _lib, ops, workloads
    from tlora_b200.overlap import GraphedShardedStep, ShardedLayer

    w = workloads.build(_spec(), device=dev)
    bwd = dist.new_group(list(range(world)))
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    layer = ShardedLayer(w.model, rank, world, bwd_group=bwd, comm=comm, err_word=err)
    g = None
    try:
        plan = ops.route(w.ids.cpu(), layer.table, dev)
        x_p = layer.shard_input(w.x)
        if graphed:
            A0, B0 = layer.A_pack.clone(), layer.B_pack.clone()
            g = GraphedShardedStep(layer, x_p, plan, w.dy, 3, w.spec.lr)
            with torch.no_grad():
                layer.A_pack.copy_(A0)
                layer.B_pack.copy_(B0)
            for _ in range(2):  # replay twice: the second replay must wait for the other rank's sums too
                with torch.no_grad():
                    layer.A_pack.copy_(A0)
                    layer.B_pack.copy_(B0)
                y, dx_p = g()
            dA_p, dB = g.grads
        else:
            y, dx_p = layer.step(x_p, plan, w.dy, 3, lr=w.spec.lr)
            dA_p, dB = layer.last_grads
        torch.cuda.synchronize(dev)
        layer.check()

        def f64(t):
            return t.detach().float().cpu().numpy().astype(np.float64)

        return {"y": f64(y), "dx": f64(dx_p), "dA": f64(dA_p), "dB": f64(dB), "A": f64(layer.A_pack),
                "B": f64(layer.B_pack), "cols": (layer.k0, layer.k1), "err": int(err.item()),
                "lib_err": _lib.device_error()}
    finally:
        torch.cuda.synchronize(dev)
        del g  # the graph before the buffers it uses
        layer.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ksharded_step_two_gpus_every_allreduce_path():
    from test_gpu_ksharded import check_against_oracle

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, out = q.get(timeout=600)
            res[r] = out
    finally:
        for p in procs:
            p.join(timeout=120)
    for p in procs:
        assert p.exitcode == 0
    checked = []
    for comm in COMMS:
        for graphed in (False, True):
            parts = [res[r][(comm, graphed)] for r in range(world)]
            if any("unsupported" in p for p in parts):
                assert comm == "mc"
                continue
            check_against_oracle(parts)
            checked.append((comm, graphed))
    assert {("nccl", False), ("nccl", True), ("peer", False), ("peer", True)} <= set(checked)
    fw = res[0]["forwards"]
    ref = fw["nccl"]
    for comm, y in fw.items():
        d = np.abs(y - ref)
        assert np.linalg.norm(d) / np.linalg.norm(ref) <= 4e-3, comm
