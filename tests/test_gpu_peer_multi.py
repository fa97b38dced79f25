"""The peer all-reduce of the K-sharded forward across real GPUs: one process
per GPU (NCCL for the plumbing, CUDA IPC for the peer buffers).  The forward
with the all-reduce issued from the epilogue (``comm="peer"``) must give the
same Y as the same forward with NCCL's all-reduce of each nano-batch
(``comm="nccl"``, the reference's phase6_two_gpu_overlap.py:247-280) — equal
up to the rounding of the bf16 sum (NCCL may add in another order) — and
match the fp64 oracle of the unsharded layer within 2e-2; a full training
step in peer mode must run without a device error.  Needs >= 2 GPUs."""

import os
import socket
from datetime import timedelta

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


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    layer = None
    try:
        import mlora_oracle as orc
        from _util import oracle_params, to_np
        from tlora_b200 import _lib, ops, workloads
        from tlora_b200.overlap import ShardedLayer

        w = workloads.build(workloads.spec("c3", scale=0.125), device=dev)
        rows = np.sort(np.random.default_rng(5).choice(w.spec.rows, 96, replace=False))
        rt = torch.from_numpy(rows).to(dev)
        W, b, ads = oracle_params(w.model)
        Y = orc.multi_lora_forward(to_np(w.x[rt]), w.ids.cpu().numpy()[rows], W, b, ads)
        layer = ShardedLayer(w.model, rank, world, comm="peer")
        plan = ops.route(w.ids.cpu(), layer.table, dev)
        x_p = layer.shard_input(w.x)
        out = {}
        for n_nano in (1, 3):
            layer.comm = "peer"
            y_peer, _ = layer.forward(x_p, plan, n_nano)
            y_peer = y_peer.clone()
            layer.comm = "nccl"
            y_nccl, _ = layer.forward(x_p, plan, n_nano)
            torch.cuda.synchronize(dev)
            d = (y_peer.float() - y_nccl.float()).abs()
            out[n_nano] = {"max_diff": float(d.max()), "rel": float(d.norm() / y_nccl.float().norm()),
                           "oracle": orc.relative_l2(to_np(y_peer[rt]), Y)}
        layer.comm = "peer"
        layer.step(x_p, plan, w.dy, 3, lr=1e-3)
        torch.cuda.synchronize(dev)
        out["err"] = _lib.device_error()
        if rank == 0:
            q.put(out)
    finally:
        if layer is not None:
            torch.cuda.synchronize(dev)
            dist.barrier()
            layer.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_allreduce_two_gpus():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res["err"] == 0
    for n_nano in (1, 3):
        r = res[n_nano]
        assert r["rel"] <= 4e-3, r
        assert r["oracle"] <= BF16_TOL, r
