"""Multi-rank gloo tests (CPU, world sizes 1-3) of the K-sharded nano-batch
pipeline: the sharding, the per-nano-batch all-reduce choreography (Z, Y, dZ
and the async dB all-reduce) and the bias / LoRA expand added by one owner
rank per nano-batch must reproduce the unsharded layer (the oracle).  The
native kernels are replaced by a dense torch stand-in with the same stage
semantics; the kernels themselves are covered by the GPU parity tests."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import mlora_oracle as orc
from tlora_b200 import MultiLoRALinear
from tlora_b200.overlap import ShardedLayer, shard_columns
from tlora_b200.nano import split_ranges
from tlora_b200 import ops

from tlora_b200._lib import TILE_ROWS as TILE  # noqa: E402


class DenseCompute:
    """Stage-for-stage dense stand-in of NativeCompute (fp64 on CPU)."""

    def _rowmask(self, layer, plan, rows):
        # per-row scale on the packed rank columns of the row's adapter
        R = layer.table.r_pack
        m = torch.zeros(rows, R, dtype=torch.float64)
        for s in range(plan.n_seg):
            a = int(plan.seg_adapter[s])
            if a < 0:
                continue
            o, r = int(layer.table.pack_off[a]), int(layer.table.rank[a])
            m[plan.seg_start[s]:plan.seg_start[s + 1], o:o + r] = float(layer.scaling[a])
        return m

    def begin(self, layer, x_p, plan):
        rows = x_p.shape[0]
        return {"x": x_p, "plan": plan, "mask": self._rowmask(layer, plan, rows),
                "z": torch.zeros(rows, layer.table.r_pack, dtype=torch.float64),
                "y": torch.zeros(rows, layer.B_pack.shape[0], dtype=torch.float64),
                "n_tiles": (rows + TILE - 1) // TILE, "layer": layer}

    def shrink(self, ctx):
        L = ctx["layer"]
        ctx["z"].copy_((ctx["x"] @ L.A_pack.T) * ctx["mask"])

    def main(self, ctx, t0, t1, expand, add_bias):
        L = ctx["layer"]
        r0, r1 = t0 * TILE, min(t1 * TILE, ctx["x"].shape[0])
        v = ctx["x"][r0:r1] @ L.W.T
        if expand:
            v = v + ctx["z"][r0:r1] @ L.B_pack.T
        if add_bias and L.bias is not None:
            v = v + L.bias
        ctx["y"][r0:r1] = v

    def bwd_begin(self, ctx, layer, x_p, dy, overlapped=False, partial=True):
        rows = x_p.shape[0]
        d_out = layer.B_pack.shape[0]
        return {"ctx": ctx, "layer": layer, "x": x_p, "dy": dy,
                "dz": torch.zeros(rows, layer.table.r_pack, dtype=torch.float64),
                "dx": None, "dA": None, "dB": torch.zeros_like(layer.B_pack),
                "n_tiles": (rows + TILE - 1) // TILE, "n_db": (d_out + 127) // 128}

    def bwd_dz(self, b, t0, t1):
        L, ctx = b["layer"], b["ctx"]
        r0, r1 = t0 * TILE, min(t1 * TILE, b["x"].shape[0])
        b["dz"][r0:r1] = (b["dy"][r0:r1] @ L.B_pack) * ctx["mask"][r0:r1]

    def bwd_dx(self, b):
        L = b["layer"]
        b["dx"] = b["dy"] @ L.W + b["dz"] @ L.A_pack

    def bwd_da(self, b):
        b["dA"] = b["dz"].T @ b["x"]

    def bwd_db(self, b, b0, b1):
        r0, r1 = b0 * 128, min(b1 * 128, b["dB"].shape[0])
        b["dB"][r0:r1] = b["dy"][:, r0:r1].T @ b["ctx"]["z"]

    def bwd_dadb(self, b):
        self.bwd_da(b)
        self.bwd_db(b, 0, b["n_db"])

    def sgd(self, layer, plan, dA, dB, lr, which=("A", "B")):
        for i in range(layer.table.n):
            if plan.active[i]:
                o, r = int(layer.table.pack_off[i]), int(layer.table.rank[i])
                if "A" in which:
                    layer.A_pack[o:o + r] -= lr * dA[o:o + r]
                if "B" in which:
                    layer.B_pack[:, o:o + r] -= lr * dB[:, o:o + r]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _build(seed=0):
    torch.manual_seed(seed)
    m = MultiLoRALinear(256, 300, {0: 4, 1: 70, 2: 8}).double()
    with torch.no_grad():
        m.base.bias.normal_(0, 0.1)
        for ad in m.adapters.values():
            ad.B.normal_(0, 0.05)
            ad.scaling = 2.0
    ids = torch.tensor([0] * 300 + [1] * 200 + [2] * 77 + [9] * 5)
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(ids.shape[0], 256, generator=g, dtype=torch.float64)
    dy = torch.randn(ids.shape[0], 300, generator=g, dtype=torch.float64)
    return m, ids, x, dy


def _worker(rank, world, port, n_nano, pipelined, q, dz="split", split="even"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m, ids, x, dy = _build()
        layer = ShardedLayer(m, rank, world, compute=DenseCompute(), bwd_group=dist.new_group(list(range(world))),
                             dz=dz)
        layer.split = split
        plan = ops.route(ids, layer.table, torch.device("cpu"))
        x_p = layer.shard_input(x)
        y, dx_p = layer.step(x_p, plan, dy, n_nano, lr=0.01, pipelined=pipelined)
        # shards of unequal width (64-column blocks): gathered as objects
        parts = [None] * world
        dist.all_gather_object(parts, dx_p.contiguous())
        a_parts = [None] * world
        dist.all_gather_object(a_parts, layer.A_pack.contiguous())
        if rank == 0:
            q.put({"y": y.numpy().copy(), "dx": torch.cat(parts, 1).numpy(),
                   "A_pack": torch.cat(a_parts, 1).numpy(), "B_pack": layer.B_pack.numpy().copy(),
                   "pack_off": layer.table.pack_off.copy(), "rank": layer.table.rank.copy()})
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_nano,pipelined,dz,split", [(2, 1, True, "split", "even"), (2, 3, True, "split", "even"),
                                                             (2, 2, False, "split", "even"),
                                                             (3, 4, True, "split", "even"),
                                                             (1, 2, True, "split", "even"),
                                                             (2, 3, True, "replicated", "even"),
                                                             (3, 2, True, "replicated", "even"),
                                                             (2, 3, True, "split", "ramp")])
def test_sharded_step_matches_unsharded(world, n_nano, pipelined, dz, split):
    """Every rank's step against the fp64 oracle of the unsharded layer; dZ
    split across the ranks and summed, or computed whole on every rank; even
    nano-batches or a short first one."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_nano, pipelined, q, dz, split))
             for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0

    m, ids, x, dy = _build()
    W = m.base.weight.detach().numpy()
    b = m.base.bias.detach().numpy()
    ads = {int(k): orc.OracleAdapter(a.A.detach().numpy(), a.B.detach().numpy(), float(a.scaling))
           for k, a in m.adapters.items()}
    xn, idn, dyn = x.numpy(), ids.numpy(), dy.numpy()
    Y = orc.multi_lora_forward(xn, idn, W, b, ads)
    dX, dA, dB = orc.multi_lora_backward(xn, idn, W, ads, dyn)
    assert orc.relative_l2(res["y"], Y) < 1e-12
    assert orc.relative_l2(res["dx"], dX) < 1e-12
    for i, a in enumerate(sorted(ads)):
        o, r = int(res["pack_off"][i]), int(res["rank"][i])
        A_next = orc.sgd_step(ads[a].A, dA[a], 0.01)
        B_next = orc.sgd_step(ads[a].B, dB[a], 0.01)
        assert orc.relative_l2(res["A_pack"][o:o + r], A_next) < 1e-12
        assert orc.relative_l2(res["B_pack"][:, o:o + r], B_next) < 1e-12


def test_shard_columns_cover_exactly():
    for d in [64, 192, 4096, 8192, 11008]:
        for world in [1, 2, 4, 8]:
            spans = [shard_columns(d, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == d
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert all(s % 64 == 0 for s, _ in spans)


def test_split_setting_is_checked():
    from tlora_b200.overlap import ShardedLayer
    m, _, _, _ = _build()
    layer = ShardedLayer(m, 0, 1, compute=DenseCompute())
    assert layer.ranges(10, 3) == [(0, 4), (4, 7), (7, 10)]
    layer.split = "ramp:0.25"
    assert layer.ranges(153, 4)[0] == (0, 12)
    for bad in ("bogus", "ramp:0", "ramp:-1"):
        layer.split = bad
        with pytest.raises(ValueError):
            layer.ranges(10, 3)


def test_ramp_ranges_cover_exactly():
    from tlora_b200.nano import ramp_ranges
    for total in (1, 2, 5, 39, 153):
        for n in (1, 2, 3, 4, 8, 16):
            r = ramp_ranges(total, n)
            assert r[0][0] == 0 and r[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
            assert all(e > s for s, e in r)
            assert len(r) == min(n, total)
            if len(r) > 2:
                assert r[0][1] - r[0][0] <= min(e - s for s, e in r[1:])


def test_nano_ranges_over_tiles():
    for tiles in [1, 3, 512]:
        for n in [1, 2, 4, 8, 16, 32]:
            r = split_ranges(tiles, n)
            assert r[0][0] == 0 and r[-1][1] == tiles and len(r) == min(n, tiles)


# ---------------------------------------------------------------- failure detection
# A rank that is lost (exits before the step's collectives) or late must not
# hang the others: the process group carries a short timeout, a lost peer
# surfaces as an exception on the surviving rank, a late one within the
# timeout only delays the step.  Host-side only (gloo on CPU): no GPU is
# faulted or hung to test this.

def _fault_worker(rank, world, port, mode, q):
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    m, ids, x, dy = _build()
    layer = ShardedLayer(m, rank, world, compute=DenseCompute(), bwd_group=dist.new_group([0, 1]))
    plan = ops.route(ids, layer.table, torch.device("cpu"))
    x_p = layer.shard_input(x)
    if rank == 1 and mode == "lost":
        os._exit(0)  # leaves between steps, none of its collectives in flight
    if rank == 1 and mode == "late":
        time.sleep(1.5)
    t0 = time.monotonic()
    try:
        layer.step(x_p, plan, dy, 2, lr=0.01)
        outcome = "ok"
    except Exception as e:  # noqa: BLE001 - the failure is what is being tested
        outcome = f"error: {type(e).__name__}"
    if rank == 0:
        q.put((outcome, time.monotonic() - t0))
        q.close()
        q.join_thread()  # flush before os._exit
    if outcome == "ok":
        dist.destroy_process_group()
    os._exit(0)


@pytest.mark.parametrize("mode", ["lost", "late"])
def test_lost_or_late_rank(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fault_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        outcome, seconds = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    if mode == "lost":
        assert outcome.startswith("error"), outcome  # surfaced, not hung
        assert seconds < 60
    else:
        assert outcome == "ok", outcome
