"""The K-sharded forward's partial-Y all-reduce issued from the forward
epilogue (mlora_forward_push, mlora_ar_finish, mlora_ar_wait), with the
ranks emulated on ONE GPU: every rank's buffers are linked to the others'
directly, and all ranks' pushes, finishes and waits are issued in order on
one stream, so each bounded wait finds its counts already complete.

Reference semantics: the per-nano-batch SUM all-reduce of the partial output
rows (phase6_two_gpu_overlap.py:247-280).  The sum of bf16 partials is formed
in fp32 in rank order and rounded once, so the result must equal, bit for
bit, the same sum of the partials that the plain staged forward writes; and,
against the fp64 oracle of the unsharded layer, stay within the bf16
tolerance of 2e-2 relative L2."""

import numpy as np
import pytest
import torch

import mlora_oracle as orc
from _util import oracle_params, to_np

from tlora_b200 import _lib, ops, peer, workloads
from tlora_b200.nano import split_ranges
from tlora_b200.overlap import NativeCompute, ShardedLayer

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
DEV = "cuda"


def _ragged_spec():
    # 1000 rows (last tile 232 rows), d_out 1000 (last 256-column block 232
    # wide), d_in 640 (64-column shards of unequal width)
    return workloads.WorkloadSpec("ragged", 640, 1000, [16, 64, 8, 40], [300, 250, 200, 250], 7, torch.bfloat16)


def _emulated(w, world, impl, n_nano, timeout_s=2.0):
    dev = w.x.device
    rows, d_out = w.x.shape[0], w.model.base.weight.shape[0]
    layers = [ShardedLayer(w.model, r, world, compute=NativeCompute(impl)) for r in range(world)]
    plan = ops.route(w.ids.cpu(), layers[0].table, dev)
    assert plan.perm is None
    xs = [L.shard_input(w.x) for L in layers]
    ctxs = [L.compute.begin(L, x, plan) for L, x in zip(layers, xs)]
    for L, c in zip(layers, ctxs):
        L.compute.shrink(c)
    if ctxs[0]["z"] is not None:  # the Z all-reduce
        zsum = sum(c["z"].float() for c in ctxs).to(w.x.dtype)
        for c in ctxs:
            c["z"].copy_(zsum)
    n_tiles = ctxs[0]["n_tiles"]

    # the partials through the plain staged forward, summed in rank order in fp32
    for r, (L, c) in enumerate(zip(layers, ctxs)):
        L.compute.main(c, 0, n_tiles, expand=r == 0, add_bias=r == 0)
    acc = ctxs[0]["y"].float()
    for c in ctxs[1:]:
        acc = acc + c["y"].float()
    want = acc.to(w.x.dtype)

    ars = peer.PeerAllReduce.emulated(world, rows, d_out, w.x.dtype, dev, timeout_s)
    for a in ars:
        a.reset()
    for t0, t1 in split_ranges(n_tiles, n_nano):
        for r, (L, c) in enumerate(zip(layers, ctxs)):
            L.compute.push(c, ars[r], t0, t1, expand=r == 0, add_bias=r == 0)
        for a in ars:
            a.finish(t0, t1)
    for a in ars:
        a.wait()
    torch.cuda.synchronize()
    got = [a.y.clone() for a in ars]
    for a in ars:
        a.close()
    return want, got


@pytest.mark.parametrize("world,impl,n_nano", [(2, "tc", 1), (2, "tc", 3), (3, "tc", 2), (4, "tc", 4),
                                               (2, "tc2", 2), (2, "tcw", 2), (3, "tcw", 1), (8, "tc", 3)])
def test_push_allreduce_c3_scaled(world, impl, n_nano):
    """c3 (32 jobs, ranks 8-64) at 1/8 of its features and rows: 1024 x 1024,
    about 5k rows."""
    _lib.clear_device_error()
    w = workloads.build(workloads.spec("c3", scale=0.125), device=DEV)
    want, got = _emulated(w, world, impl, n_nano)
    assert _lib.device_error() == 0
    for r, y in enumerate(got):
        assert torch.equal(y, want), f"rank {r}: {(y.float() - want.float()).abs().max().item()}"
    W, b, ads = oracle_params(w.model)
    rows = np.sort(np.random.default_rng(3).choice(w.spec.rows, 96, replace=False))
    rt = torch.from_numpy(rows).to(DEV)
    Y = orc.multi_lora_forward(to_np(w.x[rt]), w.ids.cpu().numpy()[rows], W, b, ads)
    assert orc.relative_l2(to_np(got[0][rt]), Y) <= BF16_TOL


def test_push_allreduce_fp16():
    """fp16 partials (the reference's GPU kernels' type): same bit-exact
    rank-order sum."""
    _lib.clear_device_error()
    w = workloads.build(workloads.spec("c3", scale=0.125), device=DEV, dtype=torch.float16)
    want, got = _emulated(w, 3, "tc", 2)
    assert _lib.device_error() == 0
    for y in got:
        assert y.dtype == torch.float16 and torch.equal(y, want)


@pytest.mark.parametrize("world", [2, 3])
def test_push_allreduce_ragged(world):
    """Partial last tile and partial last 256-column block; every row and
    column of every rank's Y is written."""
    _lib.clear_device_error()
    w = workloads.build(_ragged_spec(), device=DEV)
    want, got = _emulated(w, world, "tc", 2)
    assert _lib.device_error() == 0
    for y in got:
        assert torch.equal(y, want)
    W, b, ads = oracle_params(w.model)
    Y = orc.multi_lora_forward(to_np(w.x), w.ids.cpu().numpy(), W, b, ads)
    assert orc.relative_l2(to_np(got[-1]), Y) <= BF16_TOL


def test_wait_without_pushes_times_out():
    """Nothing pushes: the owner's bounded waits run out, set the timeout bit
    of the error word and return; the context stays usable."""
    _lib.clear_device_error()
    ars = peer.PeerAllReduce.emulated(2, 600, 256, torch.bfloat16, DEV, timeout_s=0.005)
    for a in ars:
        a.reset()
    ars[0].finish(0, ars[0].n_tiles)
    ars[0].wait()
    torch.cuda.synchronize()
    assert _lib.device_error() & 2
    _lib.clear_device_error()
    for a in ars:
        a.close()
    torch.ones(4, device=DEV).sum().item()  # the device still answers


def test_timeout_is_one_deadline_per_launch():
    """Nothing pushes and every finisher warp holds many work units (about
    ten): the launch still returns after about one timeout, because all the
    waits of a launch share one deadline; the flag lands in this rank's own
    status word (mlora_peer_ar.err_word), not in the library-wide word."""
    import time
    _lib.clear_device_error()
    rows = 2 * 740 * 256  # 1480 tiles: rank 0 owns 740 x 32 work units, ~10 per warp at 148 x 16 warps
    timeout_s = 0.05
    ars = peer.PeerAllReduce.emulated(2, rows, 256, torch.bfloat16, DEV, timeout_s=timeout_s)
    word = torch.zeros(1, dtype=torch.int32, device=DEV)
    ars[0].set_err_word(word)
    for a in ars:
        a.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ars[0].finish(0, ars[0].n_tiles)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(word.item()) & 2
    assert _lib.device_error() == 0
    for a in ars:
        a.close()
    assert elapsed < 4 * timeout_s, f"finish took {elapsed:.3f} s with a {timeout_s} s timeout"


def test_push_argument_checks():
    w = workloads.build(_ragged_spec(), device=DEV)
    L = ShardedLayer(w.model, 0, 1, compute=NativeCompute("tc"))
    plan = ops.route(w.ids.cpu(), L.table, w.x.device)
    ctx = L.compute.begin(L, L.shard_input(w.x), plan)
    wrong_cols = peer.PeerAllReduce(1000, 992, torch.bfloat16, DEV, 0, 1)
    with pytest.raises(ValueError):
        L.compute.push(ctx, wrong_cols, 0, ctx["n_tiles"], expand=True, add_bias=True)
    wrong_cols.close()
    with pytest.raises(ValueError):
        peer.PeerAllReduce(1000, 1000, torch.bfloat16, DEV, 0, 9)
    with pytest.raises(NotImplementedError):
        peer.PeerAllReduce(1000, 1000, torch.float32, DEV, 0, 1)
