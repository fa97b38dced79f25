"""mlora_forward_noalloc: the forward for callers that cannot allocate device
memory (serving runtimes and plugin hosts that reserve all device memory at
start-up, C/Go/Java hosts without a device allocator).  Called through the C
ABI, it runs the same kernels on the same inputs as mlora_forward, so its Y
must equal mlora_forward's bit for bit on two calls in a row (the tile
scheduler hands out whole output tiles, so the result does not depend on
which CTA computes a tile); and it must reject problems whose scratch exceeds
its fixed 32 MiB array.

This file is collected last so that a run stopping at the first failure has
already run every other test."""

import ctypes

import numpy as np
import pytest
import torch

import mlora_oracle as orc
from tlora_b200 import MultiLoRALinear, _lib, ops

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _setup(dtype, d_in=512, d_out=384, ranks=None, counts=None, seed=0):
    ranks = ranks or {0: 8, 1: 64, 2: 100, 3: 1}
    counts = counts or [300, 257, 129, 1]
    torch.manual_seed(seed)
    m = MultiLoRALinear(d_in, d_out, ranks)
    with torch.no_grad():
        m.base.bias.normal_(0, 0.1)
        for ad in m.adapters.values():
            ad.B.normal_(0, 0.05)
            ad.scaling = 2.0
    m = m.to(DEV, dtype)
    A_pack, B_pack, table = m.packed()
    ids = torch.cat([torch.full((c,), a, dtype=torch.int64) for a, c in zip(ranks, counts)])
    plan = ops.route(ids, table, torch.device(DEV))
    scaling = np.array([float(a.scaling) for a in m.adapters.values()], dtype=np.float32)
    args = ops._CallArgs(int(ids.shape[0]), d_in, d_out, ops.mlora_dtype(dtype), "auto", plan, table, scaling)
    x = torch.randn(ids.shape[0], d_in, device=DEV).to(dtype)
    return m, A_pack, B_pack, args, x


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _forward(m, A_pack, B_pack, args, x):
    zb, wb = args.sizes()
    z = torch.empty(max(zb, 1), dtype=torch.uint8, device=DEV)
    ws = torch.empty(max(wb, 1), dtype=torch.uint8, device=DEV)
    y = torch.empty(x.shape[0], B_pack.shape[0], dtype=x.dtype, device=DEV)
    _lib.call("mlora_forward", ctypes.byref(args.prob), ctypes.byref(args.route), _ptr(x), _ptr(m.base.weight),
              _ptr(m.base.bias), _ptr(A_pack), _ptr(B_pack), _ptr(y), _ptr(z), _ptr(ws), wb, _stream())
    return y


def _forward_noalloc(m, A_pack, B_pack, args, x):
    y = torch.full((x.shape[0], B_pack.shape[0]), float("nan"), dtype=x.dtype, device=DEV)
    _lib.call("mlora_forward_noalloc", ctypes.byref(args.prob), ctypes.byref(args.route), _ptr(x),
              _ptr(m.base.weight), _ptr(m.base.bias), _ptr(A_pack), _ptr(B_pack), _ptr(y), _stream())
    return y


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 2e-2), (torch.float32, 1e-5)])
def test_noalloc_matches_forward_twice(dtype, tol):
    m, A_pack, B_pack, args, x = _setup(dtype)
    y_ref = _forward(m, A_pack, B_pack, args, x).float()
    for _ in range(2):  # the array keeps the previous call's contents
        y = _forward_noalloc(m, A_pack, B_pack, args, x).float()
        torch.cuda.synchronize()
        assert torch.isfinite(y).all()
        err = orc.relative_l2(y.cpu().numpy(), y_ref.cpu().numpy())
        assert err <= tol, err
        assert torch.equal(y, y_ref), f"not bit-identical to mlora_forward (relative L2 {err:.3e})"


def test_noalloc_second_problem_after_first():
    """A different routing plan right after: stale scratch must not leak in."""
    m, A_pack, B_pack, args, x = _setup(torch.bfloat16)
    _forward_noalloc(m, A_pack, B_pack, args, x)
    m2, A2, B2, args2, x2 = _setup(torch.bfloat16, ranks={5: 16, 7: 3}, counts=[77, 500], seed=3)
    y_ref = _forward(m2, A2, B2, args2, x2).float()
    y = _forward_noalloc(m2, A2, B2, args2, x2).float()
    torch.cuda.synchronize()
    assert orc.relative_l2(y.cpu().numpy(), y_ref.cpu().numpy()) <= 2e-2
    assert torch.equal(y, y_ref)


def test_noalloc_rejects_oversized_problem():
    # 2,344 tiles x one 64-column rank chunk = 38 MB of intermediate > 32 MiB
    m, A_pack, B_pack, args, x = _setup(torch.bfloat16, d_in=64, d_out=64, ranks={0: 64},
                                        counts=[300000])
    y = torch.empty(x.shape[0], 64, dtype=x.dtype, device=DEV)
    st = _lib.lib().mlora_forward_noalloc(ctypes.byref(args.prob), ctypes.byref(args.route), _ptr(x),
                                          _ptr(m.base.weight), _ptr(m.base.bias), _ptr(A_pack), _ptr(B_pack),
                                          _ptr(y), _stream())
    assert st == _lib.ERR_WORKSPACE
