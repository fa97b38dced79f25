"""Shared helpers of the parity tests: run the module and the numpy oracle on
the same inputs and compare."""

import numpy as np
import torch

import mlora_oracle as orc


def to_np(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def oracle_params(m):
    W = to_np(m.base.weight)
    b = to_np(m.base.bias) if m.base.bias is not None else None
    ads = {int(k): orc.OracleAdapter(A=to_np(a.A), B=to_np(a.B), scaling=float(a.scaling))
           for k, a in m.adapters.items()}
    return W, b, ads


def module_step(m, x, ids, dy, add_base=True):
    """Forward + backward with upstream grad dy; returns numpy Y, dX and the
    per-adapter grads (None where autograd left them unset)."""
    for a in m.adapters.values():
        a.A.grad = None
        a.B.grad = None
    xg = x.detach().clone().requires_grad_(True)
    y = m(xg, ids, add_base=add_base)
    y.backward(dy)
    torch.cuda.synchronize()
    dA = {int(k): (to_np(a.A.grad) if a.A.grad is not None else None) for k, a in m.adapters.items()}
    dB = {int(k): (to_np(a.B.grad) if a.B.grad is not None else None) for k, a in m.adapters.items()}
    return to_np(y), to_np(xg.grad), dA, dB


def oracle_step(m, x, ids, dy, add_base=True):
    W, b, ads = oracle_params(m)
    xn, dyn = to_np(x), to_np(dy)
    idn = ids.detach().cpu().numpy()
    if not add_base:
        W = np.zeros_like(W)
        b = None
    Y = orc.multi_lora_forward(xn, idn, W, b, ads)
    dX, dA, dB = orc.multi_lora_backward(xn, idn, W, ads, dyn)
    return Y, dX, dA, dB


def assert_parity(got, want, tol, what=""):
    Y, dX, dA, dB = got
    Yr, dXr, dAr, dBr = want
    errs = {"Y": orc.relative_l2(Y, Yr), "dX": orc.relative_l2(dX, dXr)}
    for a in dAr:
        if dAr[a] is None:
            assert dA[a] is None and dB[a] is None, f"{what}: adapter {a} owns no rows but got a gradient"
            continue
        assert dA[a] is not None and dB[a] is not None, f"{what}: adapter {a} missing gradient"
        errs[f"dA{a}"] = orc.relative_l2(dA[a], dAr[a])
        errs[f"dB{a}"] = orc.relative_l2(dB[a], dBr[a])
    bad = {k: v for k, v in errs.items() if not v <= tol}
    assert not bad, f"{what}: relative L2 above {tol}: {bad}"
    return errs
