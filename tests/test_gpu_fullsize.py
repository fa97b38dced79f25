"""GPU parity at the full sizes of the bf16 configurations, through properties
the CPU oracle can check in seconds: Y and dX on a random sample of rows
(both are row-local, so the sampled rows of the fp64 oracle are exact),
bilinear probes u^T dA v and u^T dB v of every active adapter's gradients
(oracle.grad_projections), within the bf16 bound of 2e-2 relative L2 (fp32
accumulation); and the one-step SGD update applied elementwise to those
gradients."""

import numpy as np
import pytest
import torch

import mlora_oracle as orc
from _util import oracle_params, to_np

from tlora_b200 import workloads

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
DEV = "cuda"
N_ROWS = 64
N_PROBES = 8


def _probes(rng, ads, d_in, d_out):
    return {a: (rng.standard_normal((N_PROBES, ad.A.shape[0])), rng.standard_normal((N_PROBES, d_in)),
                rng.standard_normal((N_PROBES, d_out)), rng.standard_normal((N_PROBES, ad.A.shape[0])))
            for a, ad in ads.items()}


def _probe(M, u, v):
    return np.einsum("ki,ij,kj->k", u, M, v)


@pytest.mark.parametrize("cfg", ["c2", "c4"])
def test_full_size_training_step(cfg):
    w = workloads.build(workloads.spec(cfg), device=DEV)
    m, sp = w.model, w.spec
    xg = w.x.detach().clone().requires_grad_(True)
    y = m(xg, w.ids)
    y.backward(w.dy)
    torch.cuda.synchronize()
    W, b, ads = oracle_params(m)
    ids = w.ids.cpu().numpy()
    rng = np.random.default_rng(11)

    # Y and dX on sampled rows
    rows = np.sort(rng.choice(sp.rows, N_ROWS, replace=False))
    rt = torch.from_numpy(rows).to(DEV)
    xr, dyr = to_np(w.x[rt]), to_np(w.dy[rt])
    Y_want = orc.multi_lora_forward(xr, ids[rows], W, b, ads)
    dX_want, _, _ = orc.multi_lora_backward(xr, ids[rows], W, ads, dyr)
    assert orc.relative_l2(to_np(y[rt]), Y_want) <= BF16_TOL
    assert orc.relative_l2(to_np(xg.grad[rt]), dX_want) <= BF16_TOL
    del xg, y

    # adapter gradients through bilinear probes
    x_np = w.x.float().cpu().numpy()
    dy_np = w.dy.float().cpu().numpy()
    probes = _probes(rng, ads, sp.d_in, sp.d_out)
    want = orc.grad_projections(x_np, ids, ads, dy_np, probes)
    assert want, "no active adapter"
    for a, ad in m.adapters.items():
        a = int(a)
        if a not in want:
            assert ad.A.grad is None and ad.B.grad is None, f"adapter {a} owns no rows but got a gradient"
            continue
        uA, vA, uB, vB = probes[a]
        gA, gB = to_np(ad.A.grad), to_np(ad.B.grad)
        assert orc.relative_l2(_probe(gA, uA, vA), want[a][0]) <= BF16_TOL, f"{cfg} dA of adapter {a}"
        assert orc.relative_l2(_probe(gB, uB, vB), want[a][1]) <= BF16_TOL, f"{cfg} dB of adapter {a}"

    # isolated SGD step: P' = bf16(P - lr G) elementwise with the gradients
    # checked above, and adapters without rows untouched
    before = {int(a): (to_np(ad.A), to_np(ad.B), to_np(ad.A.grad) if ad.A.grad is not None else None,
                       to_np(ad.B.grad) if ad.B.grad is not None else None) for a, ad in m.adapters.items()}
    m.sgd_step(sp.lr)
    torch.cuda.synchronize()
    for a, ad in m.adapters.items():
        a = int(a)
        A0, B0, gA, gB = before[a]
        if a not in want:
            assert np.array_equal(to_np(ad.A), A0) and np.array_equal(to_np(ad.B), B0)
            continue
        assert _sgd_ok(to_np(ad.A), A0, gA, sp.lr), f"{cfg} SGD on A of adapter {a}"
        assert _sgd_ok(to_np(ad.B), B0, gB, sp.lr), f"{cfg} SGD on B of adapter {a}"


def _sgd_ok(got: np.ndarray, P: np.ndarray, G: np.ndarray, lr: float) -> bool:
    """got (bf16 values) is P - lr G rounded to bf16: within half a bf16 ulp
    (2^-9 relative; 2^-8 allowed) plus the fp32 evaluation of the product
    (1e-6 of the operands)."""
    want = P - lr * G
    bound = 2.0 ** -8 * np.abs(want) + 1e-6 * (np.abs(P) + lr * np.abs(G)) + 1e-30
    return bool(np.all(np.abs(got - want) <= bound))


def test_full_size_forward_c1():
    """c1 (forward only, 16 adapters, ~18k rows) at full size, sampled rows."""
    w = workloads.build(workloads.spec("c1"), device=DEV)
    with torch.no_grad():
        y = w.model(w.x, w.ids)
    torch.cuda.synchronize()
    W, b, ads = oracle_params(w.model)
    ids = w.ids.cpu().numpy()
    rows = np.sort(np.random.default_rng(12).choice(w.spec.rows, N_ROWS, replace=False))
    rt = torch.from_numpy(rows).to(DEV)
    want = orc.multi_lora_forward(to_np(w.x[rt]), ids[rows], W, b, ads)
    assert orc.relative_l2(to_np(y[rt]), want) <= BF16_TOL
