"""GPU check of the phase 5A comparison harness (tlora_b200.compare): the
four training-step modes (independent jobs, naive grouped, shared with the
LoRA terms in PyTorch ops, shared fused native) compute the same gradients
from the same weights, and the fused shared forward matches the per-job
formula (phase5_gpu_baseline.py:331-365), within the bf16 tolerance."""

import numpy as np
import pytest
import torch

import mlora_oracle as orc
from tlora_b200 import compare

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def _np(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def test_modes_compute_the_same_gradients(monkeypatch):
    monkeypatch.setattr(compare, "LR", 0.0)  # keep the weights; compare the gradients of one step
    jb = compare.jobs("tiny")
    modes, pbytes, (seed, xs, x_all, spans, ids) = compare.build_modes(jb)
    grads = {}
    for name, (step, adapters) in modes.items():
        step()
        torch.cuda.synchronize()
        grads[name] = {a: (_np(ad.A.grad), _np(ad.B.grad)) for a, ad in adapters().items()}
    ref = grads["shared torch"]
    for name, g in grads.items():
        for a in jb.rank:
            for i, what in enumerate(("A", "B")):
                err = orc.relative_l2(g[a][i], ref[a][i])
                assert err <= BF16_TOL, f"{name}: d{what} of job {a} differs, relative L2 {err:.3e}"
    # one backbone for all jobs instead of one per job
    n_jobs = len(jb.rank)
    assert pbytes["independent"] > (n_jobs - 1) * pbytes["shared"] * 0.9
    _, rel = compare.forward_error(seed, xs, x_all, ids, spans)
    assert rel <= BF16_TOL


def test_sgd_step_moves_adapters_like_torch_sgd(monkeypatch):
    """The fused mode's native isolated SGD moves each adapter like
    torch.optim.SGD in the PyTorch shared mode (a large learning rate, so
    that the update is well above the bf16 rounding of the weights)."""
    monkeypatch.setattr(compare, "LR", 1e-2)
    jb = compare.jobs("tiny")
    modes, _, _ = compare.build_modes(jb)
    before = {a: (_np(ad.A), _np(ad.B)) for a, ad in modes["shared fused"][1]().items()}
    for name in ("shared torch", "shared fused"):
        modes[name][0]()
    torch.cuda.synchronize()
    got, want = modes["shared fused"][1](), modes["shared torch"][1]()
    for a in jb.rank:
        for i, what in enumerate(("A", "B")):
            d_got = _np((got[a].A, got[a].B)[i]) - before[a][i]
            d_want = _np((want[a].A, want[a].B)[i]) - before[a][i]
            err = orc.relative_l2(d_got, d_want)
            assert err <= BF16_TOL, f"job {a}: {what} update differs, relative L2 {err:.3e}"
