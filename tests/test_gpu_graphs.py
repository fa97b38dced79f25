"""CUDA-graph replay of a training step (tlora_b200.graphs.GraphedTrainStep):
with the routing plan resident in the workspace, the captured step replays the
same kernels as the eager module call, so Y, dX, the adapter gradients and the
SGD-updated weights are bit-identical to eager steps over several replays with
new inputs."""

import copy

import pytest
import torch

from tlora_b200 import MultiLoRALinear, ops
from tlora_b200.graphs import GraphedTrainStep

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _model(dtype, impl):
    torch.manual_seed(0)
    m = MultiLoRALinear(256, 320, {0: 8, 1: 70, 2: 16})
    with torch.no_grad():
        m.base.bias.normal_(0, 0.1)
        for ad in m.adapters.values():
            ad.B.normal_(0, 0.05)
    m = m.to(DEV, dtype)
    m.impl = impl
    return m


@pytest.mark.parametrize("dtype,impl", [(torch.bfloat16, "tc"), (torch.float32, "simt")])
def test_graphed_step_matches_eager(dtype, impl):
    ids = torch.tensor([0] * 300 + [1] * 200 + [2] * 157 + [5] * 20)
    rows = ids.shape[0]
    g = torch.Generator(device=DEV).manual_seed(3)
    xs = [torch.randn(rows, 256, generator=g, device=DEV).to(dtype) for _ in range(4)]
    dys = [torch.randn(rows, 320, generator=g, device=DEV).to(dtype) for _ in range(4)]
    eager = _model(dtype, impl)
    graphed_model = _model(dtype, impl)
    # the graph's warm-up steps update the weights too: start the eager copy from the same point
    step = GraphedTrainStep(graphed_model, xs[0], ids, dys[0], lr=1e-3, warmup=2)
    eager.load_state_dict(graphed_model.state_dict())
    plan = eager.route(ids)
    for i in range(1, 4):
        xe = xs[i].detach().clone().requires_grad_(True)
        for ad in eager.adapters.values():
            ad.A.grad = None
            ad.B.grad = None
        ye = eager(xe, ids, plan=plan)
        ye.backward(dys[i])
        eager.sgd_step(1e-3)
        yg = step(xs[i], dys[i])
        torch.cuda.synchronize()
        assert torch.equal(yg, ye), f"step {i}: Y"
        assert torch.equal(step.dx, xe.grad), f"step {i}: dX"
        for k in eager.adapters:
            assert torch.equal(graphed_model.adapters[k].A, eager.adapters[k].A), f"step {i}: A of {k}"
            assert torch.equal(graphed_model.adapters[k].B, eager.adapters[k].B), f"step {i}: B of {k}"


def test_resident_plan_skips_the_upload():
    """A call with a resident plan gives the same result as one that uploads."""
    m = _model(torch.bfloat16, "tc")
    ids = torch.tensor([0] * 100 + [2] * 60 + [1] * 40)
    x = torch.randn(200, 256, device=DEV).to(torch.bfloat16)
    plan = m.route(ids)
    with torch.no_grad():
        y0 = m(x, ids, plan=plan)
        m.make_resident(plan)
        assert len(plan.resident) == 1
        y1 = m(x, ids, plan=plan)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)
