"""GPU parity: the native kernels against the numpy oracle (and, for the
reference's own test cases, against the reference's golden outputs).

Tolerances: relative L2 <= 1e-5 in fp32 mode, <= 2e-2 in bf16
mode (fp32 accumulation), for Y, dX, dA, dB and the one-step SGD update.
"""

import os

import numpy as np
import pytest
import torch

import mlora_oracle as orc
from _util import assert_parity, module_step, oracle_step, to_np

from tlora_b200 import MultiLoRALinear, IndependentLoRALinear
from tlora_b200 import workloads

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5
BF16_TOL = 2e-2
DEV = "cuda"


def _golden_module(z):
    ranks = {int(a): int(z[f"A_{int(a)}"].shape[0]) for a in z["adapter_ids"]}
    d_out, d_in = z["W"].shape
    m = MultiLoRALinear(d_in, d_out, ranks, bias="bias" in z)
    with torch.no_grad():
        m.base.weight.copy_(torch.from_numpy(z["W"]))
        if "bias" in z:
            m.base.bias.copy_(torch.from_numpy(z["bias"]))
        for a in ranks:
            ad = m.adapters[str(a)]
            ad.A.copy_(torch.from_numpy(z[f"A_{a}"]))
            ad.B.copy_(torch.from_numpy(z[f"B_{a}"]))
            ad.scaling = float(z[f"scaling_{a}"])
    return m.to(DEV)


@pytest.mark.parametrize("name", ["fwd_equiv", "grad_equiv", "isolation", "cfg0_small", "ragged"])
@pytest.mark.parametrize("ids_on", ["cpu", "cuda"])
def test_golden_fp32(golden_dir, name, ids_on):
    """The reference's own cases (tests/test_equivalence.py shapes and seeds),
    fp32, against the reference's outputs."""
    z = np.load(os.path.join(golden_dir, f"{name}.npz"))
    def fwd_bwd(m):
        x = torch.from_numpy(z["x"]).to(DEV).requires_grad_(True)
        ids = torch.from_numpy(z["ids"]).to(ids_on)
        y = m(x, ids)
        loss = torch.nn.functional.mse_loss(y, torch.from_numpy(z["target"]).to(DEV), reduction="sum")
        loss.backward()
        return x, y

    m = _golden_module(z)
    x, y = fwd_bwd(m)
    assert orc.relative_l2(to_np(y), z["Y"]) <= F32_TOL
    assert orc.relative_l2(to_np(x.grad), z["dX"]) <= F32_TOL
    for a in z["adapter_ids"]:
        a = int(a)
        ad = m.adapters[str(a)]
        if f"dA_{a}" in z:
            assert orc.relative_l2(to_np(ad.A.grad), z[f"dA_{a}"]) <= F32_TOL
            assert orc.relative_l2(to_np(ad.B.grad), z[f"dB_{a}"]) <= F32_TOL
        else:
            assert ad.A.grad is None and ad.B.grad is None
    # isolated SGD with the reference's optimizer usage and with the fused step
    lr = float(z["lr"])
    opt_ids = [int(a) for a in z["opt_ids"]]
    m2 = _golden_module(z)  # same inputs through a second module for the fused step
    fwd_bwd(m2)
    opts = [torch.optim.SGD(m.adapter_parameters(a), lr=lr) for a in opt_ids]
    for o in opts:
        o.step()
    m2.sgd_step(lr, opt_ids)
    torch.cuda.synchronize()
    for a in z["adapter_ids"]:
        a = int(a)
        for mm in (m, m2):
            ad = mm.adapters[str(a)]
            assert orc.relative_l2(to_np(ad.A), z[f"A_next_{a}"]) <= F32_TOL
            assert orc.relative_l2(to_np(ad.B), z[f"B_next_{a}"]) <= F32_TOL
            if a not in opt_ids or f"dA_{a}" not in z:
                # isolation: bit-identical (tests/test_equivalence.py:137-141)
                assert np.array_equal(ad.A.detach().cpu().numpy(), z[f"A_{a}"])
                assert np.array_equal(ad.B.detach().cpu().numpy(), z[f"B_{a}"])


def test_reference_equivalence_suite_on_gpu():
    """tests/test_equivalence.py:17-99 rerun with the new module on the GPU:
    shared vs independent forward and adapter gradients, 1e-6."""
    torch.manual_seed(7)
    ranks = {0: 2, 1: 4, 2: 8}
    shared = MultiLoRALinear(16, 12, ranks)
    refs = {aid: IndependentLoRALinear(16, 12, r) for aid, r in ranks.items()}
    for aid, ref in refs.items():
        ref.base.weight.data.copy_(shared.base.weight.data)
        ref.base.bias.data.copy_(shared.base.bias.data)
        ref.adapter.A.data.copy_(shared.adapters[str(aid)].A.data)
    for ad in shared.adapters.values():
        torch.nn.init.normal_(ad.B, mean=0.0, std=0.02)
    for aid, ref in refs.items():
        ref.adapter.B.data.copy_(shared.adapters[str(aid)].B.data)
    shared = shared.to(DEV)
    refs = {a: r.to(DEV) for a, r in refs.items()}
    x = torch.randn(12, 16, device=DEV)
    ids = torch.tensor([0, 0, 1, 2, 1, 0, 2, 2, 1, 0, 1, 2], device=DEV)
    target = torch.randn(12, 12, device=DEV)
    y = shared(x, ids)
    torch.nn.functional.mse_loss(y, target, reduction="sum").backward()
    y_ref = torch.empty_like(y)
    for aid, ref in refs.items():
        mask = ids == aid
        yr = ref(x[mask])
        y_ref[mask] = yr.detach()
        torch.nn.functional.mse_loss(yr, target[mask], reduction="sum").backward()
        sa = shared.adapters[str(aid)]
        assert torch.allclose(sa.A.grad, ref.adapter.A.grad, atol=1e-6, rtol=1e-6)
        assert torch.allclose(sa.B.grad, ref.adapter.B.grad, atol=1e-6, rtol=1e-6)
    assert torch.allclose(y, y_ref, atol=1e-6, rtol=1e-6)


def test_config0_fp32_full_size():
    """Config 0 at its full size (640 rows, 1024 x 1024) in fp32 mode."""
    w = workloads.build(workloads.spec("c0"), device=DEV)
    got = module_step(w.model, w.x, w.ids, w.dy)
    want = oracle_step(w.model, w.x, w.ids, w.dy)
    assert_parity(got, want, F32_TOL, "c0 fp32")
    # one SGD step, lr 1e-3
    m = w.model
    before = {k: (to_np(a.A), to_np(a.B)) for k, a in m.adapters.items()}
    m.sgd_step(w.spec.lr)
    torch.cuda.synchronize()
    for k, a in m.adapters.items():
        A_next = orc.sgd_step(before[k][0], want[2][int(k)], w.spec.lr)
        B_next = orc.sgd_step(before[k][1], want[3][int(k)], w.spec.lr)
        assert orc.relative_l2(to_np(a.A), A_next) <= F32_TOL
        assert orc.relative_l2(to_np(a.B), B_next) <= F32_TOL


@pytest.mark.parametrize("cfg,scale", [("c1", 0.125), ("c2", 0.0625), ("c3", 0.0625), ("c4", 0.03125)])
@pytest.mark.parametrize("impl", ["tc", "tc1", "tc2", "tcw", "simt"])
def test_bf16_configs_scaled(cfg, scale, impl):
    """bf16 configurations at reduced size: native kernels vs the fp64 oracle
    on the same bf16-rounded inputs."""
    w = workloads.build(workloads.spec(cfg, scale), device=DEV)
    w.model.impl = impl
    got = module_step(w.model, w.x, w.ids, w.dy)
    want = oracle_step(w.model, w.x, w.ids, w.dy)
    assert_parity(got, want, BF16_TOL, f"{cfg} x{scale} {impl}")


@pytest.mark.parametrize("cfg,scale", [("c2", 0.0625), ("c4", 0.03125)])
@pytest.mark.parametrize("impl", ["tc", "tc2", "tcw", "simt"])
def test_fp16_configs_scaled(cfg, scale, impl):
    """fp16, the element type of the reference's GPU kernels
    (phase5c_fused_triton.py, phase5d_triton_training.py): forward, backward
    and the isolated SGD step against the fp64 oracle on the same
    fp16-rounded inputs, within the 16-bit tolerance."""
    w = workloads.build(workloads.spec(cfg, scale), device=DEV, dtype=torch.float16)
    m = w.model
    m.impl = impl
    got = module_step(m, w.x, w.ids, w.dy)
    want = oracle_step(m, w.x, w.ids, w.dy)
    assert_parity(got, want, BF16_TOL, f"{cfg} x{scale} fp16 {impl}")
    before = {int(k): (to_np(a.A), to_np(a.B)) for k, a in m.adapters.items()}
    # dY is N(0, 1) / rows: a learning rate scaled by the rows makes the step
    # large enough to be resolved in fp16 next to the weights
    lr = 0.05 * w.spec.rows
    m.sgd_step(lr)
    torch.cuda.synchronize()
    for k, a in m.adapters.items():
        k = int(k)
        if want[2][k] is None:
            assert np.array_equal(to_np(a.A), before[k][0])
            continue
        step_A = to_np(a.A) - before[k][0]
        step_B = to_np(a.B) - before[k][1]
        assert orc.relative_l2(step_A, -lr * want[2][k]) <= BF16_TOL
        assert orc.relative_l2(step_B, -lr * want[3][k]) <= BF16_TOL


def _edge_module(d_in, d_out, ranks, dtype, seed=0, bias_std=0.1):
    torch.manual_seed(seed)
    m = MultiLoRALinear(d_in, d_out, ranks)
    with torch.no_grad():
        m.base.bias.normal_(0.0, bias_std)
        for ad in m.adapters.values():
            ad.B.normal_(0.0, 0.05)
            ad.scaling = 1.5
    return m.to(device=DEV, dtype=dtype)


EDGE_CASES = {
    # name: (d_in, d_out, ranks, ids builder)
    "ragged_ranks": (256, 192, {0: 1, 1: 127, 2: 128, 3: 129, 4: 64},
                     lambda: [0] * 1 + [1] * 130 + [2] * 5 + [3] * 77 + [4] * 200),
    "empty_and_one_token": (128, 256, {0: 8, 1: 16, 2: 32, 3: 4},
                            lambda: [1] * 1 + [3] * 300 + [2] * 1),
    "many_segments_one_tile": (128, 128, {i: 1 + 7 * i for i in range(10)},
                               lambda: sum(([i] * (3 + i) for i in range(10)), [])),
    "unknown_ids": (128, 128, {0: 8, 5: 16}, lambda: [5] * 40 + [9] * 30 + [0] * 60 + [7] * 3),
    "interleaved": (64, 64, {0: 2, 1: 4, 2: 8}, lambda: [0, 1, 2, 0, 2, 1, 0, 1, 2] * 31),
    "tile_straddle": (192, 320, {0: 16, 1: 48, 2: 80}, lambda: [0] * 100 + [1] * 60 + [2] * 150 + [0] * 40),
    "odd_shape": (200, 136, {0: 3, 1: 70}, lambda: [0] * 129 + [1] * 3),
}


@pytest.mark.parametrize("dtype,impl", [(torch.float32, "simt"), (torch.bfloat16, "tc1"), (torch.bfloat16, "tc2"),
                                        (torch.bfloat16, "tcw"), (torch.float16, "tc1"), (torch.float16, "tc2"),
                                        (torch.float16, "tcw"), (torch.float16, "simt")])
@pytest.mark.parametrize("case", sorted(EDGE_CASES))
def test_edge_cases(case, dtype, impl):
    d_in, d_out, ranks, idf = EDGE_CASES[case]
    m = _edge_module(d_in, d_out, ranks, dtype)
    m.impl = impl
    ids = torch.tensor(idf(), dtype=torch.int64, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(11)
    x = torch.randn(ids.shape[0], d_in, generator=g, device=DEV).to(dtype)
    dy = torch.randn(ids.shape[0], d_out, generator=g, device=DEV).to(dtype)
    tol = F32_TOL if dtype == torch.float32 else BF16_TOL
    assert_parity(module_step(m, x, ids, dy), oracle_step(m, x, ids, dy), tol, case)


@pytest.mark.parametrize("dtype,impl", [(torch.float32, "simt"), (torch.bfloat16, "tc1"), (torch.bfloat16, "tc2"),
                                        (torch.float16, "tc")])
def test_delta_only(dtype, impl):
    """add_base=False: only the LoRA delta (the reference kernel's ADD_BASE=False)."""
    m = _edge_module(256, 256, {0: 8, 1: 16, 2: 64}, dtype, bias_std=0.0)
    m.impl = impl
    ids = torch.tensor([0] * 100 + [1] * 200 + [2] * 37, device=DEV)
    x = torch.randn(ids.shape[0], 256, device=DEV).to(dtype)
    dy = torch.randn(ids.shape[0], 256, device=DEV).to(dtype)
    tol = F32_TOL if dtype == torch.float32 else BF16_TOL
    got = module_step(m, x, ids, dy, add_base=False)
    want = oracle_step(m, x, ids, dy, add_base=False)
    assert_parity(got, want, tol, "delta-only")


def test_tc_matches_simt_bf16():
    """The kernel families agree on the same bf16 inputs; the 1-SM, 2-SM and
    wide 2-SM mainloops accumulate identically (same K order), so they agree
    bit for bit."""
    w = workloads.build(workloads.spec("c1", 0.125), device=DEV)
    outs = {}
    for impl in ("tc", "tc1", "tc2", "tcw", "simt"):
        w.model.impl = impl
        outs[impl] = module_step(w.model, w.x, w.ids, w.dy)
    for u, v in zip(outs["tc"][:2], outs["simt"][:2]):
        assert orc.relative_l2(u, v) <= 1e-2
    for other in ("tc1", "tc2", "tcw"):
        for u, v in zip(outs["tc"][:2], outs[other][:2]):
            assert np.array_equal(u, v)


def test_independent_adapter_forward():
    torch.manual_seed(3)
    ref = IndependentLoRALinear(64, 48, 8)
    with torch.no_grad():
        ref.adapter.B.normal_(0, 0.05)
    ref = ref.to(DEV)
    x = torch.randn(33, 64, device=DEV)
    y = ref(x)
    W, b = to_np(ref.base.weight), to_np(ref.base.bias)
    ad = orc.OracleAdapter(to_np(ref.adapter.A), to_np(ref.adapter.B), ref.adapter.scaling)
    want = to_np(x) @ W.T + b + orc.adapter_delta(to_np(x), ad)
    assert orc.relative_l2(to_np(y), want) <= F32_TOL
    d = ref.adapter(x)
    assert orc.relative_l2(to_np(d), orc.adapter_delta(to_np(x), ad)) <= F32_TOL


def test_no_device_error_word():
    from tlora_b200 import _lib
    assert _lib.device_error() == 0


@pytest.mark.parametrize("dtype,impl", [(torch.float32, "simt"), (torch.bfloat16, "tc")])
def test_staged_backward_matches_backward(dtype, impl):
    """The staged backward (dZ by tile ranges, dB by d_out block ranges, as the
    K-sharded ranks split it) pieces together exactly mlora_backward."""
    from tlora_b200 import ops
    m = _edge_module(256, 640, {0: 8, 1: 70, 2: 16}, dtype)
    m.impl = impl
    ids = torch.tensor([0] * 300 + [1] * 200 + [2] * 157, device=DEV)
    x = torch.randn(ids.shape[0], 256, device=DEV).to(dtype)
    dy = torch.randn(ids.shape[0], 640, device=DEV).to(dtype)
    A_pack, B_pack, table = m.packed()
    plan = ops.route(ids, table, torch.device(DEV))
    st = ops.LayerState(table, np.array([float(a.scaling) for a in m.adapters.values()], np.float32), plan,
                        A_pack, B_pack, impl)
    _, z, xs, _ = ops.forward_raw(x, m.base.weight, m.base.bias, st)
    dx, dA, dB = ops.backward_raw(dy, xs, m.base.weight, z, st, True, True, True)
    bw = ops.StagedBackward(dy, xs, m.base.weight, z, st)
    half_t = bw.n_tiles // 2
    bw.run_dz(0, half_t)
    bw.run_dz(half_t, bw.n_tiles)
    bw.run_dx()
    bw.run_da()
    bw.run_db(0, 2)
    bw.run_db(2, bw.n_db)
    torch.cuda.synchronize()
    assert torch.equal(bw.dx, dx)
    for i in range(table.n):
        o, r = int(table.pack_off[i]), int(table.rank[i])
        assert torch.equal(bw.dA[o:o + r], dA[o:o + r])
        assert torch.equal(bw.dB[:, o:o + r], dB[:, o:o + r])


@pytest.mark.parametrize("impl", ["tc", "tc1", "tc2", "tcw"])
@pytest.mark.parametrize("max_ctas", [2, 3, 7])
def test_scheduler_result_independent_of_cta_count(impl, max_ctas):
    """The persistent kernels hand work items out dynamically; with only a few
    resident CTAs (one 2-SM pair for max_ctas 2 and 3) every item is still
    computed exactly once and the results are bit-identical to a full grid."""
    from tlora_b200 import ops
    m = _edge_module(256, 640, {0: 8, 1: 70, 2: 16}, torch.bfloat16)
    ids = torch.tensor([0] * 300 + [1] * 200 + [2] * 157 + [5] * 40, device=DEV)
    x = torch.randn(ids.shape[0], 256, device=DEV).to(torch.bfloat16)
    dy = torch.randn(ids.shape[0], 640, device=DEV).to(torch.bfloat16)
    A_pack, B_pack, table = m.packed()
    plan = ops.route(ids, table, torch.device(DEV))
    scal = np.array([float(a.scaling) for a in m.adapters.values()], np.float32)
    outs = []
    for cap in (0, max_ctas):
        st = ops.LayerState(table, scal, plan, A_pack, B_pack, impl, cap)
        y, z, xs, _ = ops.forward_raw(x, m.base.weight, m.base.bias, st)
        dx, dA, dB = ops.backward_raw(dy, xs, m.base.weight, z, st, True, True, True)
        torch.cuda.synchronize()
        outs.append((y.clone(), dx.clone(), dA.clone(), dB.clone()))
    (y0, dx0, dA0, dB0), (y1, dx1, dA1, dB1) = outs
    assert torch.equal(y0, y1) and torch.equal(dx0, dx1)
    for i in range(table.n):  # the packs' padding rows/columns are not outputs
        o, r = int(table.pack_off[i]), int(table.rank[i])
        assert torch.equal(dA0[o:o + r], dA1[o:o + r])
        assert torch.equal(dB0[:, o:o + r], dB1[:, o:o + r])


@pytest.mark.parametrize("dtype,impl", [(torch.float32, "simt"), (torch.bfloat16, "tc1"), (torch.bfloat16, "tc2")])
def test_out_rows_writes_the_callers_row_order(dtype, impl):
    """mlora_routing.out_rows: the forward writes row i of the (adapter-sorted)
    input to row out_rows[i] of Y and the backward does the same for dX, bit
    for bit what a separate scatter of the sorted outputs gives."""
    import ctypes
    from tlora_b200 import ops, _lib
    m = _edge_module(256, 200, {0: 8, 1: 70, 2: 16}, dtype)
    m.impl = impl
    ids = torch.tensor([0] * 300 + [1] * 200 + [2] * 157, device=DEV)
    rows = ids.shape[0]
    x = torch.randn(rows, 256, device=DEV).to(dtype)
    dy = torch.randn(rows, 200, device=DEV).to(dtype)
    A_pack, B_pack, table = m.packed()
    plan = ops.route(ids, table, torch.device(DEV))
    scal = np.array([float(a.scaling) for a in m.adapters.values()], np.float32)
    st = ops.LayerState(table, scal, plan, A_pack, B_pack, impl)
    y_sorted, z, _, _ = ops.forward_raw(x, m.base.weight, m.base.bias, st)
    dx_sorted, _, _ = ops.backward_raw(dy, x, m.base.weight, z, st, True, False, False)
    perm = torch.randperm(rows, device=DEV).to(torch.int32)
    st_p = ops.LayerState(table, scal, ops.RoutePlan(rows, plan.seg_start, plan.seg_adapter, perm, plan.active),
                          A_pack, B_pack, impl)
    y, z2, _, _ = ops.forward_raw(x, m.base.weight, m.base.bias, st_p, x_sorted=x)
    dy_in = torch.empty_like(dy)
    dy_in[perm.long()] = dy  # the backward gathers dY by perm back to the sorted rows
    dx, _, _ = ops.backward_raw(dy_in, x, m.base.weight, z2, st_p, True, False, False)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    want_y = torch.empty_like(y_sorted)
    want_y[perm.long()] = y_sorted
    want_dx = torch.empty_like(dx_sorted)
    want_dx[perm.long()] = dx_sorted
    assert torch.equal(y, want_y)
    assert torch.equal(dx, want_dx)


def test_out_rows_outside_the_rows_sets_the_bounds_flag():
    """An out_rows entry outside [0, rows) is not written: the kernel's own
    bounds check skips the store and raises the device error word."""
    from tlora_b200 import ops, _lib
    m = _edge_module(256, 200, {0: 8}, torch.bfloat16)
    ids = torch.zeros(300, dtype=torch.int64, device=DEV)
    x = torch.randn(300, 256, device=DEV).to(torch.bfloat16)
    A_pack, B_pack, table = m.packed()
    plan = ops.route(ids, table, torch.device(DEV))
    bad = torch.arange(300, dtype=torch.int32, device=DEV)
    bad[7] = 300
    st = ops.LayerState(table, np.array([1.5], np.float32),
                        ops.RoutePlan(300, plan.seg_start, plan.seg_adapter, bad, plan.active), A_pack, B_pack, "tc")
    _lib.clear_device_error()
    y, _, _, _ = ops.forward_raw(x, m.base.weight, m.base.bias, st, x_sorted=x)
    torch.cuda.synchronize()
    assert _lib.device_error() & 1
    _lib.clear_device_error()
    assert _lib.device_error() == 0


@pytest.mark.parametrize("impl", ["tc", "simt"])
def test_per_call_error_words_on_two_streams(impl):
    """Two calls running at the same time on two streams, each with its own
    status word (mlora_problem.err_word): the call whose out_rows has an entry
    outside the rows flags bit 0 in its own word only; the other call's word
    and the library-wide word stay zero, and the good call's Y is complete."""
    from tlora_b200 import ops, _lib
    dtype = torch.bfloat16
    m = _edge_module(256, 200, {0: 8}, dtype)
    ids = torch.zeros(300, dtype=torch.int64, device=DEV)
    x = torch.randn(300, 256, device=DEV).to(dtype)
    A_pack, B_pack, table = m.packed()
    plan = ops.route(ids, table, torch.device(DEV))
    bad = torch.arange(300, dtype=torch.int32, device=DEV)
    bad[7] = 300
    good = torch.arange(300, dtype=torch.int32, device=DEV)
    words = [torch.zeros(1, dtype=torch.int32, device=DEV) for _ in range(2)]
    sts = [ops.LayerState(table, np.array([1.5], np.float32),
                          ops.RoutePlan(300, plan.seg_start, plan.seg_adapter, perm, plan.active), A_pack, B_pack,
                          impl, err_word=wd) for perm, wd in ((bad, words[0]), (good, words[1]))]
    _lib.clear_device_error()
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream() for _ in range(2)]
    ys = []
    for st, s in zip(sts, streams):
        with torch.cuda.stream(s):
            ys.append(ops.forward_raw(x, m.base.weight, m.base.bias, st, x_sorted=x)[0])
    torch.cuda.synchronize()
    assert int(words[0].item()) & 1
    assert int(words[1].item()) == 0
    assert _lib.device_error() == 0
    y_ref, _, _, _ = ops.forward_raw(x, m.base.weight, m.base.bias,
                                     ops.LayerState(table, np.array([1.5], np.float32), plan, A_pack, B_pack, impl),
                                     x_sorted=x)
    torch.cuda.synchronize()
    assert torch.equal(ys[1], y_ref)


@pytest.mark.parametrize("impl", ["tc", "tc2", "simt"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_sgd_equals_separate_sgd(impl, dtype):
    """The isolated SGD step fused into the dA / dB reduction's epilogue
    (MLORA_BWD_SGD_A | MLORA_BWD_SGD_B, and MLORA_FUSED_SGD of mlora_backward)
    writes the same gradients and leaves A_pack / B_pack bit-identical to the
    backward followed by the separate SGD pass (mlora_sgd); adapters that own
    no rows are neither read nor written (phase5d_triton_training.py:554-559)."""
    import ctypes
    from tlora_b200 import ops, _lib
    m = _edge_module(320, 272, {0: 8, 1: 100, 2: 3, 3: 64}, dtype)
    ids = torch.tensor([0] * 300 + [1] * 129 + [3] * 40, dtype=torch.int64)  # adapter 2 owns no rows
    x = torch.randn(ids.shape[0], 320, device=DEV).to(dtype)
    dy = torch.randn(ids.shape[0], 272, device=DEV).to(dtype)
    A_pack, B_pack, table = m.packed()
    plan = ops.route(ids, table, torch.device(DEV))
    sc = np.array([1.5, 0.5, 2.0, 1.0], np.float32)
    lr = 0.25
    A0, B0 = A_pack.clone(), B_pack.clone()
    st = ops.LayerState(table, sc, plan, A_pack, B_pack, impl)
    fw = ops.StagedForward(x, m.base.weight, m.base.bias, st)
    fw.shrink_main()
    bw = ops.StagedBackward(dy, x, m.base.weight, fw.z, st)
    bw.run_all()
    pairs = []
    for i in range(table.n):
        if plan.active[i]:
            o, r = int(table.pack_off[i]), int(table.rank[i])
            pairs += [(A_pack[o:o + r], bw.dA[o:o + r]), (B_pack[:, o:o + r], bw.dB[:, o:o + r])]
    ops.sgd_step_(pairs, lr)
    want = [t.clone() for t in (bw.dA, bw.dB, bw.dx, A_pack, B_pack)]
    # fused, staged call
    with torch.no_grad():
        A_pack.copy_(A0)
        B_pack.copy_(B0)
    bw2 = ops.StagedBackward(dy, x, m.base.weight, fw.z, st)
    bw2.run_all(sgd_lr=lr)
    torch.cuda.synchronize()
    for name, a, b in zip(("dA", "dB", "dX", "A", "B"), (bw2.dA, bw2.dB, bw2.dx, A_pack, B_pack), want):
        if name in ("dA", "dB"):  # rows / columns of adapter 2 are never written
            o, r = int(table.pack_off[2]), int(table.rank[2])
            keep = torch.ones_like(a, dtype=torch.bool)
            if name == "dA":
                keep[o:o + r] = False
            else:
                keep[:, o:o + r] = False
            a, b = a[keep], b[keep]
        assert torch.equal(a, b), name
    o, r = int(table.pack_off[2]), int(table.rank[2])
    assert torch.equal(A_pack[o:o + r], A0[o:o + r]) and torch.equal(B_pack[:, o:o + r], B0[:, o:o + r])
    assert not torch.equal(A_pack, A0) and not torch.equal(B_pack, B0)
    # fused through mlora_backward's MLORA_FUSED_SGD flag
    with torch.no_grad():
        A_pack.copy_(A0)
        B_pack.copy_(B0)
    args = ops._CallArgs(ids.shape[0], 320, 272, ops.mlora_dtype(dtype), impl, plan, table, sc)
    _, wb = args.sizes()
    ws = torch.empty(wb, dtype=torch.uint8, device=DEV)
    dA = torch.zeros_like(A_pack)
    dB = torch.zeros_like(B_pack)
    args.prob.flags = _lib.FUSED_SGD
    args.prob.lr = lr
    _lib.call("mlora_backward", ctypes.byref(args.prob), ctypes.byref(args.route), ctypes.c_void_p(dy.data_ptr()),
              ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(m.base.weight.data_ptr()),
              ctypes.c_void_p(A_pack.data_ptr()), ctypes.c_void_p(B_pack.data_ptr()),
              ctypes.c_void_p(fw.z.data_ptr()), None, ctypes.c_void_p(dA.data_ptr()),
              ctypes.c_void_p(dB.data_ptr()), ctypes.c_void_p(ws.data_ptr()), wb,
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert torch.equal(A_pack, want[3]) and torch.equal(B_pack, want[4])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_gather_scatter_rows_round_trip(dtype):
    """mlora_gather_rows / mlora_scatter_rows (the C ABI's row permutation for
    callers that do not use out_rows): dst[i] = src[perm[i]] and back."""
    from tlora_b200 import ops
    src = torch.randn(1000, 72, device=DEV).to(dtype)
    perm = torch.randperm(1000, device=DEV).to(torch.int32)
    g = ops.gather_rows(src, perm)
    torch.cuda.synchronize()
    assert torch.equal(g, src[perm.long()])
    assert torch.equal(ops.scatter_rows(g, perm), src)
