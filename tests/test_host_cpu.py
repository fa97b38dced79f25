"""CPU tests of the host side: the C-ABI library loads and exports every
declared symbol, routing and packing logic, module API parity (constructor,
errors, state_dict keys, seeded initialisation) and the nano-batch / AIMD
logic.  No kernel is launched here."""

import json
import os
import re

import numpy as np
import pytest
import torch

import mlora_oracle as orc
from tlora_b200 import MultiLoRALinear, LoRAAdapter, IndependentLoRALinear, _lib, ops
from tlora_b200.nano import AIMDController, split_ranges

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    hdr = open(os.path.join(ROOT, "include", "mlora.h")).read()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"\b(mlora_\w+)\s*\(", hdr)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    syms = declared_symbols()
    assert len(syms) >= 14
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/mlora.h but not exported"
    assert set(syms) == set(_lib.SIGNATURES), "ctypes signatures out of sync with include/mlora.h"


def test_status_strings_and_sizes_without_gpu():
    lib = _lib.lib()
    assert lib.mlora_status_string(0) == b"ok"
    assert b"workspace" in lib.mlora_status_string(3)
    # plan sizing is pure host logic
    table = ops.AdapterTable.build([0, 1, 2], [4, 70, 1])
    assert list(table.pack_off) == [0, 64, 192] and table.r_pack == 256
    plan = ops.RoutePlan(300, np.array([0, 100, 101, 300], np.int32), np.array([0, 1, 2], np.int32))
    args = ops._CallArgs(300, 256, 128, _lib.BF16, "auto", plan, table, np.ones(3, np.float32))
    zb, wb = args.sizes()
    # 256-row tiles: [0,256) has seg0 (1 chunk), seg1 (2 chunks), seg2 (1 chunk) -> 4; [256,300) seg2 -> 1
    assert zb == 5 * 256 * 64 * 2
    assert wb >= zb
    # invalid routing is rejected with ValueError
    bad = ops.RoutePlan(300, np.array([0, 100, 99, 300], np.int32), np.array([0, 1, 2], np.int32))
    with pytest.raises(ValueError):
        ops._CallArgs(300, 256, 128, _lib.BF16, "auto", bad, table, np.ones(3, np.float32)).sizes()


def test_misaligned_pointers_rejected_before_any_launch():
    """The tensor-core kernels read every tensor with TMA or 16-byte vector
    accesses: an explicit tensor-core call given a pointer that is not 16-byte
    aligned (here a bias slice 2 bytes in) returns MLORA_ERR_UNSUPPORTED before
    any CUDA call, and a pointer not aligned to its element size is rejected on
    every kernel family.  Fake device addresses: nothing is dereferenced."""
    import ctypes

    lib = _lib.lib()
    table = ops.AdapterTable.build([0, 1], [8, 64])
    plan = ops.RoutePlan(300, np.array([0, 100, 300], np.int32), np.array([0, 1], np.int32))
    base = 1 << 40  # 16-byte aligned fake device addresses
    P = [ctypes.c_void_p(base + i * (1 << 30)) for i in range(8)]

    def fwd(impl, bias, x=P[0]):
        args = ops._CallArgs(300, 256, 128, _lib.BF16, impl, plan, table, np.ones(2, np.float32))
        zb, wb = args.sizes()
        return lib.mlora_forward(ctypes.byref(args.prob), ctypes.byref(args.route), x, P[1], bias, P[2], P[3],
                                 P[4], P[5], P[6], wb, None)

    for impl in ("tc", "tc1", "tc2", "tcw"):
        assert fwd(impl, ctypes.c_void_p(base + 2)) == _lib.ERR_UNSUPPORTED  # bias 2 bytes in
        assert fwd(impl, P[7], x=ctypes.c_void_p(base + 8)) == _lib.ERR_UNSUPPORTED
    for impl in ("tc", "simt", "auto"):  # odd address: not even element-aligned
        assert fwd(impl, ctypes.c_void_p(base + 1)) == _lib.ERR_UNSUPPORTED

    args = ops._CallArgs(300, 256, 128, _lib.BF16, "tc", plan, table, np.ones(2, np.float32))
    _, wb = args.sizes()
    assert lib.mlora_backward(ctypes.byref(args.prob), ctypes.byref(args.route), P[0], P[1], P[2], P[3], P[4],
                              P[5], P[6], P[7], ctypes.c_void_p(base + 4), P[1], wb, None) == _lib.ERR_UNSUPPORTED


def test_peer_allreduce_layout_and_checks_without_gpu():
    """Receive-buffer and counter sizes of the peer all-reduce (host
    arithmetic), and the argument checks that run before any CUDA call."""
    import ctypes

    lib = _lib.lib()
    recv, cnt = ctypes.c_size_t(0), ctypes.c_size_t(0)
    # c3: 40,960 rows = 160 tiles, d_out 8192 = 32 blocks of 256 columns
    for world, lt in ((1, 160), (2, 80), (3, 54), (8, 20)):
        assert lib.mlora_ar_layout(160, 8192, world, ctypes.byref(recv), ctypes.byref(cnt)) == 0
        assert recv.value == world * lt * 32 * 256 * 256 * 2
        assert cnt.value >= 4 * (lt + 1) and cnt.value % 256 == 0
    # a partial last block still takes a whole 256-column block
    assert lib.mlora_ar_layout(4, 1000, 2, ctypes.byref(recv), ctypes.byref(cnt)) == 0
    assert recv.value == 2 * 2 * 4 * 256 * 256 * 2
    for bad in ((0, 8192, 2), (4, 1004, 2), (4, 8192, 0), (4, 8192, 9)):
        assert lib.mlora_ar_layout(*bad, ctypes.byref(recv), ctypes.byref(cnt)) == _lib.ERR_INVALID_ARG
    ar = _lib.PeerAr()
    ar.rank, ar.world, ar.n_tiles, ar.d_out = 0, 2, 4, 1000
    # null peer pointers are rejected before anything is launched
    assert lib.mlora_ar_finish(ctypes.byref(ar), 1000, _lib.BF16, 0, 4, None) == _lib.ERR_INVALID_ARG
    assert lib.mlora_ar_wait(ctypes.byref(ar), None) == _lib.ERR_INVALID_ARG
    assert lib.mlora_ar_reset(ctypes.byref(ar), None) == _lib.ERR_INVALID_ARG
    ar.rank = 2
    assert lib.mlora_ar_wait(ctypes.byref(ar), None) == _lib.ERR_INVALID_ARG


@pytest.mark.parametrize("ids", [
    [0, 0, 1, 1, 1, 2],
    [0, 1, 2, 0, 2, 1, 0, 1, 2],
    [3, 3, 3, 0, 1, 1, 1, 1, 1, 9, 0, 0, 3, 1],
    [5] * 7,
    [9, 9, 9],
])
def test_host_routing_covers_every_row_once(ids):
    table = ops.AdapterTable.build([0, 1, 2, 3, 5], [2, 4, 8, 1, 3])
    plan = ops.route(torch.tensor(ids), table, torch.device("cpu"))
    slot_of = table.slot_of()
    rows = len(ids)
    order = plan.perm.numpy() if plan.perm is not None else np.arange(rows)
    assert sorted(order.tolist()) == list(range(rows))
    for s in range(plan.n_seg):
        a, b = plan.seg_start[s], plan.seg_start[s + 1]
        for pos in range(a, b):
            want = slot_of.get(ids[order[pos]], -1)
            assert want == plan.seg_adapter[s]
    # stable: rows of one adapter keep their relative order
    if plan.perm is not None:
        for s in range(plan.n_seg):
            seg = order[plan.seg_start[s]:plan.seg_start[s + 1]]
            assert list(seg) == sorted(seg)
    for i, a in enumerate(table.ids):
        assert plan.active[i] == (a in ids)


def test_grouped_ids_use_runs_without_permutation():
    table = ops.AdapterTable.build([0, 1, 2, 3], [4, 8, 16, 32])
    ids = torch.tensor([0] * 64 + [1] * 128 + [2] * 192 + [3] * 256)
    plan = ops.route(ids, table, torch.device("cpu"))
    assert plan.perm is None
    assert plan.seg_start.tolist() == [0, 64, 192, 384, 640]
    assert plan.seg_adapter.tolist() == [0, 1, 2, 3]


def test_module_api_errors_and_keys():
    with pytest.raises(ValueError):
        MultiLoRALinear(8, 6, {})
    with pytest.raises(ValueError):
        LoRAAdapter(8, 6, 0)
    m = MultiLoRALinear(8, 6, {0: 2, 1: 4})
    assert sorted(m.state_dict().keys()) == sorted(
        ["base.weight", "base.bias", "adapters.0.A", "adapters.0.B", "adapters.1.A", "adapters.1.B"])
    assert not m.base.weight.requires_grad and not m.base.bias.requires_grad
    assert len(list(m.adapter_parameters(1))) == 2
    with pytest.raises(ValueError):
        m(torch.randn(2, 3, 8), torch.zeros(2, dtype=torch.long))
    with pytest.raises(ValueError):
        m(torch.randn(3, 8), torch.zeros(2, dtype=torch.long))
    # no CPU compute path
    with pytest.raises(RuntimeError):
        m(torch.randn(3, 8), torch.zeros(3, dtype=torch.long))


def test_seeded_init_matches_reference(golden_dir):
    """Same constructor RNG sequence as the reference: the golden fixture of
    tests/test_equivalence.py:17-34 is reproduced bit for bit."""
    z = np.load(os.path.join(golden_dir, "fwd_equiv.npz"))
    torch.manual_seed(7)
    m = MultiLoRALinear(16, 12, {0: 2, 1: 4, 2: 8})
    for ad in m.adapters.values():
        torch.nn.init.normal_(ad.B, mean=0.0, std=0.02)
    assert np.array_equal(m.base.weight.detach().numpy(), z["W"])
    assert np.array_equal(m.base.bias.detach().numpy(), z["bias"])
    for a in range(3):
        assert np.array_equal(m.adapters[str(a)].A.detach().numpy(), z[f"A_{a}"])
        assert np.array_equal(m.adapters[str(a)].B.detach().numpy(), z[f"B_{a}"])
    x = torch.randn(9, 16)
    assert np.array_equal(x.numpy(), z["x"])


def test_independent_api():
    m = IndependentLoRALinear(8, 6, 2, bias=False)
    assert m.base.bias is None and m.adapter.scaling == 1.0
    assert IndependentLoRALinear(8, 6, 4, alpha=8).adapter.scaling == 2.0


def test_split_ranges_matches_oracle():
    for total in [1, 5, 60, 960, 40961]:
        for n in [0, 1, 2, 3, 4, 8, 9, 16, 33, 100]:
            assert split_ranges(total, n) == orc.split_ranges(total, n)


def test_aimd_matches_known_answer(golden_dir):
    kat = json.load(open(os.path.join(golden_dir, "aimd_trace.json")))
    c = AIMDController(start_n=1, alpha=4, beta=0.5, tau_ms=kat["tau_ms"], max_n=60)
    for want in kat["rows"]:
        used = c.n
        t_ms = orc.synthetic_iteration_time(used) * 1000.0
        nxt, _ = c.observe(t_ms)
        assert used == want["n"] and nxt == want["next_n"]
    assert c.best_n == kat["best_n"]
    assert abs(c.best_ms - kat["best_ms"]) < 1e-4


def test_aimd_matches_oracle_on_random_landscapes():
    rng = np.random.default_rng(0)
    for _ in range(20):
        times = rng.uniform(1.0, 5.0, size=30)
        a = AIMDController(tau_ms=0.05, max_n=32)
        b = orc.AIMDController(tau=0.05, max_n=32)
        for t in times:
            assert a.observe(t)[0] == b.observe(t)[0]
        assert a.best_n == b.best_n
