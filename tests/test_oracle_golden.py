"""Pin the numpy oracle to the reference's own outputs (golden vectors made by
tests/golden/make_golden.py from the reference's tlora package) and to the
AIMD known-answer trace of the reference's results/phase4_aimd.txt."""

import json
import os

import numpy as np
import pytest

import mlora_oracle as orc

CASES = ["fwd_equiv", "grad_equiv", "isolation", "cfg0_small", "ragged"]


def load_case(golden_dir, name):
    z = np.load(os.path.join(golden_dir, f"{name}.npz"))
    ads = {}
    for a in z["adapter_ids"]:
        a = int(a)
        ads[a] = orc.OracleAdapter(
            A=z[f"A_{a}"].astype(np.float64),
            B=z[f"B_{a}"].astype(np.float64),
            scaling=float(z[f"scaling_{a}"]),
        )
    bias = z["bias"].astype(np.float64) if "bias" in z else None
    return z, ads, bias


@pytest.mark.parametrize("name", CASES)
def test_forward_matches_reference(golden_dir, name):
    z, ads, bias = load_case(golden_dir, name)
    y = orc.multi_lora_forward(z["x"].astype(np.float64), z["ids"], z["W"].astype(np.float64), bias, ads)
    # reference ran in fp32; 1e-6 is the pin of tests/test_equivalence.py:48
    np.testing.assert_allclose(y, z["Y"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", CASES)
def test_backward_and_sgd_match_reference(golden_dir, name):
    z, ads, bias = load_case(golden_dir, name)
    x = z["x"].astype(np.float64)
    y = orc.multi_lora_forward(x, z["ids"], z["W"].astype(np.float64), bias, ads)
    dY = 2.0 * (y - z["target"])  # d/dY of sum-reduction MSE
    dX, dA, dB = orc.multi_lora_backward(x, z["ids"], z["W"].astype(np.float64), ads, dY)
    np.testing.assert_allclose(dX, z["dX"], rtol=1e-5, atol=1e-5)
    lr = float(z["lr"])
    opt_ids = set(int(a) for a in z["opt_ids"])
    for a in ads:
        if f"dA_{a}" in z:
            # the reference accumulates in fp32, the oracle in fp64: pin by
            # relative L2 (the fp32 bound 1e-5) plus an absolute 2e-5,
            # the gradient tolerance of phase4_aimd.py:143-147
            for got, key in ((dA[a], f"dA_{a}"), (dB[a], f"dB_{a}")):
                assert orc.relative_l2(got, z[key]) <= 1e-5
                np.testing.assert_allclose(got, z[key], rtol=0, atol=2e-5)
        else:
            assert dA[a] is None and dB[a] is None
        stepped = a in opt_ids
        A_next = orc.sgd_step(ads[a].A, dA[a] if stepped else None, lr)
        B_next = orc.sgd_step(ads[a].B, dB[a] if stepped else None, lr)
        np.testing.assert_allclose(A_next, z[f"A_next_{a}"], rtol=1e-6, atol=1e-7)
        np.testing.assert_allclose(B_next, z[f"B_next_{a}"], rtol=1e-6, atol=1e-7)
        if not stepped or dA[a] is None:
            # optimizer isolation: bit-identical (tests/test_equivalence.py:137-141)
            assert np.array_equal(z[f"A_next_{a}"], z[f"A_{a}"])
            assert np.array_equal(z[f"B_next_{a}"], z[f"B_{a}"])


def test_nano_split_invariance(golden_dir):
    z, ads, bias = load_case(golden_dir, "cfg0_small")
    x = z["x"].astype(np.float64)
    spans = {a: (s, e) for s, e, a in orc.segments_from_ids(z["ids"])}
    full = orc.multi_lora_forward(x, z["ids"], z["W"].astype(np.float64), bias, ads)
    for n in [1, 2, 4, 5, 8, 9, 16, 32, 40, 100]:
        got = orc.nano_forward_by_count(x, z["W"].astype(np.float64), bias, ads, spans, n)
        np.testing.assert_allclose(got, full, rtol=1e-12, atol=1e-12)


def test_split_ranges_semantics():
    assert orc.split_ranges(10, 3) == [(0, 4), (4, 7), (7, 10)]
    assert orc.split_ranges(5, 0) == [(0, 5)]
    assert orc.split_ranges(3, 8) == [(0, 1), (1, 2), (2, 3)]
    for total in [1, 7, 960, 1001]:
        for n in [1, 2, 4, 8, 16, 33]:
            r = orc.split_ranges(total, n)
            assert r[0][0] == 0 and r[-1][1] == total
            sizes = [e - s for s, e in r]
            assert max(sizes) - min(sizes) <= 1
            assert all(r[i][1] == r[i + 1][0] for i in range(len(r) - 1))


def test_aimd_known_answer(golden_dir):
    kat = json.load(open(os.path.join(golden_dir, "aimd_trace.json")))
    rows = orc.aimd_trace(len(kat["rows"]), kat["tau_ms"] / 1000.0)
    for got, want in zip(rows, kat["rows"]):
        assert got[0] == want["n"]
        assert abs(got[1] - want["ms"]) < 1e-4
        assert got[3] == want["next_n"]
    c = orc.AIMDController(start_n=1, alpha=4, beta=0.5, tau=kat["tau_ms"] / 1000.0, max_n=60)
    for _ in range(len(kat["rows"])):
        c.observe(orc.synthetic_iteration_time(c.n))
    assert c.best_n == kat["best_n"]
    assert abs(c.best * 1000.0 - kat["best_ms"]) < 1e-4


def test_relative_l2():
    a = np.ones(4)
    assert orc.relative_l2(a, a) == 0.0
    assert abs(orc.relative_l2(2 * a, a) - 1.0) < 1e-12


def test_grad_projections_match_full_gradients():
    """The oracle's bilinear gradient probes equal u^T dA v and u^T dB v of the
    full oracle gradients (used by the full-size GPU checks)."""
    rng = np.random.default_rng(3)
    d_in, d_out = 24, 20
    ads = {a: orc.OracleAdapter(A=rng.standard_normal((r, d_in)), B=rng.standard_normal((d_out, r)), scaling=s)
           for a, r, s in ((0, 3, 2.0), (4, 5, 0.5), (7, 2, 1.0))}
    ids = rng.choice([0, 4, 9], size=50)
    x = rng.standard_normal((50, d_in))
    dy = rng.standard_normal((50, d_out))
    W = rng.standard_normal((d_out, d_in))
    _, dA, dB = orc.multi_lora_backward(x, ids, W, ads, dy)
    probes = {a: (rng.standard_normal((4, ad.A.shape[0])), rng.standard_normal((4, d_in)),
                  rng.standard_normal((4, d_out)), rng.standard_normal((4, ad.A.shape[0]))) for a, ad in ads.items()}
    got = orc.grad_projections(x, ids, ads, dy, probes)
    assert set(got) == {0, 4}  # adapter 7 owns no rows
    for a, (pa, pb) in got.items():
        uA, vA, uB, vB = probes[a]
        np.testing.assert_allclose(pa, [u @ dA[a] @ v for u, v in zip(uA, vA)], rtol=1e-10, atol=1e-10)
        np.testing.assert_allclose(pb, [u @ dB[a] @ v for u, v in zip(uB, vB)], rtol=1e-10, atol=1e-10)
