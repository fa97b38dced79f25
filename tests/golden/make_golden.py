"""Generate the golden vectors that pin the CPU oracle to the reference.

Run once, in a container where the reference checkout is readable:

    python tests/golden/make_golden.py /path/to/mini-tlora-reproduction

It imports the reference's own ``tlora.multi_lora_linear`` (pure PyTorch,
CPU, fp32), runs forward, autograd backward and per-adapter SGD on small
seeded cases, and writes the inputs and outputs to ``tests/golden/*.npz``.
It also converts the reference's captured AIMD known-answer trace
(``results/phase4_aimd.txt``, UTF-16) into ``aimd_trace.json``.

The cases:
  fwd_equiv   the shapes and seed of tests/test_equivalence.py:17-48
  grad_equiv  the shapes and seed of tests/test_equivalence.py:51-99
              (sum-reduction MSE, interleaved ids)
  isolation   tests/test_equivalence.py:102-143 (only adapter 1 steps)
  cfg0_small  a scaled-down config-0 case: contiguous segments in adapter
              order, alpha = 2r (scaling 2), W ~ N(0, 1/d), A ~ U(-1/sqrt(d),
              1/sqrt(d)), B ~ N(0, 0.02), X ~ N(0, 1), SGD lr = 1e-3
  ragged      uneven segments, an absent adapter and ids not in adapter order
"""

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _save(name, model, x, ids, target, lr, opt_ids=None):
    from torch.nn.functional import mse_loss

    ads = {int(k): v for k, v in model.adapters.items()}
    if opt_ids is None:
        opt_ids = list(ads)
    opts = {a: torch.optim.SGD(model.adapter_parameters(a), lr=lr) for a in opt_ids}
    for o in opts.values():
        o.zero_grad(set_to_none=True)
    xg = x.clone().requires_grad_(True)
    y = model(xg, ids)
    loss = mse_loss(y, target, reduction="sum")
    loss.backward()

    out = {
        "x": x.numpy(),
        "ids": ids.numpy().astype(np.int64),
        "W": model.base.weight.detach().numpy(),
        "target": target.numpy(),
        "lr": np.array(lr),
        "Y": y.detach().numpy(),
        "dX": xg.grad.numpy(),
        "adapter_ids": np.array(sorted(ads), dtype=np.int64),
        "opt_ids": np.array(opt_ids, dtype=np.int64),
    }
    if model.base.bias is not None:
        out["bias"] = model.base.bias.detach().numpy()
    for a, ad in ads.items():
        out[f"A_{a}"] = ad.A.detach().numpy().copy()
        out[f"B_{a}"] = ad.B.detach().numpy().copy()
        out[f"scaling_{a}"] = np.array(ad.scaling)
        if ad.A.grad is not None:
            out[f"dA_{a}"] = ad.A.grad.numpy().copy()
            out[f"dB_{a}"] = ad.B.grad.numpy().copy()
    for o in opts.values():
        o.step()
    for a, ad in ads.items():
        out[f"A_next_{a}"] = ad.A.detach().numpy().copy()
        out[f"B_next_{a}"] = ad.B.detach().numpy().copy()
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"wrote {name}.npz: rows={x.shape[0]} in={x.shape[1]} out={y.shape[1]}")


def main(ref_root):
    sys.path.insert(0, ref_root)
    from tlora.multi_lora_linear import MultiLoRALinear

    torch.set_num_threads(1)

    # tests/test_equivalence.py:17-48
    torch.manual_seed(7)
    m = MultiLoRALinear(16, 12, {0: 2, 1: 4, 2: 8})
    for ad in m.adapters.values():
        torch.nn.init.normal_(ad.B, mean=0.0, std=0.02)
    x = torch.randn(9, 16)
    ids = torch.tensor([0, 1, 2, 0, 2, 1, 0, 1, 2])
    _save("fwd_equiv", m, x, ids, torch.randn(9, 12), 0.1)

    # tests/test_equivalence.py:51-99
    torch.manual_seed(11)
    m = MultiLoRALinear(10, 7, {0: 2, 1: 4, 2: 8})
    for ad in m.adapters.values():
        torch.nn.init.normal_(ad.B, mean=0.0, std=0.02)
    x = torch.randn(12, 10)
    ids = torch.tensor([0, 0, 1, 2, 1, 0, 2, 2, 1, 0, 1, 2])
    _save("grad_equiv", m, x, ids, torch.randn(12, 7), 0.1)

    # tests/test_equivalence.py:102-143
    torch.manual_seed(13)
    m = MultiLoRALinear(8, 6, {0: 2, 1: 4, 2: 8})
    for ad in m.adapters.values():
        torch.nn.init.normal_(ad.B, mean=0.0, std=0.02)
    x = torch.randn(5, 8)
    ids = torch.ones(5, dtype=torch.long)
    _save("isolation", m, x, ids, torch.randn(5, 6), 0.1, opt_ids=[1])

    # config 0, scaled down from 1024 to 64 features and 64/128/192/256 to
    # 4/8/12/16 rows so the fixture stays small.
    torch.manual_seed(0)
    d = 64
    ranks = {0: 4, 1: 8, 2: 16, 3: 32}
    m = MultiLoRALinear(d, d, ranks)
    with torch.no_grad():
        m.base.weight.normal_(0.0, 1.0 / np.sqrt(d))
        m.base.bias.zero_()
        for a, r in ranks.items():
            ad = m.adapters[str(a)]
            ad.alpha = 2.0 * r
            ad.scaling = 2.0
            ad.A.uniform_(-1.0 / np.sqrt(d), 1.0 / np.sqrt(d))
            ad.B.normal_(0.0, 0.02)
    rows = [4, 8, 12, 16]
    x = torch.randn(sum(rows), d)
    ids = torch.cat([torch.full((n,), a) for a, n in zip(ranks, rows)])
    _save("cfg0_small", m, x, ids, torch.randn(sum(rows), d), 1e-3)

    # ragged: ids out of adapter order, adapter 2 absent, a 1-row segment,
    # and an id (9) that no adapter owns (it gets the backbone output only).
    torch.manual_seed(5)
    m = MultiLoRALinear(24, 20, {0: 3, 1: 5, 2: 7, 3: 1})
    with torch.no_grad():
        m.base.bias.normal_(0.0, 0.1)
        for ad in m.adapters.values():
            ad.B.normal_(0.0, 0.05)
    ids = torch.tensor([3, 3, 3, 0, 1, 1, 1, 1, 1, 9, 0, 0, 3, 1])
    x = torch.randn(ids.shape[0], 24)
    _save("ragged", m, x, ids, torch.randn(ids.shape[0], 20), 0.05)

    # AIMD known-answer trace (results/phase4_aimd.txt:26-38)
    raw = open(os.path.join(ref_root, "results", "phase4_aimd.txt"), "rb").read()
    text = raw.decode("utf-16")
    rows = []
    lines = text.splitlines()
    start = next(i for i, l in enumerate(lines) if "SYNTHETIC U-SHAPED" in l)
    for l in lines[start:]:
        parts = l.split()
        if len(parts) >= 4 and parts[0].isdigit() and "->" in l:
            nxt = int(l.rsplit("N=", 1)[1])
            rows.append({"horizon": int(parts[0]), "n": int(parts[1]),
                         "ms": float(parts[2]), "next_n": nxt})
        if l.startswith("Synthetic best observed"):
            best = l
            break
    tau_line = next(l for l in lines if "Local tau" in l)
    tau_ms = float(tau_line.split(":")[1].split()[0])
    best_n = int(best.split("N=")[1].split(",")[0])
    best_ms = float(best.split("time=")[1].split()[0])
    with open(os.path.join(HERE, "aimd_trace.json"), "w") as f:
        json.dump({"source": "results/phase4_aimd.txt", "tau_ms": tau_ms,
                   "rows": rows, "best_n": best_n, "best_ms": best_ms}, f, indent=1)
    print(f"wrote aimd_trace.json: {len(rows)} horizons, best N={best_n}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
