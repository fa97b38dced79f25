"""Training-step comparison of four ways to train many LoRA jobs on one frozen
backbone: the reference's phase 5A experiment (phase5_gpu_baseline.py:298-480:
modes at :169-243, timing at :246-295) rerun on B200 with this package.

  independent     one IndependentLoRALinear per job, each with its own copy
                  of the backbone (phase5_gpu_baseline.py:124-146, 169-182);
                  one native fused call per job
  naive grouped   one shared module; per job a backbone call plus an adapter
                  call, losses summed (phase5_gpu_baseline.py:185-205)
  shared torch    one backbone call on the concatenated batch, then the
                  per-span LoRA terms in PyTorch ops: the reference's own
                  shared_contiguous_forward (phase5_gpu_baseline.py:208-224)
                  run on the GPU by PyTorch, the reference's shared path
  shared fused    MultiLoRALinear.forward: backbone, routing and every LoRA
                  term in one native call, analytic backward, one native
                  isolated SGD launch

Every mode takes the same step: per-job zero_grad, forward, fp32 MSE loss with
reduction "sum" against a per-job target, backward, per-job SGD (lr 1e-5).
The baselines use torch.optim.SGD per adapter as the reference does; the
fused mode uses MultiLoRALinear.sgd_step, which updates the same tensors.

    python -m tlora_b200.compare [--workload phase5a|c2] [--dtype fp16|bf16] [--warmup 10] [--iters 40]

The phase5a workload is the reference's (4096 -> 4096, jobs ranks 2/4/8/16
with batches 32/64/16/128) in its element type, fp16 (the default; bf16 on
request).  c2 is the 4096 -> 11008 training-step shape (8 jobs, ranks
alternating 16/64, 8192 rows each).  Inputs are seeded synthetic tensors.
"""

from __future__ import annotations

import argparse
import json
import statistics
from dataclasses import dataclass
from typing import Dict, List

import torch
import torch.nn.functional as F

from .multi_lora_linear import IndependentLoRALinear, MultiLoRALinear

LR = 1e-5


@dataclass
class Jobs:
    name: str
    d_in: int
    d_out: int
    rank: Dict[int, int]
    batch: Dict[int, int]

    @property
    def rows(self) -> int:
        return sum(self.batch.values())


def jobs(name: str) -> Jobs:
    if name == "phase5a":
        # phase5_gpu_baseline.py:16-21
        return Jobs("phase5a", 4096, 4096, {0: 2, 1: 4, 2: 8, 3: 16}, {0: 32, 1: 64, 2: 16, 3: 128})
    if name == "c2":
        return Jobs("c2", 4096, 11008, {i: (16 if i % 2 == 0 else 64) for i in range(8)},
                    {i: 8192 for i in range(8)})
    if name == "tiny":  # parity checks
        return Jobs("tiny", 256, 192, {0: 2, 1: 16, 2: 70}, {0: 40, 1: 300, 2: 7})
    raise ValueError(f"unknown workload {name}")


def make_seed(jb: Jobs, device, dtype=torch.bfloat16, seed=2026) -> MultiLoRALinear:
    """phase5_gpu_baseline.py:59-77: shared module with non-zero B."""
    torch.manual_seed(seed)
    m = MultiLoRALinear(jb.d_in, jb.d_out, dict(jb.rank)).to(device=device, dtype=dtype)
    with torch.no_grad():
        for ad in m.adapters.values():
            torch.nn.init.normal_(ad.B, mean=0.0, std=0.01)
    return m


def make_data(jb: Jobs, device, dtype=torch.bfloat16, seed=2027):
    """phase5_gpu_baseline.py:80-123: per-job inputs and targets, their
    concatenation in job order, the job spans and per-row adapter ids."""
    g = torch.Generator(device=device).manual_seed(seed)
    xs, ys, spans, ids = {}, {}, {}, []
    cur = 0
    for aid, b in jb.batch.items():
        xs[aid] = torch.randn(b, jb.d_in, generator=g, device=device, dtype=torch.float32).to(dtype)
        ys[aid] = torch.randn(b, jb.d_out, generator=g, device=device, dtype=torch.float32).to(dtype)
        spans[aid] = (cur, cur + b)
        ids.append(torch.full((b,), aid, dtype=torch.int64))
        cur += b
    x_all = torch.cat([xs[a] for a in jb.batch])
    y_all = torch.cat([ys[a] for a in jb.batch])
    return xs, ys, x_all, y_all, spans, torch.cat(ids).to(device)


def clone_shared(seed: MultiLoRALinear, jb: Jobs) -> MultiLoRALinear:
    ref = seed.base.weight
    m = MultiLoRALinear(jb.d_in, jb.d_out, dict(jb.rank)).to(device=ref.device, dtype=ref.dtype)
    m.load_state_dict(seed.state_dict())
    return m


def make_independent(seed: MultiLoRALinear, jb: Jobs) -> Dict[int, IndependentLoRALinear]:
    """phase5_gpu_baseline.py:124-146: one job per module, backbone copied."""
    ref = seed.base.weight
    out = {}
    for aid, r in jb.rank.items():
        m = IndependentLoRALinear(jb.d_in, jb.d_out, r).to(device=ref.device, dtype=ref.dtype)
        m.base.load_state_dict(seed.base.state_dict())
        m.adapter.load_state_dict(seed.adapters[str(aid)].state_dict())
        out[aid] = m
    return out


def _loss(pred, y):
    return F.mse_loss(pred.float(), y.float(), reduction="sum")


def independent_step(models, opts, xs, ys):
    """phase5_gpu_baseline.py:169-182."""
    for aid, m in models.items():
        opts[aid].zero_grad(set_to_none=True)
        _loss(m(xs[aid]), ys[aid]).backward()
        opts[aid].step()


def naive_grouped_step(model, opts, xs, ys):
    """phase5_gpu_baseline.py:185-205."""
    for o in opts.values():
        o.zero_grad(set_to_none=True)
    total = None
    for aid in opts:
        pred = model.base(xs[aid]) + model.adapters[str(aid)](xs[aid])
        loss = _loss(pred, ys[aid])
        total = loss if total is None else total + loss
    total.backward()
    for o in opts.values():
        o.step()


def shared_torch_forward(model, x_all, spans):
    """phase5_gpu_baseline.py:208-224 with the adapter delta
    (tlora/multi_lora_linear.py:28-31) in PyTorch ops."""
    out = model.base(x_all)
    result = out.clone()
    for aid, (s, e) in spans.items():
        ad = model.adapters[str(aid)]
        xs = x_all[s:e]
        result[s:e] = result[s:e] + F.linear(F.linear(xs, ad.A), ad.B) * ad.scaling
    return result


def shared_torch_step(model, opts, x_all, y_all, spans):
    """phase5_gpu_baseline.py:227-243."""
    for o in opts.values():
        o.zero_grad(set_to_none=True)
    _loss(shared_torch_forward(model, x_all, spans), y_all).backward()
    for o in opts.values():
        o.step()


def shared_fused_step(model, x_all, y_all, ids, plan):
    for ad in model.adapters.values():
        ad.A.grad = None
        ad.B.grad = None
    _loss(model(x_all, ids, plan=plan), y_all).backward()
    model.sgd_step(LR)


def _opts(params_by_job):
    return {aid: torch.optim.SGD(list(ps), lr=LR) for aid, ps in params_by_job.items()}


def build_modes(jb: Jobs, device="cuda", dtype=torch.bfloat16):
    """The four modes, each with its own copy of the same initial weights,
    as {name: (step_fn, adapters_fn)}; adapters_fn returns the mode's
    LoRAAdapter of each job (weights and gradients after a step)."""
    seed = make_seed(jb, device, dtype)
    xs, ys, x_all, y_all, spans, ids = make_data(jb, device, dtype)
    ind = make_independent(seed, jb)
    ind_opts = _opts({a: m.adapter.parameters() for a, m in ind.items()})
    naive = clone_shared(seed, jb)
    naive_opts = _opts({a: naive.adapter_parameters(a) for a in jb.rank})
    sht = clone_shared(seed, jb)
    sht_opts = _opts({a: sht.adapter_parameters(a) for a in jb.rank})
    fused = clone_shared(seed, jb)
    plan = fused.route(ids)

    def ad_of(mod):
        return lambda: {a: mod.adapters[str(a)] for a in jb.rank}

    modes = {
        "independent": (lambda: independent_step(ind, ind_opts, xs, ys),
                        lambda: {a: m.adapter for a, m in ind.items()}),
        "naive grouped": (lambda: naive_grouped_step(naive, naive_opts, xs, ys), ad_of(naive)),
        "shared torch": (lambda: shared_torch_step(sht, sht_opts, x_all, y_all, spans), ad_of(sht)),
        "shared fused": (lambda: shared_fused_step(fused, x_all, y_all, ids, plan), ad_of(fused)),
    }
    param_bytes = {
        "independent": sum(sum(p.numel() * p.element_size() for p in m.parameters()) for m in ind.values()),
        "shared": sum(p.numel() * p.element_size() for p in seed.parameters()),
    }
    data = (seed, xs, x_all, spans, ids)
    return modes, param_bytes, data


def forward_error(seed, xs, x_all, ids, spans):
    """phase5_gpu_baseline.py:331-365: the fused shared forward against the
    per-job formula, computed in fp32 from the same 16-bit weights."""
    with torch.no_grad():
        y = seed(x_all, ids).float()
        W = seed.base.weight.float()
        b = seed.base.bias.float()
        ref = torch.empty_like(y)
        for aid, (s, e) in spans.items():
            ad = seed.adapters[str(aid)]
            x = xs[aid].float()
            ref[s:e] = x @ W.t() + b + ad.scaling * (x @ ad.A.float().t()) @ ad.B.float().t()
        err = (y - ref).abs().max().item()
        rel = ((y - ref).norm() / ref.norm()).item()
    return err, rel


def time_mode(fn, warmup: int, iters: int, rows: int) -> dict:
    """phase5_gpu_baseline.py:246-295: CUDA events around each step."""
    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times: List[float] = []
    for _ in range(iters):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    mean = statistics.mean(times)
    return {"mean_ms": round(mean, 4), "median_ms": round(statistics.median(times), 4),
            "stdev_ms": round(statistics.stdev(times) if len(times) > 1 else 0.0, 4),
            "peak_mb": round(torch.cuda.max_memory_allocated() / 2**20, 1),
            "samples_s": round(rows / (mean / 1000.0), 1)}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--workload", default="phase5a", choices=["phase5a", "c2", "tiny"])
    ap.add_argument("--dtype", default="fp16", choices=["fp16", "bf16"])
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--iters", type=int, default=40)
    a = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("a CUDA device is required")
    jb = jobs(a.workload)
    dt = torch.float16 if a.dtype == "fp16" else torch.bfloat16
    modes, pbytes, (seed, xs, x_all, spans, ids) = build_modes(jb, dtype=dt)
    err, rel = forward_error(seed, xs, x_all, ids, spans)
    print(f"workload {jb.name}: {jb.d_in} -> {jb.d_out}, jobs {len(jb.rank)}, rows {jb.rows}, {a.dtype}")
    print(f"fused shared forward vs per-job formula: max abs error {err:.3e}, relative L2 {rel:.3e}")
    red = 100.0 * (1.0 - pbytes["shared"] / pbytes["independent"])
    print(f"parameter storage: independent {pbytes['independent'] / 2**20:.2f} MB, "
          f"shared {pbytes['shared'] / 2**20:.2f} MB, reduction {red:.2f}%")
    res = {}
    for name, (fn, _) in modes.items():
        res[name] = time_mode(fn, a.warmup, a.iters, jb.rows)
    print(f"{'mode':16s}{'mean ms':>10s}{'median ms':>11s}{'samples/s':>14s}{'peak MB':>10s}")
    for name, r in res.items():
        print(f"{name:16s}{r['mean_ms']:10.3f}{r['median_ms']:11.3f}{r['samples_s']:14.1f}{r['peak_mb']:10.1f}")
    print(json.dumps({"workload": jb.name, "dtype": a.dtype, "rows": jb.rows, "forward_max_abs_err": err, "forward_rel_l2": rel,
                      "param_mb": {k: round(v / 2**20, 2) for k, v in pbytes.items()}, "modes": res}))


if __name__ == "__main__":
    main()
