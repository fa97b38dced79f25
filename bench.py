#!/usr/bin/env python
"""Benchmark of the fused multi-LoRA training step (one JSON line on rank 0).

Default workload (N = 1): the bf16 training step on the MLP up-projection
shape (4096 -> 11008, 8 adapters with ranks alternating 16/64, 65,536 rows):
fused forward, analytic backward (dX, dA, dB) and the isolated SGD step,
through the drop-in module API.  Synthetic seeded inputs and random-init
weights (no dataset).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the reference algorithm's CPU path (the oracle
port of tlora/multi_lora_linear.py, fp32, all host threads) on a bounded
sample of the same workload.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mini-tlora-reproduction_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "tokens/s fused multi-LoRA fwd+bwd (d=4096 bf16, 1–8 B200); % TC/HBM roofline"
UNIT = "tokens/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="c2", choices=["c1", "c2", "c3", "c4"])
    p.add_argument("--ksharded-workload", default="c3", choices=["c2", "c3", "c4"],
                   help="N > 1: workload of the K-sharded nano-batch pipeline (the multi-GPU configuration "
                        "is c3, 8192 x 8192 with 32 jobs)")
    p.add_argument("--rows-scale", type=float, default=1.0,
                   help="scale the rows of every adapter (profiling captures of a smaller case)")
    p.add_argument("--ksharded-comm", default="both", choices=["both", "nccl"],
                   help="N > 1: time the K-sharded pipeline with NCCL's all-reduce only, or also with the "
                        "all-reduce issued from the forward epilogue over peer memory (both)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--kernels", default="auto", choices=["auto", "tc", "tc1", "tc2", "simt"],
                   help="kernel family of the module (tc: per-role best mainloops; tc1: all single-SM; "
                        "tc2: all on 2-SM pairs)")
    p.add_argument("--no-cublas", action="store_true", help="skip the cuBLAS backbone-GEMM context measurement")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="target CPU time of the baseline sample")
    return p.parse_args()


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                f = [v.strip() for v in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    mx = float(f[2])
                except ValueError:
                    continue
                for n, v in zip(names, f[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
            os.unlink(self.path)
        except Exception:
            pass
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- CPU baseline (oracle port)
def cpu_baseline(w, target_s, steps=1):
    """Time the reference algorithm's CPU path (numpy fp32 restatement of
    MultiLoRALinear forward + analytic backward + isolated SGD) on a bounded
    row sample of the workload.  Returns (tokens/s, cores, sample text)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import mlora_oracle as orc
    from threadpoolctl import threadpool_info

    sp = w.spec
    m = w.model
    W = m.base.weight.detach().float().cpu().numpy()
    b = m.base.bias.detach().float().cpu().numpy()
    ads = {int(k): orc.OracleAdapter(a.A.detach().float().cpu().numpy(), a.B.detach().float().cpu().numpy(),
                                     float(a.scaling)) for k, a in m.adapters.items()}
    ids_all = w.ids.cpu().numpy()
    # sample: the same share of rows from every adapter, contiguous per adapter
    def sample(n_rows):
        per = max(1, n_rows // len(sp.counts))
        idx = []
        start = 0
        for c in sp.counts:
            idx.extend(range(start, start + min(per, c)))
            start += c
        idx = np.asarray(idx)
        sel = torch.from_numpy(idx).to(w.x.device)
        x = w.x.detach()[sel].float().cpu().numpy()
        dy = w.dy.detach()[sel].float().cpu().numpy()
        return x, ids_all[idx], dy

    def run(n_rows):
        x, ids, dy = sample(n_rows)
        t0 = time.perf_counter()
        with np.errstate(all="ignore"):  # timed only; the values are not used
            orc.training_step(x, ids, W, b, ads, dy, sp.lr)
        return x.shape[0], time.perf_counter() - t0

    n, t = run(256)  # warm-up + estimate
    rows = int(min(sp.rows, max(256, 256 * target_s / max(t, 1e-3) / max(steps, 1))))
    times = []
    for _ in range(max(1, steps)):
        n, t = run(rows)
        times.append(t)
    threads = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    tps = n / statistics.median(times)
    return tps, threads, f"{n} of {sp.rows} rows ({n // len(sp.counts)} per adapter), fp32, median of {len(times)}"


# ---------------------------------------------------------------- our arm, one GPU
def train_step(m, x, ids, dy, lr, plan=None):
    for ad in m.adapters.values():
        ad.A.grad = None
        ad.B.grad = None
    x.grad = None
    y = m(x, ids, plan=plan)
    y.backward(dy)
    m.sgd_step(lr)
    return y


def ops_sizes(m, w, sp):
    """Bytes of the low-rank intermediate Zt of this workload's routing plan."""
    from tlora_b200 import ops
    A_pack, B_pack, table = m.packed()
    plan = ops.route(w.ids.cpu(), table, A_pack.device)
    sc = np.array([float(a.scaling) for a in m.adapters.values()], dtype=np.float32)
    return ops._CallArgs(sp.rows, sp.d_in, sp.d_out, ops.mlora_dtype(sp.dtype), "auto", plan, table, sc).sizes()[0]


def rooflines(sp, kinds, zbytes, peaks_d, peaks_kind):
    """Per kernel role: algorithmic work per launch / measured average launch
    time against the bound that applies (tensor: the measured sustained bf16
    GEMM peak, the kernels run inside a long step; HBM: the measured copy
    bandwidth).  `traffic` = DRAM bytes per launch from the committed ncu
    captures (profiles/traffic.json) where one exists for this workload."""
    M, di, do = sp.rows, sp.d_in, sp.d_out
    rsum = float(sum(r * n for r, n in zip(sp.ranks, sp.counts)))
    e = 2  # bf16
    rpack = sum(-(-r // 64) * 64 for r in sp.ranks)
    work = {
        "fwd_main": ("tensor", 2.0 * di * do * M + 2.0 * do * rsum),
        "dx_main": ("tensor", 2.0 * di * do * M + 2.0 * di * rsum),
        "fwd_shrink": ("hbm", e * M * di + zbytes + e * rpack * di),
        "bwd_shrink": ("hbm", e * M * do + zbytes + e * rpack * do),
        "dadb_reduce": ("hbm", e * M * (di + do) + 2 * zbytes + e * rpack * (di + do)),
    }
    traffic = {}
    try:
        t = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))
        if sp.name in t and abs(t[sp.name]["scaled_to_rows"] - M) < 1:
            traffic = t[sp.name]["bytes_per_launch"]
    except Exception:
        pass
    out = {}
    for k, (ms_tot, n) in kinds.items():
        if k not in work:
            continue
        bound, w = work[k]
        avg = ms_tot / n
        if bound == "tensor":
            ach = w / (avg / 1000.0) / 1e12
            peak = float(peaks_d.get("bf16_tflops_sustained", peaks_d.get("bf16_tflops")))
            unit, pk = "TFLOP/s", f"{peaks_kind} sustained bf16 GEMM"
        else:
            ach = w / (avg / 1000.0) / 1e9
            peak = float(peaks_d.get("hbm_gbs"))
            unit, pk = "GB/s", f"{peaks_kind} HBM copy"
        out[k] = {"bound": bound, "achieved": round(ach, 1), "peak": peak, "unit": unit,
                  "frac": round(ach / peak, 4), "peak_kind": pk, "algorithmic": w,
                  "traffic": traffic.get(k), "avg_launch_ms": round(avg, 4)}
    return out


def cublas_backbone(w, dev, reps=10):
    """Context only: cuBLAS (torch.matmul) on the backbone GEMM shapes of the
    step, Y = X W^T and dX = dY W, without the LoRA terms."""
    W = w.model.base.weight.detach()
    x = w.x.detach()
    dy = w.dy.detach()
    out = {}
    for name, fn, flops in (("fwd", lambda: torch.matmul(x, W.t()), 2.0 * x.shape[0] * W.shape[0] * W.shape[1]),
                            ("dx", lambda: torch.matmul(dy, W), 2.0 * x.shape[0] * W.shape[0] * W.shape[1])):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        t = e0.elapsed_time(e1) / reps
        out[name] = {"ms": round(t, 4), "tflops": round(flops / (t / 1000.0) / 1e12, 1)}
    return out


def run_single(args, peaks_d, peaks_kind):
    from tlora_b200 import _lib, workloads

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    sp = workloads.spec(args.workload, rows_scale=args.rows_scale)
    w = workloads.build(sp, device=dev)
    m = w.model
    m.impl = args.kernels
    x = w.x.requires_grad_(True)
    lr = sp.lr
    # per-row adapter ids as the job packer produces them: on the host (the
    # reference's packed batches carry host-side spans, phase5c_fused_triton.py:338-377);
    # routing them is a vectorised host pass with no device synchronisation
    ids_host = w.ids.cpu()
    step_fn = (lambda: train_step(m, x, ids_host, w.dy, lr)) if sp.train else (lambda: m(x, ids_host))

    # warm-up
    with torch.no_grad() if not sp.train else torch.enable_grad():
        for _ in range(max(3, args.warmup)):
            step_fn()
    torch.cuda.synchronize()

    # timed region: device-resident inputs (X is 512 MiB, larger than L2)
    clocks = ClockSampler(dev.index)
    launches0 = _lib.launch_count()
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(st)
    with torch.no_grad() if not sp.train else torch.enable_grad():  # forward-only workloads: inference
        for _ in range(args.steps):
            step_fn()
    e1.record(st)
    torch.cuda.synchronize()
    ck = clocks.stop()
    launches = _lib.launch_count() - launches0
    ms = e0.elapsed_time(e1) / args.steps

    # per-kernel device times: the same steps again with the library's
    # per-launch events on (events between two launches also keep the
    # mainloop from overlapping the shrink before it, so this pass is not
    # the one the step time comes from)
    _lib.timing_reset()
    _lib.timing_enable(True)
    with torch.no_grad() if not sp.train else torch.enable_grad():
        for _ in range(args.steps):
            step_fn()
    torch.cuda.synchronize()
    _lib.timing_enable(False)
    ktimes = _lib.timing_read()

    # end to end through the module API: every step copies its X from pinned
    # host memory (on a copy stream, double-buffered so the copy of step i+1
    # overlaps the compute of step i, as a data loader's prefetch does) and
    # reads a probe of the updated adapter weights back to the host, waited
    # for one step later (as a training loop logs its loss), so that the host
    # queues step i+1 while step i runs; the last read is waited for inside the
    # timed region
    x_host = w.x.detach().cpu().pin_memory()
    ids_host = w.ids.cpu()
    bufs = [torch.empty_like(w.x.detach()) for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    copy_stream = torch.cuda.Stream(dev)
    probes = [torch.empty(64, dtype=w.x.dtype).pin_memory() for _ in range(2)]
    read = [torch.cuda.Event() for _ in range(2)]
    a0 = m.adapters["0"].A
    compute = torch.cuda.current_stream(dev)

    def issue_copy(i):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(consumed[i % 2])
            bufs[i % 2].copy_(x_host, non_blocking=True)
            copied[i % 2].record(copy_stream)

    def e2e_step(i):
        compute.wait_event(copied[i % 2])
        issue_copy(i + 1)  # prefetch the next step's X
        xi = bufs[i % 2].detach().requires_grad_(sp.train)
        if sp.train:
            train_step(m, xi, ids_host, w.dy, lr)
        else:
            with torch.no_grad():
                m(xi, ids_host)
        consumed[i % 2].record(compute)
        probes[i % 2].copy_(a0.detach()[0, :64], non_blocking=True)
        read[i % 2].record(compute)
        if i > 0:  # the previous step's result
            read[(i - 1) % 2].synchronize()
            return float(probes[(i - 1) % 2][0])
        return None

    for ev in consumed:
        ev.record(compute)
    issue_copy(0)
    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    n_e2e = max(3, args.steps // 2)
    t0 = time.perf_counter()
    for i in range(2, 2 + n_e2e):
        e2e_step(i)
    read[(1 + n_e2e) % 2].synchronize()  # the last step's result
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / n_e2e
    torch.cuda.synchronize()

    cublas = None if args.no_cublas else cublas_backbone(w, dev)

    rows = sp.rows
    tokens_s = rows / (ms / 1000.0)
    kinds = {k: v for k, v in ktimes.items() if v[1] > 0}
    zbytes = ops_sizes(m, w, sp)
    roofs = rooflines(sp, kinds, zbytes, peaks_d, peaks_kind)
    top = max(kinds, key=lambda k: kinds[k][0]) if kinds else None
    roof = dict(roofs[top]) if top in roofs else None
    step_flops = sp.flops()
    out = {
        "metric": METRIC, "value": round(tokens_s, 1), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded; random-init weights)",
        "config": workload_config(sp),
        "step_tflops": round(step_flops / (ms / 1000.0) / 1e12, 1),
        "step_frac_of_peak": round(step_flops / (ms / 1000.0) / 1e12 /
                                   float(peaks_d.get("bf16_tflops_sustained", 1370.6)), 4),
        "roofline": roof,
        "rooflines": roofs,
        "kernels_ms_per_step": {k: round(v[0] / args.steps, 4) for k, v in kinds.items()},
        "e2e": {"value": round(rows / (e2e_ms / 1000.0), 1), "unit": UNIT, "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": int(w.x.numel() * w.x.element_size()),
                "d2h_bytes_per_step": int(probes[0].numel() * probes[0].element_size())},
        "gpu_launches": int(launches),
        "clocks": ck,
        "cublas_backbone": cublas,
    }
    if not args.no_cpu_baseline:
        tps, cores, smp = cpu_baseline(w, args.cpu_seconds)
        out["cpu_baseline"] = {"value": round(tps, 1), "unit": UNIT, "cores": cores, "kind": "port", "sample": smp}
    return out


def workload_config(sp):
    """The `config` of the single-GPU line (shared by the reference arm)."""
    x_mib = sp.rows * sp.d_in * 2 / 2**20
    return {"workload": f"{sp.name}: {'fwd+bwd+isolated SGD' if sp.train else 'fwd'} "
                        f"d_in={sp.d_in} d_out={sp.d_out} adapters={len(sp.ranks)} ranks={sorted(set(sp.ranks))}",
            "rows": sp.rows, "global_batch": sp.rows, "seq_len": None, "parallelism": "single GPU",
            "l2": f"inputs larger than L2 (X {x_mib:.0f} MiB)" if x_mib > 126 else f"X {x_mib:.0f} MiB"}


def run_reference(args):
    """CPU reference arm: the oracle port of the reference's MultiLoRALinear
    (fp32, all host threads) on a bounded sample per step."""
    from tlora_b200 import workloads

    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    sp = workloads.spec(args.workload)
    w = workloads.build(sp, device=dev, dtype=sp.dtype if dev.type == "cuda" else torch.float32)
    target = max(2.0, min(args.cpu_seconds, 60.0 / max(1, args.steps)))
    tps, cores, smp = cpu_baseline(w, target, steps=args.steps)
    return {
        "metric": METRIC, "value": round(tps, 1), "unit": UNIT, "n_gpus": 0, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "impl": "reference", "dtype": "f32",
        "data": "synthetic (seeded)", "config": workload_config(sp),
        "cpu_baseline": {"value": round(tps, 1), "unit": UNIT, "cores": cores, "kind": "port", "sample": smp},
        "e2e": {"value": round(tps, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "vs_baseline": None,
    }


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    peaks_d, peaks_kind = peaks()
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)))
        return
    if world > 1 or args.gpus > 1:
        from tlora_b200 import overlap
        out = overlap.bench_multi(args, peaks_d, peaks_kind, METRIC, UNIT)
        if out is not None and rank == 0:
            print(json.dumps(out))
        return
    print(json.dumps(run_single(args, peaks_d, peaks_kind)))


if __name__ == "__main__":
    main()
