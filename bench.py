#!/usr/bin/env python
"""Benchmark of the fused multi-LoRA training step (one JSON line on rank 0).

Headline workload, at every GPU count N: the multi-GPU configuration's layer
(8192 x 8192 bf16 backbone, 32 jobs with ranks in {8, 16, 32, 64} and
512-2048 tokens each, 40,960 rows), one fused forward + analytic backward
(dX, dA, dB) + isolated SGD step of the K-sharded nano-batch pipeline
(tlora_b200.overlap.ShardedLayer): the backbone sharded along K over the N
ranks, each nano-batch's partial Y summed across the ranks while the next
nano-batch computes, the nano-batch count from the reference's AIMD
controller.  With N = 1 it is the same pipeline on one rank with no
collective, so the N = 1 .. 8 values form one strong-scaling curve.  At N > 1
the three all-reduce paths (NCCL, peer stores from the epilogue, NVSwitch
multicast) are each timed and checked; the value is the fastest.

The single-GPU line also carries the other bf16 configurations through the
drop-in module API (``workloads``): c2 (the 4096 -> 11008 MLP training step),
c1 (the 4096 x 4096 forward) and c4 (the 8192 x 8192 heterogeneity stress).
Synthetic seeded inputs and random-init weights (no dataset).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --peer-emulated 2      # one-GPU timing of the peer all-reduce

``--impl reference`` times the reference algorithm's CPU path (the oracle
port of tlora/multi_lora_linear.py, fp32, all host threads) on the fixed row
sample of the same workload that the GPU arm's ``cpu_baseline`` times.
"""

import os

# numpy's BLAS sizes its thread pool when numpy loads; torchrun sets
# OMP_NUM_THREADS=1, and the CPU legs below want every host core
os.environ.setdefault("OPENBLAS_NUM_THREADS", str(os.cpu_count() or 1))

import argparse  # noqa: E402
import datetime  # noqa: E402
import json  # noqa: E402
import statistics  # noqa: E402
import subprocess  # noqa: E402
import sys  # noqa: E402
import tempfile  # noqa: E402
import time  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mini-tlora-reproduction_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "tokens/s fused multi-LoRA fwd+bwd (d=4096 bf16, 1–8 B200); % TC/HBM roofline"
UNIT = "tokens/s"
TOL = 2e-2          # bf16 parity bound (relative L2, fp32 accumulation)
CPU_ROWS_PER_ADAPTER = 64   # the CPU baseline's fixed sample: the first rows of every adapter's segment
NANO_SWEEP = (1, 2, 4, 8, 16)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="c3", choices=["c1", "c2", "c3", "c4"],
                   help="headline workload of the K-sharded pipeline (the multi-GPU configuration is c3)")
    p.add_argument("--rows-scale", type=float, default=1.0,
                   help="scale the rows of every adapter (profiling captures of a smaller case)")
    p.add_argument("--comm", default="all", help="N > 1: all-reduce paths to time: all, or a comma list of "
                                                 "nccl, peer, mc")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-workloads", action="store_true", help="N = 1: skip the c1 / c2 / c4 module-API lines")
    p.add_argument("--no-job-parallel", action="store_true", help="N > 1: skip the job-parallel replica line")
    p.add_argument("--kernels", default="auto", choices=["auto", "tc", "tc1", "tc2", "simt"],
                   help="kernel family (tc: per-role best mainloops; tc1: all single-SM; tc2: all on 2-SM pairs)")
    p.add_argument("--no-cublas", action="store_true", help="skip the cuBLAS backbone-GEMM comparison")
    p.add_argument("--peer-emulated", type=int, default=0, metavar="WORLD",
                   help="one-GPU timing of the peer all-reduce with WORLD ranks emulated on the GPU")
    p.add_argument("--nano", default="1,2,4", help="--peer-emulated: nano-batch counts to time")
    p.add_argument("--iters", type=int, default=10, help="--peer-emulated: timed iterations")
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
def cpu_sample(sp, w):
    """The fixed row sample of the CPU legs: the first CPU_ROWS_PER_ADAPTER
    rows of every adapter's segment (fp32 host copies)."""
    idx, start = [], 0
    for c in sp.counts:
        idx.extend(range(start, start + min(CPU_ROWS_PER_ADAPTER, c)))
        start += c
    idx = np.asarray(idx, dtype=np.int64)
    sel = torch.from_numpy(idx).to(w.x.device)
    x = w.x.detach()[sel].float().cpu().numpy()
    dy = w.dy.detach()[sel].float().cpu().numpy()
    return x, w.ids.cpu().numpy()[idx], dy


def cpu_baseline(w, runs=5, warmup=1):
    """Time the reference algorithm's CPU path (numpy fp32 restatement of
    MultiLoRALinear forward + analytic backward + isolated SGD) on the fixed
    row sample with every host core.  Returns (tokens/s, threads, sample
    text, per-run seconds)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import mlora_oracle as orc
    from threadpoolctl import threadpool_info, threadpool_limits

    sp, m = w.spec, w.model
    W = m.base.weight.detach().float().cpu().numpy()
    b = m.base.bias.detach().float().cpu().numpy()
    ads = {int(k): orc.OracleAdapter(a.A.detach().float().cpu().numpy(), a.B.detach().float().cpu().numpy(),
                                     float(a.scaling)) for k, a in m.adapters.items()}
    x, ids, dy = cpu_sample(sp, w)
    cores = os.cpu_count() or 1
    times = []
    with threadpool_limits(limits=cores), np.errstate(all="ignore"):  # timed only; the values are not used
        threads = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
        for i in range(warmup + runs):
            t0 = time.perf_counter()
            orc.training_step(x, ids, W, b, ads, dy, sp.lr)
            if i >= warmup:
                times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    smp = (f"{x.shape[0]} of {sp.rows} rows (the first {CPU_ROWS_PER_ADAPTER} of each of the {len(sp.counts)} "
           f"adapters' segments), fp32 fwd+bwd+SGD, median of {len(times)} runs after {warmup} warm-up")
    return x.shape[0] / med, threads, smp, times


# ---------------------------------------------------------------- configs
def ksharded_config(sp, world):
    """The `config` of the headline line at `world` GPUs (shared by the reference arm)."""
    x_mib = sp.rows * sp.d_in * 2 / 2**20
    return {"workload": f"{sp.name}: fwd+bwd+isolated SGD d_in={sp.d_in} d_out={sp.d_out} adapters={len(sp.ranks)} "
                        f"ranks={sorted(set(sp.ranks))}, backbone K-sharded over {world} GPU(s)",
            "rows": sp.rows, "global_batch": sp.rows, "seq_len": None,
            "parallelism": (f"K-sharded x{world}, partial-Y all-reduce per nano-batch overlapped with compute"
                            if world > 1 else "single GPU (the K-sharded pipeline on one rank, no collective)"),
            "l2": f"inputs larger than L2 (X {x_mib:.0f} MiB)" if x_mib > 126 else f"X {x_mib:.0f} MiB"}


def module_config(sp):
    x_mib = sp.rows * sp.d_in * 2 / 2**20
    return {"workload": f"{sp.name}: {'fwd+bwd+isolated SGD' if sp.train else 'fwd'} "
                        f"d_in={sp.d_in} d_out={sp.d_out} adapters={len(sp.ranks)} ranks={sorted(set(sp.ranks))}",
            "rows": sp.rows, "l2": f"inputs larger than L2 (X {x_mib:.0f} MiB)" if x_mib > 126 else f"X {x_mib:.0f} MiB"}


# ---------------------------------------------------------------- rooflines
def role_work(sp, zbytes, world=1):
    """Algorithmic work per step of each kernel role on one rank (K-shard of
    d_in / world): FLOPs for the tensor-bound mainloops, bytes for the rest."""
    M, do = sp.rows, sp.d_out
    di = sp.d_in // world
    rsum = float(sum(r * n for r, n in zip(sp.ranks, sp.counts)))
    e = 2  # bf16
    rpack = sum(-(-r // 64) * 64 for r in sp.ranks)
    return {
        "fwd_main": ("tensor", 2.0 * di * do * M + (2.0 * do * rsum if world == 1 else 2.0 * do * rsum / world)),
        "dx_main": ("tensor", 2.0 * di * do * M + 2.0 * di * rsum),
        "fwd_shrink": ("hbm", e * M * di + zbytes + e * rpack * di),
        "bwd_shrink": ("hbm", (e * M * do + zbytes) / world + e * rpack * do),
        # one launch (dA and dB) on one GPU; with K-sharding two launches per step, dA over the
        # rank's d_in shard and dB over its share of d_out: their mean per launch
        # dA over the rank's d_in shard and dB over its share of d_out (one launch on one GPU)
        "dadb_reduce": ("hbm", (e * M * di + zbytes + e * rpack * di) + (e * M * do / world + zbytes +
                                                                         e * rpack * do / world)),
    }


def rooflines(sp, kinds, zbytes, peaks_d, peaks_kind, world=1, steps=1):
    """Per kernel role: algorithmic work per step / the role's measured device
    time per step (``steps`` steps timed; a role may launch several times a
    step, e.g. one forward mainloop per nano-batch) against the bound that
    applies.  Tensor-bound roles against the
    measured burst bf16 GEMM peak (``frac``; the sustained peak of a
    seconds-long GEMM loop under the power cap as ``frac_sustained``); HBM
    roles against the measured copy bandwidth.  `traffic` = DRAM bytes per
    launch from the committed ncu captures (profiles/traffic.json) where one
    exists for this workload."""
    work = role_work(sp, zbytes, world)
    traffic = {}
    try:
        t = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))
        key = sp.name if world == 1 else f"{sp.name}@{world}"
        if key in t and abs(t[key]["scaled_to_rows"] - sp.rows) < 1:
            traffic = t[key]["bytes_per_launch"]
    except Exception:
        pass
    out = {}
    for k, (ms_tot, n) in kinds.items():
        if k not in work or n <= 0:
            continue
        bound, w = work[k]
        avg = ms_tot / steps  # device ms of the role per step
        if bound == "tensor":
            ach = w / (avg / 1000.0) / 1e12
            peak = float(peaks_d.get("bf16_tflops"))
            sus = float(peaks_d.get("bf16_tflops_sustained", peak))
            out[k] = {"bound": bound, "achieved": round(ach, 1), "peak": peak, "unit": "TFLOP/s",
                      "frac": round(ach / peak, 4), "peak_kind": f"{peaks_kind} burst bf16 GEMM",
                      "frac_sustained": round(ach / sus, 4), "algorithmic": w, "traffic": traffic.get(k),
                      "ms_per_step": round(avg, 4), "launches_per_step": round(n / steps, 2)}
        else:
            ach = w / (avg / 1000.0) / 1e9
            peak = float(peaks_d.get("hbm_gbs"))
            out[k] = {"bound": bound, "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                      "frac": round(ach / peak, 4), "peak_kind": f"{peaks_kind} HBM copy", "algorithmic": w,
                      "traffic": traffic.get(k), "ms_per_step": round(avg, 4), "launches_per_step": round(n / steps, 2)}
    return out


def cublas_backbone(x, W, dy, dev, reps=10):
    """cuBLAS (torch.matmul) on the backbone GEMM shapes of the step, Y = X W^T
    and dX = dY W, without the LoRA terms, timed in the same run."""
    out = {}
    flops = 2.0 * x.shape[0] * W.shape[0] * W.shape[1]
    for name, fn in (("fwd", lambda: torch.matmul(x, W.t())), ("dx", lambda: torch.matmul(dy, W))):
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


def vs_cublas(roofs, cub):
    """Our mainloop's average launch time over cuBLAS's time for the same
    backbone shape (the mainloop also does the LoRA k-blocks)."""
    if not cub:
        return None
    out = {}
    for role, key in (("fwd_main", "fwd"), ("dx_main", "dx")):
        if role in roofs and key in cub and cub[key]["ms"] > 0:
            out[role] = round(roofs[role]["ms_per_step"] / cub[key]["ms"], 4)
    return out


# ---------------------------------------------------------------- timing
def _world():
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), \
        int(os.environ.get("LOCAL_RANK", "0"))


def timed(fn, iters, dev, world):
    """Device ms per call over `iters` calls, bracketed by a barrier and a
    synchronize on both sides, max over ranks (phase6_two_gpu_overlap.py:283-343)."""
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed_med(fn, iters, dev, world, reps=3):
    """Median of `reps` timings: the collectives' speed varies from one
    measurement to the next on a shared node."""
    return float(statistics.median(timed(fn, iters, dev, world) for _ in range(reps)))


# ---------------------------------------------------------------- self-check of the K-sharded step
def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def reference_rows(w, rows):
    """Y and dX of the unsharded layer on rows `rows`, in fp64 on the GPU
    (a plain restatement of MultiLoRALinear's forward and its analytic
    backward, tlora/multi_lora_linear.py:92-118, phase5d_triton_training.py:287-312)."""
    m = w.model
    W = m.base.weight.detach().double()
    b = m.base.bias.detach().double()
    x, dy = w.x.detach()[rows].double(), w.dy.detach()[rows].double()
    ids = w.ids[rows]
    Y, dX = x @ W.t() + b, dy @ W
    for k, ad in m.adapters.items():
        mask = ids == int(k)
        if not bool(mask.any()):
            continue
        A, B, s = ad.A.detach().double(), ad.B.detach().double(), float(ad.scaling)
        Y[mask] += s * (x[mask] @ A.t()) @ B.t()
        dX[mask] += (s * dy[mask] @ B) @ A
    return Y, dX


def reference_probes(w, probes):
    """u^T dA v and u^T dB v of every active adapter of the unsharded layer in
    fp64 on the GPU, matrix-vector products only: u^T dA v = s (g (B u))^T (x v)
    and u^T dB v = s (g u)^T (x (A^T v)) over the adapter's rows."""
    m, out, start = w.model, {}, 0
    for i, c in enumerate(w.spec.counts):
        a = str(i)
        if c == 0:
            continue
        ad = m.adapters[a]
        A, B, s = ad.A.detach().double(), ad.B.detach().double(), float(ad.scaling)
        xs, g = w.x.detach()[start:start + c].double(), w.dy.detach()[start:start + c].double()
        uA, vA, uB, vB = probes[a]
        pa = s * ((g @ (B @ uA.t())) * (xs @ vA.t())).sum(0)
        pb = s * ((g @ uB.t()) * (xs @ (A.t() @ vB.t()))).sum(0)
        out[a] = (pa, pb)
        start += c
    return out


def ksharded_parity(layer, w, x_p, plan, n_nano, world, dev, n_rows=64, n_probes=8, step=None):
    """One K-sharded training step checked against the unsharded layer
    (fp64), eager or replayed from a graph (``step``): Y and dX on sampled
    rows (dX gathered from the ranks' shards),
    the gradients dA and dB through bilinear probes (each rank's partial
    probe of its d_in shard summed across the ranks), and the SGD update
    elementwise on this rank's shards.  Returns max relative L2 per tensor."""
    g = torch.Generator(device=dev).manual_seed(1234)
    rows = torch.sort(torch.randperm(w.spec.rows, generator=g, device=dev)[:n_rows]).values
    # the timed steps have moved the layer's adapters by SGD: start from the
    # unsharded model's weights, which the reference uses
    A_full, B_full, _ = w.model.packed()
    with torch.no_grad():
        layer.A_pack.copy_(A_full[:, layer.k0:layer.k1])
        layer.B_pack.copy_(B_full)
    A0, B0 = layer.A_pack.clone(), layer.B_pack.clone()
    if step is not None:  # a GraphedShardedStep of this layer and inputs
        y, dx_p = step()
        dA_p, dB = step.grads
    else:
        y, dx_p = layer.step(x_p, plan, w.dy, n_nano, w.spec.lr)
        dA_p, dB = layer.last_grads
    torch.cuda.synchronize(dev)
    Y_ref, dX_ref = reference_rows(w, rows)
    out = {"Y": _rel(y[rows], Y_ref)}
    parts = [dx_p[rows].float().cpu()]
    if world > 1:
        parts = [None] * world
        dist.all_gather_object(parts, dx_p[rows].float().cpu())
    out["dX"] = _rel(torch.cat(parts, 1).to(dev), dX_ref)
    # probes: the same random vectors on every rank (seeded), full d_in length
    d_in, d_out = w.spec.d_in, w.spec.d_out
    probes = {}
    for i, r in enumerate(w.spec.ranks):
        if w.spec.counts[i] == 0:
            continue
        probes[str(i)] = tuple(torch.randn(n_probes, n, generator=g, device=dev, dtype=torch.float64)
                               for n in (r, d_in, d_out, r))
    want = reference_probes(w, probes)
    errs_a, errs_b, sgd_ok = [], [], True
    sgd_bad = {"A": 0, "B": 0}  # elements outside the bound, per tensor
    k0, k1 = layer.k0, layer.k1
    for i in range(layer.table.n):
        a = str(layer.table.ids[i])
        if a not in want:
            continue
        o, r = int(layer.table.pack_off[i]), int(layer.table.rank[i])
        uA, vA, uB, vB = probes[a]
        gA = dA_p[o:o + r].double()       # [r, k1 - k0]
        gB = dB[:, o:o + r].double()      # [d_out, r]
        pa = ((uA @ gA) * vA[:, k0:k1]).sum(1)
        if world > 1:
            dist.all_reduce(pa, op=dist.ReduceOp.SUM)
        pb = ((uB @ gB) * vB).sum(1)
        errs_a.append(_rel(pa, want[a][0]))
        errs_b.append(_rel(pb, want[a][1]))
        # P' = bf16(P - lr G): within 2^-8 relative (half a bf16 ulp, doubled)
        for name, P1, P0, G in (("A", layer.A_pack[o:o + r], A0[o:o + r], dA_p[o:o + r]),
                                ("B", layer.B_pack[:, o:o + r], B0[:, o:o + r], dB[:, o:o + r])):
            exp = P0.double() - w.spec.lr * G.double()
            bound = 2.0 ** -8 * exp.abs() + 1e-6 * (P0.double().abs() + w.spec.lr * G.double().abs()) + 1e-30
            bad = int(((P1.double() - exp).abs() > bound).sum())
            sgd_bad[name] += bad
            sgd_ok = sgd_ok and bad == 0
    out["dA"] = max(errs_a) if errs_a else 0.0
    out["dB"] = max(errs_b) if errs_b else 0.0
    ok = torch.tensor([1.0 if sgd_ok else 0.0], device=dev)
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        t = torch.tensor([out["Y"], out["dA"], out["dB"]], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out["Y"], out["dA"], out["dB"] = (float(v) for v in t.tolist())
    out["sgd_elementwise_ok"] = bool(ok.item() > 0)
    bad = torch.tensor([sgd_bad["A"], sgd_bad["B"]], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(bad, op=dist.ReduceOp.SUM)
    out["sgd_elements_outside"] = {"A": int(bad[0].item()), "B": int(bad[1].item())}
    res = {k: (round(v, 6) if isinstance(v, float) else v) for k, v in out.items()}
    res["tol"] = TOL
    res["ok"] = all(out[k] <= TOL for k in ("Y", "dX", "dA", "dB")) and out["sgd_elementwise_ok"]
    res["checked"] = f"Y, dX on {n_rows} sampled rows; dA, dB through {n_probes} bilinear probes per active adapter; " \
                     "SGD elementwise; reference: the unsharded layer in fp64"
    return res


# ---------------------------------------------------------------- the K-sharded pipeline
def nvlink_roofline(sp, world, ms, comm, peaks_d, link_gbs):
    """Fused compute + collective roofline of a rank's step: the slower of its
    FLOPs at the measured burst bf16 GEMM peak and the bytes it must send over
    NVLink per direction at the measured link bandwidth (NCCL ring and peer
    path: 2 (P-1)/P M d_out 2 bytes; the multicast path: (1 + 1/P) M d_out 2)."""
    peak_tf = float(peaks_d.get("bf16_tflops"))
    flops = sp.flops() / world
    y_bytes = sp.rows * sp.d_out * 2
    nvl = (1.0 + 1.0 / world) * y_bytes if comm == "mc" else 2.0 * (world - 1) / world * y_bytes
    t_tc = flops / (peak_tf * 1e12) * 1e3
    t_nvl = nvl / (link_gbs * 1e9) * 1e3 if link_gbs else 0.0
    tensor = t_tc >= t_nvl
    if tensor:
        ach, peak, unit = flops / (ms / 1e3) / 1e12, peak_tf, "TFLOP/s"
    else:
        ach, peak, unit = nvl / (ms / 1e3) / 1e9, link_gbs, "GB/s"
    return {"bound": "tensor" if tensor else "nvlink", "achieved": round(ach, 1), "peak": round(peak, 1),
            "unit": unit, "frac": round(max(t_tc, t_nvl) / ms, 4), "traffic": None,
            "target_ms": round(max(t_tc, t_nvl), 4), "tensor_ms": round(t_tc, 4), "nvlink_ms": round(t_nvl, 4),
            "nvlink_bytes_per_direction": int(nvl),
            "peaks": f"{peak_tf} TFLOP/s bf16 burst (measured), {link_gbs} GB/s per direction (peer copy, "
                     "measured in this run)"}


def peer_copy_gbs(dev, world, rank, nbytes=512 << 20, iters=5):
    """Per-direction link bandwidth between ranks, measured now with this
    library's plain copy kernel (mlora_peer_copy): every rank writes `nbytes`
    into the next rank's buffer (a CUDA IPC mapping), all ranks at once, so
    each GPU sends and receives `nbytes`; device time, max over ranks."""
    if world < 2:
        return None
    import ctypes

    from tlora_b200 import _lib
    src = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    src.fill_(rank)
    dst = ctypes.c_void_p(0)
    _lib.call("mlora_peer_alloc", nbytes, ctypes.byref(dst))
    h = (ctypes.c_char * 64)()
    _lib.call("mlora_ipc_handle", dst, h)
    handles = [None] * world
    dist.all_gather_object(handles, bytes(h))
    peer = ctypes.c_void_p(0)
    _lib.call("mlora_ipc_open", (ctypes.c_char * 64).from_buffer_copy(handles[(rank + 1) % world]),
              ctypes.byref(peer))
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    def xfer():
        _lib.call("mlora_peer_copy", peer, ctypes.c_void_p(src.data_ptr()), nbytes, stream)

    try:
        xfer()
        ms = timed(xfer, iters, dev, world)
    finally:
        torch.cuda.synchronize(dev)
        dist.barrier()
        _lib.call("mlora_ipc_close", peer)
        dist.barrier()
        _lib.call("mlora_peer_free", dst)
    return round(nbytes / (ms / 1e3) / 1e9, 1)


def one_timeline(layer, step, dev):
    torch.cuda.synchronize(dev)
    layer.timeline = []
    try:
        step()
        try:
            return layer.timeline_ms()
        except Exception as e:  # a timing record only: never fail the bench over it
            return {"error": f"{type(e).__name__}: {e}"[:200]}
    finally:
        layer.timeline = None


def host_and_device(fn, iters, dev, world):
    """(device ms per call, host ms per call to enqueue it) over `iters`
    calls, bracketed as `timed`; both max over ranks.  A host time at the
    device time means the host's launches set the pace."""
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    t0 = time.perf_counter()
    for _ in range(iters):
        fn()
    host = (time.perf_counter() - t0) * 1e3 / iters
    e1.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) / iters, host], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0].item()), float(t[1].item())


def run_path(layer, w, x_p, plan, comm, args, dev, world):
    """Time one all-reduce path of the K-sharded step, each step replayed from
    a CUDA graph (one graph per nano-batch count): the nano-batch sweep, AIMD
    over the real step (phase6b_real_aimd.py:245-302), the timed steps, the
    eager step beside it (device and host time), the overlap accounting, one
    step's phase timeline and the parity check of the graphed step."""
    from tlora_b200 import _lib
    from tlora_b200.nano import AIMDController
    from tlora_b200.overlap import GraphedShardedStep, comm_only

    layer.comm = comm
    n_tiles = (w.spec.rows + 255) // 256
    lr, dy = w.spec.lr, w.dy
    graphs = {}

    def graphed(n, comm_on=True):
        key = (n, comm_on, layer.split)
        if key not in graphs:
            graphs[key] = GraphedShardedStep(layer, x_p, plan, dy, n, lr, comm=comm_on)
        return graphs[key]

    def stepper(n, pipelined=True, comm_on=True):
        return lambda: layer.step(x_p, plan, dy, n, lr, pipelined, comm_on)

    for _ in range(max(3, args.warmup)):
        stepper(1 if world == 1 else 2)()
    torch.cuda.synchronize(dev)
    res = {"allreduce": comm}
    try:
        if world > 1:
            sweep = {n: timed_med(graphed(n), 3, dev, world) for n in NANO_SWEEP if n <= n_tiles}
            ctl = AIMDController(start_n=1, alpha=4, beta=0.5, tau_ms=0.05, max_n=min(32, n_tiles))
            horizons = []
            for _ in range(8):
                n = ctl.n
                t = timed(graphed(n), 3, dev, world)
                nxt, why = ctl.observe(t)
                horizons.append({"n": n, "ms": round(t, 4), "decision": why, "next_n": nxt})
            best_n = min(sweep, key=sweep.get)
            if ctl.best_ms < sweep[best_n] and ctl.best_n in sweep:
                best_n = ctl.best_n
            res["n_sweep_ms"] = {str(k): round(v, 4) for k, v in sweep.items()}
            res["aimd"] = horizons
            res["aimd_best_n"] = ctl.best_n
            # the reference's even nano-batches against a first one half as long
            # (starts the all-reduce chain earlier), at the chosen N
            if best_n > 1:
                layer.split = "ramp"
                t_ramp = timed_med(graphed(best_n), 3, dev, world)
                layer.split = "even"
                t_even = timed_med(graphed(best_n), 3, dev, world)
                res["split_ms"] = {"even": round(t_even, 4), "ramp": round(t_ramp, 4)}
                if t_ramp < t_even:
                    layer.split = "ramp"
        else:
            best_n = 1
        ms = timed_med(graphed(best_n), args.steps, dev, world)
        res["n"] = best_n
        res["split"] = layer.split
        res["ms_per_step"] = round(ms, 4)
        launches0 = _lib.launch_count()
        eager_ms, host_ms = host_and_device(stepper(best_n), args.steps, dev, world)
        res["gpu_launches_per_step"] = round((_lib.launch_count() - launches0) / args.steps, 2)
        res["eager"] = {"ms_per_step": round(eager_ms, 4), "host_enqueue_ms_per_step": round(host_ms, 4)}
        if world > 1:
            t_compute = timed_med(graphed(best_n, comm_on=False), 3, dev, world)
            t_serial = timed_med(stepper(best_n, pipelined=False), 3, dev, world) if comm == "nccl" else None
            y_buf, ctx = layer.forward(x_p, plan, best_n)
            t_comm = timed_med(lambda: comm_only(layer, y_buf, ctx["z"], n_tiles, best_n), 3, dev, world)
            res["overlap"] = {"pipelined_ms": round(ms, 4), "compute_only_ms": round(t_compute, 4),
                              "comm_only_ms": round(t_comm, 4),
                              "serial_ms_eager": round(t_serial, 4) if t_serial is not None else None,
                              "comm_hidden_frac": (round(1.0 - max(0.0, ms - t_compute) / t_comm, 4)
                                                   if t_comm > 0 else None),
                              "comm_only_path": "multicast" if comm == "mc" else "nccl"}
        res["timeline_ms"] = one_timeline(layer, stepper(best_n), dev)
        _lib.clear_device_error()
        res["parity"] = ksharded_parity(layer, w, x_p, plan, best_n, world, dev, step=graphed(best_n))
        torch.cuda.synchronize(dev)
        res["device_error"] = _lib.device_error()
    finally:
        torch.cuda.synchronize(dev)
        graphs.clear()  # before the layer's buffers are released
        layer.split = "even"
    return res


def e2e_ksharded(layer, w, x_p, plan, n, args, dev, world):
    """End to end through the public API (a GraphedShardedStep per input
    buffer) with host buffers: every step copies this rank's X shard from
    pinned host memory (on a copy stream, double-buffered: the copy of step
    i + 1 overlaps step i, as a data loader's prefetch does) and reads a probe
    of the updated adapter weights back to the host (waited for one step
    later, as a training loop logs its loss; the last read inside the timed
    region).  Device time over the loop, barrier and max over ranks."""
    from tlora_b200.overlap import GraphedShardedStep

    x_host = x_p.detach().cpu().pin_memory()
    bufs = [x_p.clone() for _ in range(2)]
    steps = [GraphedShardedStep(layer, b, plan, w.dy, n, w.spec.lr) for b in bufs]
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    copy_stream = torch.cuda.Stream(dev)
    compute = torch.cuda.current_stream(dev)
    probes = [torch.empty(64, dtype=x_p.dtype).pin_memory() for _ in range(2)]
    read = [torch.cuda.Event() for _ in range(2)]
    state = {"i": 0}

    def issue_copy(i):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(consumed[i % 2])
            bufs[i % 2].copy_(x_host, non_blocking=True)
            copied[i % 2].record(copy_stream)

    def step():
        i = state["i"]
        state["i"] += 1
        compute.wait_event(copied[i % 2])
        issue_copy(i + 1)
        steps[i % 2]()
        consumed[i % 2].record(compute)
        probes[i % 2].copy_(layer.A_pack[0, :64], non_blocking=True)
        read[i % 2].record(compute)
        if i > 0:
            read[(i - 1) % 2].synchronize()

    for ev in consumed:
        ev.record(compute)
    issue_copy(0)
    for _ in range(2):
        step()
    n_e2e = max(3, args.steps // 2)
    ms = timed(step, n_e2e, dev, world)
    torch.cuda.synchronize(dev)
    out = {"ms_per_step": round(ms, 4), "h2d_bytes_per_step": int(x_p.numel() * x_p.element_size()) * world,
           "d2h_bytes_per_step": int(probes[0].numel() * probes[0].element_size()) * world,
           "path": "GraphedShardedStep replays, X shard copied from pinned host memory each step"}
    del steps, bufs
    return out


def kernel_times(fn, steps):
    """Per-kernel device times of `steps` calls with the library's per-launch
    events on (a second pass: the events between launches also keep a
    mainloop from overlapping the shrink before it)."""
    from tlora_b200 import _lib
    _lib.timing_reset()
    _lib.timing_enable(True)
    for _ in range(steps):
        fn()
    torch.cuda.synchronize()
    _lib.timing_enable(False)
    return {k: v for k, v in _lib.timing_read().items() if v[1] > 0}


def zsave_bytes(layer, x_p, plan):
    from tlora_b200 import ops
    return ops._CallArgs(x_p.shape[0], x_p.shape[1], layer.B_pack.shape[0], ops.mlora_dtype(x_p.dtype), "auto",
                         plan, layer.table, layer.scaling).sizes()[0]


def run_ours(args, peaks_d, peaks_kind):
    from tlora_b200 import _lib, ops, workloads
    from tlora_b200.overlap import GraphedShardedStep, NativeCompute, ShardedLayer

    world, rank, local = _world()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        sp = workloads.spec(args.workload, rows_scale=args.rows_scale)
        w = workloads.build(sp, device=dev)
        w.model.impl = args.kernels
        bwd_group = dist.new_group(list(range(world))) if world > 1 else None
        layer = ShardedLayer(w.model, rank, world, compute=NativeCompute(args.kernels), bwd_group=bwd_group)
        plan = ops.route(w.ids.cpu(), layer.table, dev)
        x_p = layer.shard_input(w.x)
        comms = ["nccl"]
        if world > 1:
            comms = ["nccl", "peer", "mc"] if args.comm == "all" else [c.strip() for c in args.comm.split(",")]
        paths = {}
        for comm in comms:
            try:
                paths[comm] = run_path(layer, w, x_p, plan, comm, args, dev, world)
            except Exception as e:  # reported beside the other paths, which stand
                paths[comm] = {"allreduce": comm, "error": f"{type(e).__name__}: {e}"[:300]}
                if world > 1:  # every rank raised in the same collective step (or the call failed everywhere)
                    torch.cuda.synchronize(dev)
            finally:
                layer.close()
                layer.comm = "nccl"
        good = {c: r for c, r in paths.items() if "ms_per_step" in r and r.get("parity", {}).get("ok")}
        if not good:
            raise RuntimeError(f"no all-reduce path ran and passed its parity check: {paths}")
        best = min(good, key=lambda c: good[c]["ms_per_step"])
        bres = good[best]
        n = bres["n"]
        layer.comm = best
        layer.split = split = bres.get("split", "even")

        # clocks and launch count over a timed region of the chosen path
        clocks = ClockSampler(dev.index) if rank == 0 else None
        if clocks:
            clocks.start()
            time.sleep(0.3)
        graph = GraphedShardedStep(layer, x_p, plan, w.dy, n, sp.lr)
        ms = timed_med(graph, args.steps, dev, world)
        launches = graph.kernels * args.steps  # this library's kernels in one timed region of K replays
        ck = clocks.stop() if clocks else None
        del graph
        # per-kernel device times of this rank (an eager pass, library events on)
        ksteps = max(3, args.steps // 2)
        kinds = kernel_times(lambda: layer.step(x_p, plan, w.dy, n, sp.lr), ksteps)
        kinds = {k: (v[0], v[1]) for k, v in kinds.items()}
        e2e = e2e_ksharded(layer, w, x_p, plan, n, args, dev, world)
        layer.close()
        zb = zsave_bytes(layer, x_p, plan)
        roofs = rooflines(sp, kinds, zb, peaks_d, peaks_kind, world, steps=ksteps)
        cub = None
        if not args.no_cublas:
            cub = cublas_backbone(x_p, layer.W, w.dy, dev)
        link = peer_copy_gbs(dev, world, rank)
        jp = None
        if world > 1 and not args.no_job_parallel:
            jp = job_parallel(args, rank, world, dev)
        cpu = None
        if rank == 0 and not args.no_cpu_baseline:
            tps, cores, smp, _ = cpu_baseline(w)
            cpu = {"value": round(tps, 1), "unit": UNIT, "cores": cores, "kind": "port", "sample": smp}
        wl = None
        if world == 1 and not args.no_workloads:
            del w, layer, x_p
            torch.cuda.empty_cache()
            wl = module_workloads(args, dev, peaks_d, peaks_kind)
        if world > 1:
            dist.barrier()
        if rank != 0:
            return None
        top = max(kinds, key=lambda k: kinds[k][0]) if kinds else None
        if world == 1:
            roof = dict(roofs[top]) if top in roofs else None
        else:
            roof = nvlink_roofline(sp, world, ms, best, peaks_d, link)
            roof["dominant_kernel"] = top
        out = {
            "metric": METRIC, "value": round(sp.rows / (ms / 1000.0), 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; random-init weights)",
            "config": ksharded_config(sp, world),
            "allreduce": best if world > 1 else None,
            "nano_batches": n,
            "nano_split": split,
            "step_tflops": round(sp.flops() / (ms / 1000.0) / 1e12, 1),
            "step_frac_of_peak": round(sp.flops() / world / (ms / 1000.0) / 1e12 / float(peaks_d["bf16_tflops"]), 4),
            "roofline": roof,
            "rooflines": roofs,
            "kernels_ms_per_step": {k: round(v[0] / ksteps, 4) for k, v in kinds.items()},
            "step_replay": "CUDA graph of the whole step (GraphedShardedStep); the eager step is in ksharded.<path>.eager",
            "cublas_backbone": cub,
            "mainloop_vs_cublas": vs_cublas(roofs, cub),
            "e2e": {"value": round(sp.rows / (e2e["ms_per_step"] / 1000.0), 1), "unit": UNIT, **e2e},
            "gpu_launches": int(launches),
            "clocks": ck,
            "parity": bres["parity"],
            "ksharded": paths,
            "peer_copy_gbs": link,
        }
        if cpu:
            out["cpu_baseline"] = cpu
        if jp:
            out["job_parallel"] = jp
        if wl:
            out["workloads"] = wl
        return out
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


# ---------------------------------------------------------------- other workloads through the module API
def train_step(m, x, ids, dy, lr):
    for ad in m.adapters.values():
        ad.A.grad = None
        ad.B.grad = None
    x.grad = None
    y = m(x, ids)
    y.backward(dy)
    m.sgd_step(lr)
    return y


def module_workloads(args, dev, peaks_d, peaks_kind):
    """c2, c1 and c4 through the drop-in module API (MultiLoRALinear) on one
    GPU: tokens/s, ms per step, and the roofline of every kernel role."""
    from tlora_b200 import ops, workloads

    out = {}
    for name in ("c2", "c1", "c4"):
        try:
            sp = workloads.spec(name)
            w = workloads.build(sp, device=dev)
            m = w.model
            m.impl = args.kernels
            x = w.x.requires_grad_(sp.train)
            ids_host = w.ids.cpu()
            fn = (lambda: train_step(m, x, ids_host, w.dy, sp.lr)) if sp.train else (lambda: m(x, ids_host))
            ctx = torch.enable_grad() if sp.train else torch.no_grad()
            with ctx:
                for _ in range(max(3, args.warmup)):
                    fn()
                ms = timed(fn, args.steps, dev, 1)
                ksteps = max(3, args.steps // 2)
                kinds = kernel_times(fn, ksteps)
            A_pack, B_pack, table = m.packed()
            plan = ops.route(ids_host, table, dev)
            sc = np.array([float(a.scaling) for a in m.adapters.values()], dtype=np.float32)
            zb = ops._CallArgs(sp.rows, sp.d_in, sp.d_out, ops.mlora_dtype(sp.dtype), "auto", plan, table,
                               sc).sizes()[0]
            roofs = rooflines(sp, kinds, zb, peaks_d, peaks_kind, steps=ksteps)
            cub = None if args.no_cublas else cublas_backbone(w.x.detach(), m.base.weight.detach(), w.dy, dev)
            out[name] = {"config": module_config(sp), "value": round(sp.rows / (ms / 1000.0), 1), "unit": UNIT,
                         "ms_per_step": round(ms, 4),
                         "step_tflops": round(sp.flops() / (ms / 1000.0) / 1e12, 1),
                         "step_frac_of_peak": round(sp.flops() / (ms / 1000.0) / 1e12 / float(peaks_d["bf16_tflops"]), 4),
                         "rooflines": roofs, "cublas_backbone": cub, "mainloop_vs_cublas": vs_cublas(roofs, cub)}
            del w, m, x
            torch.cuda.empty_cache()
        except Exception as e:  # a side line: never fail the headline over it
            out[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
    return out


def job_parallel(args, rank, world, dev):
    """Weak scaling without any collective on the data path: every rank trains
    its own set of jobs (c2 per GPU: its own adapters and rows, seeded by
    rank) on its own replica of the frozen backbone."""
    from tlora_b200 import workloads

    sp = workloads.spec("c2")
    sp.seed = sp.seed + 7919 * rank
    w = workloads.build(sp, device=dev)
    m = w.model
    x = w.x.requires_grad_(True)
    ids_host = w.ids.cpu()
    fn = lambda: train_step(m, x, ids_host, w.dy, sp.lr)  # noqa: E731
    for _ in range(3):
        fn()
    ms = timed(fn, max(3, args.steps // 2), dev, world)
    del w, m, x
    torch.cuda.empty_cache()
    return {"workload": "c2 per GPU, each GPU its own adapters on a frozen-backbone replica (no collective)",
            "value": round(world * sp.rows / (ms / 1000.0), 1), "unit": UNIT, "ms_per_step": round(ms, 4),
            "scaling": "weak"}


# ---------------------------------------------------------------- reference arm
def run_reference(args):
    """CPU reference arm: the oracle port of the reference's MultiLoRALinear
    (fp32, all host threads) on the fixed row sample of the headline
    workload, W warm-up and K timed runs.  Rank 0 only."""
    from tlora_b200 import workloads

    world, _, local = _world()
    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    sp = workloads.spec(args.workload, rows_scale=args.rows_scale)
    w = workloads.build(sp, device=dev, dtype=sp.dtype if dev.type == "cuda" else torch.float32)
    tps, cores, smp, times = cpu_baseline(w, runs=max(1, args.steps), warmup=max(1, args.warmup))
    return {
        "metric": METRIC, "value": round(tps, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "impl": "reference", "dtype": "f32",
        "data": "synthetic (seeded)", "config": ksharded_config(sp, world),
        "cpu_baseline": {"value": round(tps, 1), "unit": UNIT, "cores": cores, "kind": "port", "sample": smp},
        "e2e": {"value": round(tps, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "ms_per_step": round(1000.0 * statistics.median(times), 3), "vs_baseline": None,
    }


# ---------------------------------------------------------------- one-GPU peer all-reduce harness
def peer_emulated(args):
    """One-GPU timing of the K-sharded forward with the peer all-reduce issued
    from the epilogue, with `--peer-emulated` ranks emulated on the GPU: each
    emulated rank runs its K-shard's forward mainloop with the push epilogue
    on the main stream, and the owners' finish kernels run on a side stream,
    beside the next nano-batch's mainloops.  Every finish starts after all the
    pushes it waits for, so no kernel waits on a kernel running beside it.
    Prints per nano-batch count the device ms of the plain mainloops (local
    Y), the pushes alone, pushes + finishes in sequence and overlapped, and one
    finish of all tiles alone; the GPU does every rank's work."""
    from tlora_b200 import _lib, ops, peer, workloads
    from tlora_b200.nano import split_ranges
    from tlora_b200.overlap import NativeCompute, ShardedLayer

    dev = torch.device("cuda")
    w = workloads.build(workloads.spec(args.workload, rows_scale=args.rows_scale), device=dev)
    world = args.peer_emulated
    rows, d_out = w.x.shape[0], w.model.base.weight.shape[0]
    layers = [ShardedLayer(w.model, r, world, compute=NativeCompute("auto")) for r in range(world)]
    plan = ops.route(w.ids.cpu(), layers[0].table, dev)
    xs = [L.shard_input(w.x) for L in layers]
    ars = peer.PeerAllReduce.emulated(world, rows, d_out, w.x.dtype, dev)
    ctxs = [dict(L.compute.begin(L, x, plan, y=ars[r].y)) for r, (L, x) in enumerate(zip(layers, xs))]
    for L, c in zip(layers, ctxs):
        L.compute.shrink(c)
    n_tiles = ctxs[0]["n_tiles"]
    main_s = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    ys = [torch.empty(rows, d_out, dtype=w.x.dtype, device=dev) for _ in range(world)]

    def run(n, mode):
        if mode == "main_only":
            for t0, t1 in split_ranges(n_tiles, n):
                for r, (L, c) in enumerate(zip(layers, ctxs)):
                    c["fw"].y = ys[r]
                    L.compute.main(c, t0, t1, expand=r == 0, add_bias=r == 0)
            for r, c in enumerate(ctxs):
                c["fw"].y = ars[r].y
            return
        for a in ars:
            a.reset(main_s)
        for t0, t1 in split_ranges(n_tiles, n):
            for r, (L, c) in enumerate(zip(layers, ctxs)):
                L.compute.push(c, ars[r], t0, t1, expand=r == 0, add_bias=r == 0)
            if mode == "serial":
                for a in ars:
                    a.finish(t0, t1, main_s)
            elif mode == "overlap":
                ev = torch.cuda.Event()
                ev.record(main_s)
                side.wait_event(ev)
                for a in ars:
                    a.finish(t0, t1, side)
        if mode == "serial":
            for a in ars:
                a.wait(main_s)
        elif mode == "overlap":
            for a in ars:
                a.wait(side)
            ev = torch.cuda.Event()
            ev.record(side)
            main_s.wait_event(ev)

    def timed1(fn, iters):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(main_s)
        for _ in range(iters):
            fn()
        e1.record(main_s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    _lib.clear_device_error()
    out = {"workload": f"{w.spec.name} rows={rows} d_out={d_out}, {world} ranks emulated on one GPU", "ms": {}}
    for n in (int(v) for v in args.nano.split(",")):
        out["ms"][str(n)] = {m: round(timed1(lambda: run(n, m), args.iters), 4)
                             for m in ("main_only", "push_only", "serial", "overlap")}
    for a in ars:
        a.reset(main_s)
    for r, (L, c) in enumerate(zip(layers, ctxs)):
        L.compute.push(c, ars[r], 0, n_tiles, expand=r == 0, add_bias=r == 0)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main_s)
    for a in ars:
        a.finish(0, n_tiles, main_s)
    e1.record(main_s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    # every rank reads `world` partials of its rows and writes their sum into `world` copies of Y
    out["finish_all_ms"] = round(ms, 4)
    out["finish_all_gbs"] = round(2.0 * world * rows * d_out * 2 / (ms / 1e3) / 1e9, 1)
    out["device_error"] = _lib.device_error()
    for a in ars:
        a.close()
    return out


def main():
    args = parse()
    world, rank, _ = _world()
    peaks_d, peaks_kind = peaks()
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return
    if args.peer_emulated:
        print(json.dumps(peer_emulated(args)), flush=True)
        return
    out = run_ours(args, peaks_d, peaks_kind)
    if out is not None and rank == 0:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
