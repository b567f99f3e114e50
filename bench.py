"""Benchmark: GPT2 / Hyena forward tokens/s and ResNet18 images/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Default workload ("gpt2_scaled"): GPT2(vocab 50304, d 1024,
16 heads, 24 layers), seq 1024, 8 sequences per GPU (global batch 8 N, weak
scaling), fp32 storage with TF32 tensor-core contractions, the logits
all-gathered over NVLink when N > 1.  Other workloads: gpt2_small (config 0),
resnet18 (config 2), hyena (config 3).  Inputs and weights are synthetic
(seeded), resident in HBM for ``value``; ``e2e`` runs the same step through
the public API from pinned host token ids and reads back the per-position
argmax ids.  Under torchrun (N > 1) every rank runs its shard; times are the
max over ranks.

``--impl reference`` times the reference algorithm on the host CPU instead:
the reference's own code cannot run here (its wgpu backend needs a graphics
adapter), so the CPU restatement of it (oracle/, fp32 numpy) is timed on a
bounded sample of the same workload, on rank 0 only.
"""

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


# ------------------------------------------------------------------ workloads

class Workload:
    name = ""
    metric = ""
    unit = ""

    def units_per_rank(self, world):
        raise NotImplementedError


class GPT2Scaled(Workload):
    name = "gpt2_scaled"
    metric = "GPT2 fwd tokens/s"
    unit = "tokens/s"
    V, D, H, L, S, B_PER_GPU = 50304, 1024, 16, 24, 1024, 8

    def config(self, world):
        return {"workload": "GPT2(vocab=50304,d=1024,heads=16,layers=24) fwd, seq 1024, "
                            "8 seq/GPU, logits all-gathered",
                "global_batch": self.B_PER_GPU * world, "seq_len": self.S,
                "parallelism": f"dp{world} (batch-sharded inference)",
                "matmul_mode": "tf32", "l2": "inputs larger than L2 (1.4 GB weights)"}

    def rows(self, world):
        return self.B_PER_GPU * world

    def units_per_row(self):
        return self.S

    def build(self, wxx):
        return wxx.nn.GPT2(self.V, self.D, self.H, self.L, max_len=self.S)

    def inputs(self, seed, rows):
        return np.random.default_rng(seed).integers(0, self.V, size=(rows, self.S), dtype=np.uint32)

    def gemm_flops_per_row(self):
        D, S, V, L = self.D, self.S, self.V, self.L
        per_layer = 2 * S * D * D * 4 + 2 * S * D * 4 * D * 2 + 2 * 2 * S * S * D
        return L * per_layer + 2 * S * D * V

    def cpu_sample(self, oracle_init, oracle_models, seed):
        sd = oracle_init.gpt2_state_dict(seed, self.V, self.D, self.H, self.L, self.S)
        ids = self.inputs(seed + 1, 1)
        return (lambda: oracle_models.gpt2_forward(sd, ids, self.H, self.L, fast=True)), self.S


class GPT2Small(GPT2Scaled):
    name = "gpt2_small"
    V, D, H, L, S, B_PER_GPU = 1024, 256, 8, 6, 256, 4

    def config(self, world):
        return {"workload": "GPT2(vocab=1024,d=256,heads=8,layers=6) fwd, batch 4, seq 256",
                "global_batch": self.B_PER_GPU * world, "seq_len": self.S,
                "parallelism": f"dp{world}", "matmul_mode": "tf32",
                "l2": "L2 flushed between steps"}


class ResNet18W(Workload):
    name = "resnet18"
    metric = "ResNet18 inference img/s"
    unit = "img/s"
    B_PER_GPU = 256

    def config(self, world):
        return {"workload": "ResNet18(10) eval, 3x32x32", "global_batch": self.B_PER_GPU * world,
                "seq_len": None, "parallelism": f"dp{world}", "matmul_mode": "tf32",
                "l2": "L2 flushed between steps"}

    def rows(self, world):
        return self.B_PER_GPU * world

    def units_per_row(self):
        return 1

    def build(self, wxx):
        return wxx.nn.ResNet18(num_classes=10)

    def inputs(self, seed, rows):
        return np.random.default_rng(seed).standard_normal((rows, 3, 32, 32)).astype(np.float32)

    def gemm_flops_per_row(self):
        return 74.0e6

    def cpu_sample(self, oracle_init, oracle_models, seed):
        sd = oracle_init.resnet18_state_dict(seed, 10)
        x = self.inputs(seed + 1, 16)
        return (lambda: oracle_models.resnet18_forward(sd, x, fast=True)), 16


class HyenaW(Workload):
    name = "hyena"
    metric = "Hyena fwd tokens/s"
    unit = "tokens/s"
    V, D, NL, ORDER, S, B_GLOBAL = 1024, 256, 6, 4, 8192, 16

    def config(self, world):
        return {"workload": "Hyena(vocab=1024,d=256,layers=6,order=4) fwd, seq 8192, fft 16384",
                "global_batch": self.B_GLOBAL, "seq_len": self.S, "parallelism": f"dp{world}",
                "matmul_mode": "tf32", "l2": "inputs larger than L2"}

    def rows(self, world):
        return self.B_GLOBAL

    def units_per_row(self):
        return self.S

    def build(self, wxx):
        return wxx.nn.Hyena(self.V, d_model=self.D, n_layers=self.NL, order=self.ORDER)

    def inputs(self, seed, rows):
        return np.random.default_rng(seed).integers(0, self.V, size=(rows, self.S), dtype=np.uint32)

    def gemm_flops_per_row(self):
        D, S, o = self.D, self.S, self.ORDER
        h = int(2 * 4 * D / 3)
        per_layer = 2 * S * D * D * 2 + 2 * S * D * o * D + 2 * S * D * h * 3
        return self.NL * per_layer + 2 * S * D * self.V

    def cpu_sample(self, oracle_init, oracle_models, seed):
        sd = oracle_init.hyena_state_dict(seed, self.V, self.D, self.NL, self.ORDER)
        ids = self.inputs(seed + 1, 1)[:, :2048]
        return (lambda: oracle_models.hyena_forward(sd, ids, self.NL, self.ORDER, fast=True)), 2048


WORKLOADS = {w.name: w for w in (GPT2Scaled(), GPT2Small(), ResNet18W(), HyenaW())}


# ------------------------------------------------------------------ helpers

def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="wxx_clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu), "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
            os.unlink(self.path)
        except Exception:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        pw = [num(r[3]) for r in rows if num(r[3]) is not None]
        loaded = [s for s, p in zip(sm, pw) if p is not None and p > 200] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(loaded)) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(pw) if pw else None}


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def time_cpu_sample(wl, seconds=10.0, max_reps=50):
    """Times the oracle's fp32 CPU forward on a bounded sample (>= `seconds`)."""
    from oracle import init as oracle_init, models as oracle_models

    fn, units = wl.cpu_sample(oracle_init, oracle_models, 7)
    fn()  # warm-up (BLAS threads, page faults)
    reps, t0 = 0, time.perf_counter()
    while reps < max_reps:
        fn()
        reps += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return units * reps / dt, units, reps, dt


# ------------------------------------------------------------------ reference arm

def run_reference(args, rank, world):
    if rank != 0:
        return 0
    wl = WORKLOADS[args.workload]
    from oracle import init as oracle_init, models as oracle_models

    fn, units = wl.cpu_sample(oracle_init, oracle_models, 7)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = time.perf_counter() - t0
    value = units * args.steps / dt
    sample = (f"{units} {wl.unit.split('/')[0]} per step of {wl.name} (fp32 numpy restatement of "
              "the reference's kernels; the reference's wgpu path needs a graphics adapter, "
              "unavailable on this box)")
    line = {
        "metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1000 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": wl.config(world), "impl": "reference",
        "cpu_baseline": {"value": value, "unit": wl.unit, "cores": cpu_cores(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ our arm

def run_ours(args, rank, world, local):
    os.environ.setdefault("WXX_DEVICE", str(local))
    import wxx_b200 as wxx
    from wxx_b200.backend import device as dev
    from wxx_b200 import distributed as wd
    from wxx_b200.functional._common import KernelTimer

    wl = WORKLOADS[args.workload]
    dist = wd.init_host_group() if world > 1 else None
    wxx.manual_seed(1234)           # identical replicated weights on every rank
    wxx.set_matmul_mode("tf32")
    model = wl.build(wxx)
    rows_global = wl.rows(world)
    lo, hi = wd.shard_bounds(rows_global, world, rank)
    x_host = wl.inputs(99, rows_global)[lo:hi]
    is_ids = x_host.dtype == np.uint32
    F = wxx.functional

    def upload(a):
        return F.from_numpy(a, dtype=np.uint32) if is_ids else F.from_numpy(a)

    x_dev = upload(x_host)
    comm = wd.NcclCommunicator(rank, world, dist) if world > 1 else None

    def step(inp):
        with wxx.backend.inferenceMode():
            out = model(inp)
        if comm is not None and (hi - lo) * world == rows_global:
            out = comm.allgather(out)
        return out

    def barrier():
        dev.synchronize()
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        step(x_dev)
    barrier()
    gpu_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[0]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")[0].isdigit() else local
    sampler = ClockSampler(gpu_index)
    sampler.start()
    n0 = dev.launch_count()
    e0, e1 = dev.Event(), dev.Event()
    e0.record()
    for _ in range(args.steps):
        out = step(x_dev)
    e1.record()
    barrier()
    launches = (dev.launch_count() - n0) / args.steps
    log_path = os.environ.get("WXX_LAUNCH_LOG")
    if log_path and rank == 0:
        with open(log_path, "w") as f:
            json.dump({"before_timed": n0, "per_step": launches}, f)
    ms = e0.elapsed_ms(e1) / args.steps
    clocks = sampler.stop()
    if dist is not None:
        import torch

        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    units_total = rows_global * wl.units_per_row()
    value = units_total / (ms / 1000.0)

    # e2e: pinned host ids -> device -> step -> argmax over the last axis -> host ids
    pin_in = dev.PinnedHostBuffer(x_host.nbytes)
    pin_in.as_numpy(x_host.dtype, x_host.shape)[...] = x_host
    res_rows = (hi - lo) * (wl.units_per_row() if wl.name != "resnet18" else 1)
    pin_out = dev.PinnedHostBuffer(max(4, res_rows * 4))

    from wxx_b200.Tensor import Tensor

    def e2e_step():
        t = Tensor._empty(list(x_host.shape), "u32" if is_ids else "f32")
        wxx.backend.lib.F.wxx_memcpy_h2d(t.buffer.ptr, pin_in.ptr, x_host.nbytes)
        logits = step(t)
        local_logits = logits if comm is None else logits.narrow(0, lo, hi - lo)
        ids = F.max(local_logits, -1)[1]
        wxx.backend.lib.F.wxx_memcpy_d2h_async(pin_out.ptr, ids.ptr, ids.nbytes)
        return ids.nbytes

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    e2 = dev.Event().record()
    d2h = 0
    for _ in range(args.steps):
        d2h = e2e_step()
    e3 = dev.Event().record()
    barrier()
    e2e_ms = e2.elapsed_ms(e3) / args.steps
    if dist is not None:
        import torch

        t = torch.tensor([e2e_ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = units_total / (e2e_ms / 1000.0)

    # roofline of the dominant kernel (the tcgen05 GEMM): one forward with every
    # GEMM launch bracketed by CUDA events on the library stream.
    with KernelTimer() as kt:
        with wxx.backend.inferenceMode():
            model(x_dev)
    dev.synchronize()
    ks = kt.summary()
    peaks, peak_kind = load_peaks()
    tf32_peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]) / 2.0
    achieved = ks["flops"] / (ks["ms"] / 1000.0) / 1e12 if ks["ms"] > 0 else 0.0
    roofline = {
        "kernel": "tc_gemm_kernel (tcgen05 kind::tf32, TMA-fed, TMEM accumulators)",
        "bound": "tensor", "achieved": achieved, "peak": tf32_peak, "unit": "TFLOP/s",
        "frac": achieved / tf32_peak, "traffic": None,
        "peak_basis": f"{peak_kind} bf16 dense TFLOP/s / 2 (B200 TF32 rate is half of BF16)",
        "gemm_share_of_step": ks["ms"] / ms if ms > 0 else None,
        "gemm_launches_per_step": ks["launches"],
    }

    line = {
        "metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak" if wl.name.startswith("gpt2") else "strong", "vs_baseline": None,
        "dtype": "f32 (tf32 tensor-core products)", "data": "synthetic",
        "config": wl.config(world), "roofline": roofline, "clocks": clocks,
        "gpu_launches": int(round(launches * args.steps)),
        "e2e": {"value": e2e_value, "unit": wl.unit,
                "h2d_bytes_per_step": int(x_host.nbytes), "d2h_bytes_per_step": int(d2h),
                "includes": "pinned H2D of inputs, forward, all-gather, argmax, D2H of ids"},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, units, reps, dt = time_cpu_sample(wl, seconds=args.cpu_seconds)
        line["cpu_baseline"] = {
            "value": v, "unit": wl.unit, "cores": cpu_cores(), "kind": "port",
            "sample": f"{reps} x {units} {wl.unit.split('/')[0]} of {wl.name} in {dt:.1f} s "
                      "(fp32 numpy restatement, host BLAS threads)"}
    if comm is not None:
        comm.destroy()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="gpt2_scaled")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_ours(args, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
