"""Benchmark: GPT2 / Hyena forward tokens/s and ResNet18 images/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Default workload ("gpt2_scaled"): GPT2(vocab 50304, d 1024,
16 heads, 24 layers), seq 1024, 8 sequences per GPU (global batch 8 N, weak
scaling), fp32 storage with TF32 tensor-core contractions.  A step is the
forward plus its output (the argmax token id of every position; ResNet18's
logits), all-gathered over NVLink when N > 1.  The step is recorded once as
a CUDA graph and replayed (``--eager`` launches kernel by kernel).  Other
workloads: gpt2_small (config 0), resnet18 (config 2), hyena (config 3).
Inputs and weights are synthetic (seeded), resident in HBM for ``value``;
``e2e`` runs the same step through the public API from pinned host inputs and
reads the gathered outputs back.  Under torchrun (N > 1) every rank runs its
shard; times are the max over ranks.

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

L2_FLUSHED = ("L2 flushed between steps: a 256 MB write, then a 256 MB read of a second "
              "buffer, outside the timed events (the inputs are evicted and no dirty line of "
              "the flush is written back inside the timed region)")


class L2Flush:
    """Evicts L2 (126 MB) between timed steps.  Writing a 256 MB buffer alone
    leaves L2 full of dirty lines whose write-back would then be charged to
    the next timed kernel, so a read of a second 256 MB buffer follows: L2
    ends up holding clean lines of a buffer the step never touches."""

    LAUNCHES = 2

    def __init__(self, F):
        from wxx_b200.Tensor import Tensor

        self.F = F
        self.dirty = Tensor._empty([64 * 2 ** 20], "f32")
        self.clean = Tensor._empty([65536, 1024], "f32")
        F.assign(self.clean, 0.0)

    def __call__(self):
        self.F.assign(self.dirty, 0.0)
        self.F.sum(self.clean, 1)


class Workload:
    name = ""
    metric = ""
    unit = ""
    flush_l2 = False    # True when a step's weights + activations would stay in L2
    output_ids = True   # the step's output is the argmax token id of every position

    def units_per_rank(self, world):
        raise NotImplementedError


class GPT2Scaled(Workload):
    name = "gpt2_scaled"
    metric = "GPT2 fwd tokens/s"
    unit = "tokens/s"
    V, D, H, L, S, B_PER_GPU = 50304, 1024, 16, 24, 1024, 8

    def config(self, world):
        return {"workload": "GPT2(vocab=50304,d=1024,heads=16,layers=24) fwd, seq 1024, "
                            "8 seq/GPU",
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
    flush_l2 = True

    def config(self, world):
        return {"workload": "GPT2(vocab=1024,d=256,heads=8,layers=6) fwd, batch 4, seq 256",
                "global_batch": self.B_PER_GPU * world, "seq_len": self.S,
                "parallelism": f"dp{world}", "matmul_mode": "tf32",
                "l2": L2_FLUSHED}


class ResNet18W(Workload):
    name = "resnet18"
    metric = "ResNet18 inference img/s"
    unit = "img/s"
    B_PER_GPU = 256
    flush_l2 = True
    output_ids = False  # the output is the (batch, 10) logits

    def config(self, world):
        return {"workload": "ResNet18(10) eval, 3x32x32", "global_batch": self.B_PER_GPU * world,
                "seq_len": None, "parallelism": f"dp{world}", "matmul_mode": "tf32",
                "l2": L2_FLUSHED}

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


# ------------------------------------------------------------------ kernel sweep (config 1)

class Sweep:
    """One functional op of BASELINE config 1 on seeded N(0,1) inputs.

    ``units`` is the algorithmic work of one call: FLOPs for the tensor-bound
    matmuls, bytes that must cross HBM for the rest (inputs read once, outputs
    written once)."""

    def __init__(self, name, shapes, op, units, unit, bound, kernel, flush_l2):
        self.name, self.shapes, self.op = name, shapes, op
        self.units, self.unit, self.bound, self.kernel = units, unit, bound, kernel
        self.flush_l2 = flush_l2
        self.metric = f"{name} {unit}"


def _mm(F, a, b):
    return F.matmul_add(a, b, None)


SWEEPS = {}
for _n in (512, 2048, 8192):
    SWEEPS[f"matmul_{_n}"] = Sweep(
        f"matmul_{_n}", [(_n, _n), (_n, _n)], _mm, 2.0 * _n ** 3, "TFLOP/s", "tensor",
        "tc_gemm_kernel (tcgen05 kind::tf32)", flush_l2=_n < 4096)
SWEEPS["bmm"] = Sweep("bmm", [(64, 8, 1024, 32), (64, 8, 32, 1024)], _mm,
                      (64 + 64 + 2048) * 2 ** 20, "GB/s", "hbm",
                      "tc_gemm_kernel (batched, TMA-store epilogue)", flush_l2=False)
SWEEPS["softmax"] = Sweep("softmax", [(64, 8, 1024, 1024)], lambda F, x: F.softmax(x, -1),
                          4 * 2 ** 30, "GB/s", "hbm", "softmax_warp_kernel<32>", flush_l2=False)
SWEEPS["fftconv"] = Sweep("fftconv", [(16, 256, 16384), (256, 16384)],
                          lambda F, x, h: F.fftconv(x, h, 32768, out_len=16384),
                          528 * 2 ** 20, "GB/s", "hbm",
                          "fft_pair_kernel<14, conv> (+ rfft of h)", flush_l2=False)
# Hyena's fft_conv1d at the hyena workload's shape (B 16, D 256, L 8192,
# n 16384): x and y once each (128 MiB each), h once (8 MiB), its spectrum
# written and read (2 x 16 MiB).
SWEEPS["fftconv_hyena"] = Sweep("fftconv_hyena", [(16, 256, 8192), (256, 8192)],
                                lambda F, x, h: F.fftconv(x, h, 16384, out_len=8192),
                                296 * 2 ** 20, "GB/s", "hbm",
                                "fft_conv_staged_kernel<13> (+ rfft of h)", flush_l2=False)
# GPT2-scaled attention core (B 8, S 1024, 16 heads x 64, causal): useful
# FLOPs are the two products over the S(S+1)/2 unmasked (query, key) pairs.
SWEEPS["attention"] = Sweep("attention", [(8, 1024, 1024)] * 3,
                            lambda F, q, k, v: F.attention(q, k, v, 16, causal=True),
                            4.0 * 64 * 8 * 16 * (1024 * 1025 // 2), "TFLOP/s", "tensor",
                            "attention_kernel<64> (tcgen05 kind::tf32, TMEM S/O)", flush_l2=True)
def _gpt2_scaled_gemms(F, x1, x4, wqkv, wo, w1, w2, emb):
    """The GEMM launches of one GPT2-scaled layer plus the LM head, at the
    default workload's per-GPU shapes (8 x 1024 tokens, d 1024): fused QKV
    (K-major stacked weight), out projection + residual, FC1 + GELU, FC2 +
    residual, tied LM head (N = 50304)."""
    F.linear(x1, wqkv, transpose_weight=True)
    F.linear(x1, wo, residual=x1)
    F.linear(x1, w1, activation="gelu")
    F.linear(x4, w2, residual=x1)
    return F.matmul_add(x1, emb, None, transpose_B=True)


_T, _D, _V = 8192, 1024, 50304
SWEEPS["gemm_gpt2_scaled"] = Sweep(
    "gemm_gpt2_scaled", [(_T, _D), (_T, 4 * _D), (3 * _D, _D), (_D, _D), (_D, 4 * _D),
                         (4 * _D, _D), (_V, _D)], _gpt2_scaled_gemms,
    2.0 * _T * _D * (3 * _D + _D + 4 * _D + 4 * _D + _V), "TFLOP/s", "tensor",
    "tc_gemm_pair_kernel<256> (tcgen05 kind::tf32, cta_group::2)", flush_l2=False)
for _ax in (0, 1):
    SWEEPS[f"sum_axis{_ax}"] = Sweep(
        f"sum_axis{_ax}", [(4096, 4096)], (lambda ax: lambda F, x: F.sum(x, ax))(_ax),
        64 * 2 ** 20 + 16 * 2 ** 10, "GB/s", "hbm",
        "col_reduce_cluster_kernel" if _ax == 0 else "row_reduce_kernel", flush_l2=True)
    SWEEPS[f"mean_axis{_ax}"] = Sweep(
        f"mean_axis{_ax}", [(4096, 4096)], (lambda ax: lambda F, x: F.mean(x, ax))(_ax),
        64 * 2 ** 20 + 16 * 2 ** 10, "GB/s", "hbm",
        "col_reduce_cluster_kernel" if _ax == 0 else "row_reduce_kernel", flush_l2=True)


# ------------------------------------------------------------------ helpers

def load_traffic(name):
    """Measured DRAM bytes per launch of a workload's dominant kernel, from the
    ncu capture summarised in profiles/ (None when no capture covers it)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            rec = json.load(f).get(name)
    except (OSError, ValueError):
        return None
    if not rec:
        return None
    return {"bytes_per_launch": rec["traffic_bytes_per_launch"],
            "algorithmic_bytes_per_launch": rec["algorithmic_bytes_per_launch"],
            "kernel": rec["kernel"], "source": rec["source"],
            "metric": "dram__bytes_read.sum + dram__bytes_write.sum (one ncu capture)"}


def _traffic_keys(name):
    """roofline keys: ``traffic`` (DRAM bytes per launch, or None) and its
    provenance."""
    t = load_traffic(name)
    if t is None:
        return {"traffic": None}
    return {"traffic": t["bytes_per_launch"], "traffic_unit": "bytes per launch",
            "traffic_detail": t}


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
            # nvidia-smi takes a moment to start: a timed region of a few
            # hundred ms would otherwise end before its first sample
            t_end = time.time() + 3.0
            while time.time() < t_end and self.proc.poll() is None:
                if os.path.getsize(self.path) > 0:
                    break
                time.sleep(0.02)
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


# ------------------------------------------------------------------ sweep runs

def _sweep_cpu(sw, arrays):
    """fp32 numpy version of a sweep op (CPU baseline / reference arm)."""
    import oracle.kernels as K

    if sw.name.startswith("matmul") or sw.name == "bmm":
        return lambda: np.matmul(arrays[0], arrays[1])
    if sw.name == "softmax":
        def f():
            e = np.exp(arrays[0] - arrays[0].max(-1, keepdims=True))
            return e / e.sum(-1, keepdims=True)
        return f
    if sw.name == "fftconv":
        return lambda: np.fft.irfft(np.fft.rfft(arrays[0], 32768) * np.fft.rfft(arrays[1], 32768),
                                    32768)[..., :16384]
    if sw.name == "fftconv_hyena":
        return lambda: np.fft.irfft(np.fft.rfft(arrays[0], 16384) * np.fft.rfft(arrays[1], 16384),
                                    16384)[..., :8192]
    if sw.name == "gemm_gpt2_scaled":
        def gemms():
            x1, x4, wqkv, wo, w1, w2, emb = arrays
            np.matmul(x1, wqkv.T)
            np.matmul(x1, wo) + x1
            np.matmul(x1, w1)
            np.matmul(x4, w2) + x1
            return np.matmul(x1, emb.T)
        return gemms
    if sw.name == "attention":
        def attn():
            B, S, D = arrays[0].shape
            q, k, v = (a.reshape(B, S, 16, D // 16).transpose(0, 2, 1, 3) for a in arrays)
            sc = np.matmul(q, k.transpose(0, 1, 3, 2)) * np.float32(1 / np.sqrt(D // 16))
            sc = sc + np.triu(np.full((S, S), -1e9, np.float32), 1)
            e = np.exp(sc - sc.max(-1, keepdims=True))
            return np.matmul(e / e.sum(-1, keepdims=True), v)
        return attn
    ax = int(sw.name[-1])
    if sw.name.startswith("sum"):
        return lambda: arrays[0].sum(axis=ax)
    _ = K
    return lambda: arrays[0].mean(axis=ax)


def _sweep_cpu_sample(sw, rng):
    """A bounded slice of the sweep input for CPU timing, and its fraction."""
    if sw.name == "softmax":
        return [rng.standard_normal((4, 8, 1024, 1024), dtype=np.float32)], 4 / 64
    if sw.name == "bmm":
        return [rng.standard_normal((4, 8, 1024, 32), dtype=np.float32),
                rng.standard_normal((4, 8, 32, 1024), dtype=np.float32)], 4 / 64
    if sw.name == "fftconv":
        return [rng.standard_normal((1, 256, 16384), dtype=np.float32),
                rng.standard_normal((256, 16384), dtype=np.float32)], 1 / 16
    if sw.name == "attention":
        return [rng.standard_normal((1, 1024, 1024), dtype=np.float32) for _ in range(3)], 1 / 8
    if sw.name == "fftconv_hyena":
        return [rng.standard_normal((1, 256, 8192), dtype=np.float32),
                rng.standard_normal((256, 8192), dtype=np.float32)], 1 / 16
    if sw.name == "gemm_gpt2_scaled":
        shapes = [(256,) + sw.shapes[0][1:], (256,) + sw.shapes[1][1:]] + list(sw.shapes[2:])
        return [rng.standard_normal(s, dtype=np.float32) for s in shapes], 256 / sw.shapes[0][0]
    if sw.name == "matmul_8192":
        return [rng.standard_normal((1024, 8192), dtype=np.float32),
                rng.standard_normal((8192, 8192), dtype=np.float32)], 1 / 8
    return [rng.standard_normal(s, dtype=np.float32) for s in sw.shapes], 1.0


def run_sweep(args, rank, world, local):
    """Times one config-1 kernel; N > 1 runs independent replicas (weak scaling)."""
    os.environ.setdefault("WXX_DEVICE", str(local))
    import wxx_b200 as wxx
    from wxx_b200.backend import device as dev
    from wxx_b200 import distributed as wd

    sw = SWEEPS[args.workload]
    dist = wd.init_host_group() if world > 1 else None
    F = wxx.functional
    wxx.set_matmul_mode("tf32")
    rng = np.random.default_rng(rank)
    host = [rng.standard_normal(s, dtype=np.float32) for s in sw.shapes]
    devs = [F.from_numpy(a) for a in host]
    flush = L2Flush(F) if sw.flush_l2 else None

    def timed(n, fn):
        total = 0.0
        if flush is None:
            e0 = dev.Event().record()
            for _ in range(n):
                fn()
            e1 = dev.Event().record()
            return e0.elapsed_ms(e1) / n
        for _ in range(n):
            flush()
            e0 = dev.Event().record()
            fn()
            e1 = dev.Event().record()
            total += e0.elapsed_ms(e1)
        return total / n

    for _ in range(args.warmup):
        sw.op(F, *devs)
    dev.synchronize()
    # The op is recorded once as a CUDA graph and each timed step is one
    # replay: the host's Python and argument checks for a call of ~0.1 ms
    # would otherwise show up as idle device time inside the events
    # (``--eager`` times the direct calls).
    graph = None
    if not args.eager:
        graph = wxx.graph.capture(lambda: sw.op(F, *devs))
        for _ in range(2):
            graph.replay()
        dev.synchronize()
    if dist is not None:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    n0 = dev.launch_count()
    ms = timed(args.steps, graph.replay if graph is not None else (lambda: sw.op(F, *devs)))
    if graph is not None:
        launches = graph.stats()["kernels"] * args.steps
    else:
        launches = dev.launch_count() - n0 - (args.steps * L2Flush.LAUNCHES if flush is not None else 0)
    clocks = sampler.stop()
    if graph is not None:
        dev.synchronize()
        graph.close()
    if dist is not None:
        import torch

        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    scale = 1e12 if sw.unit == "TFLOP/s" else 1e9
    value = world * sw.units / (ms / 1000.0) / scale

    # e2e through the public API from pinned host memory, result read back.
    pins = []
    for a in host:
        pb = dev.PinnedHostBuffer(a.nbytes)
        pb.as_numpy(np.float32, a.shape)[...] = a
        pins.append(pb)
    from wxx_b200.Tensor import Tensor

    res_box = {}

    def e2e():
        ts = []
        for a, pb in zip(host, pins):
            t = Tensor._empty(list(a.shape), "f32")
            wxx.backend.lib.F.wxx_memcpy_h2d(t.buffer.ptr, pb.ptr, a.nbytes)
            ts.append(t)
        out = sw.op(F, *ts)
        if "pin" not in res_box:
            res_box["pin"] = dev.PinnedHostBuffer(out.nbytes)
        wxx.backend.lib.F.wxx_memcpy_d2h_async(res_box["pin"].ptr, out.ptr, out.nbytes)
        res_box["bytes"] = out.nbytes

    for _ in range(2):
        e2e()
    dev.synchronize()
    e2e_ms = timed(max(3, args.steps // 2), e2e)
    e2e_value = world * sw.units / (e2e_ms / 1000.0) / scale
    peaks, kind = load_peaks()
    if sw.bound == "tensor":
        peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]) / 2.0
        basis = f"{kind} bf16 dense TFLOP/s / 2 (TF32 rate)"
        achieved = sw.units / (ms / 1000.0) / 1e12
    else:
        peak = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
        basis = f"{kind} HBM copy GB/s"
        achieved = sw.units / (ms / 1000.0) / 1e9
    line = {
        "metric": sw.metric, "value": value, "unit": sw.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{sw.name} {sw.shapes}", "l2": L2_FLUSHED
                   if sw.flush_l2 else "inputs larger than L2", "parallelism": "replicas",
                   "launch": "eager" if args.eager else "CUDA graph of the op, one replay per step"},
        "roofline": {"kernel": sw.kernel, "bound": sw.bound, "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s" if sw.bound == "tensor" else "GB/s",
                     "frac": achieved / peak, "peak_basis": basis,
                     **_traffic_keys(sw.name)},
        "clocks": clocks, "gpu_launches": int(launches),
        "e2e": {"value": e2e_value, "unit": sw.unit,
                "h2d_bytes_per_step": int(sum(a.nbytes for a in host)),
                "d2h_bytes_per_step": int(res_box.get("bytes", 0))},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        arrays, frac = _sweep_cpu_sample(sw, np.random.default_rng(0))
        fn = _sweep_cpu(sw, arrays)
        fn()
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < args.cpu_seconds and reps < 200:
            fn()
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        line["cpu_baseline"] = {"value": sw.units * frac / dt / scale, "unit": sw.unit,
                                "cores": cpu_cores(), "kind": "port",
                                "sample": f"{frac:.3g} of the workload per call, {reps} calls "
                                          "(numpy fp32, host BLAS threads)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def line_config(wl, world, args):
    """The ``config`` both arms print for a model workload (the reference arm
    times a bounded sample of the same workload and says so in
    ``cpu_baseline.sample``, not here)."""
    rows = wl.rows(world)
    gather = None
    if world > 1:
        out_ids = wl.output_ids and args.gather == "ids"
        per_row = 10 if not wl.output_ids else (wl.units_per_row() * (1 if out_ids else wl.V))
        slot = max(1, -(-rows // world))
        gather = {"what": "argmax ids" if out_ids else "fp32 logits",
                  "bytes_sent_per_rank": slot * per_row * 4,
                  "bytes_received_per_rank": (world - 1) * slot * per_row * 4,
                  "mode": ("asynchronous on a second stream, overlapping the next step's forward"
                           if (wl.output_ids and args.gather == "logits")
                           else "on the library stream after the forward"),
                  "padded_slots": rows % world != 0 or rows < world}
    return dict(wl.config(world),
                launch="eager" if args.eager else "CUDA graph of the forward, one replay per step",
                gather=gather)


# ------------------------------------------------------------------ reference arm

def _reference_extra(args, world):
    """The oracle's restatement of the reference's training step / sampling
    loop on a bounded sample (one sequence), timed on the host."""
    from oracle import init as oracle_init, models as oracle_models, train as oracle_train

    rng = np.random.default_rng(7)
    if args.workload == "gpt2_small_train":
        V, D, H, L, S = 1024, 256, 8, 6, 256
        sd = oracle_init.gpt2_state_dict(7, V, D, H, L, S)
        ids = rng.integers(0, V, size=(1, S))
        tgt = np.roll(ids, -1, axis=1)

        def fn():
            oracle_train.gpt2_loss_and_grads(sd, ids, tgt, H, L)

        units, what = S, "1 x 256 tokens per step (float64 numpy forward + backward)"
    else:
        V, D, H, L, S = 50304, 1024, 16, 24, 1024
        sd = oracle_init.gpt2_state_dict(7, V, D, H, L, S)
        prompt = rng.integers(0, V, size=(1, 128))

        def fn():
            oracle_models.gpt2_generate(sd, prompt, H, L, 2, temperature=0.0)

        units, what = 2, "1 prompt of 128 tokens, 2 new tokens per step (full forward per token)"
    for _ in range(max(1, min(args.warmup, 1))):
        fn()
    t0 = time.perf_counter()
    n = max(1, min(args.steps, 3))
    for _ in range(n):
        fn()
    dt = (time.perf_counter() - t0) / n
    value = units / dt
    info = EXTRA[args.workload]
    print(json.dumps({
        "metric": info["metric"], "value": value, "unit": info["unit"], "n_gpus": world,
        "steps": n, "warmup": args.warmup, "ms_per_step": dt * 1000, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64 (numpy)", "data": "synthetic",
        "config": {"workload": args.workload}, "impl": "reference",
        "cpu_baseline": {"value": value, "unit": info["unit"], "cores": cpu_cores(),
                         "kind": "port", "sample": what},
        "e2e": {"value": value, "unit": info["unit"], "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)
    return 0


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    if args.workload in EXTRA:
        return _reference_extra(args, world)
    if args.workload in SWEEPS:
        sw = SWEEPS[args.workload]
        arrays, frac = _sweep_cpu_sample(sw, np.random.default_rng(0))
        fn = _sweep_cpu(sw, arrays)
        for _ in range(args.warmup):
            fn()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            fn()
        dt = (time.perf_counter() - t0) / args.steps
        scale = 1e12 if sw.unit == "TFLOP/s" else 1e9
        value = sw.units * frac / dt / scale
        print(json.dumps({
            "metric": sw.metric, "value": value, "unit": sw.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1000,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": f"{sw.name} {sw.shapes}"},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": sw.unit, "cores": cpu_cores(), "kind": "port",
                             "sample": f"{frac:.3g} of the workload per step (numpy fp32)"},
            "e2e": {"value": value, "unit": sw.unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
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
        "data": "synthetic", "config": line_config(wl, world, args), "impl": "reference",
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

    idle = hi == lo          # more ranks than batch rows: this rank only joins the gather
    x_dev = None if idle else upload(x_host)
    comm = wd.NcclCommunicator(rank, world, dist) if world > 1 else None
    # What a step outputs (and, for N > 1, all-gathers): the argmax token id
    # of every position (--gather ids, default for the language models), the
    # fp32 logits (--gather logits), or ResNet's logits.
    out_ids = wl.output_ids and args.gather == "ids"
    if not wl.output_ids:
        row_shape, out_dtype = [10], "f32"
    elif out_ids:
        row_shape, out_dtype = [wl.units_per_row()], "u32"
    else:
        row_shape, out_dtype = [wl.units_per_row(), wl.V], "f32"

    def forward(inp):
        with wxx.backend.inferenceMode():
            if out_ids and hasattr(model, "forward_argmax"):
                # the ids straight from the LM head's GEMM (logits not stored)
                return model.forward_argmax(inp)
            out = model(inp)
        return F.max(out, -1)[1] if out_ids else out

    # One CUDA graph per step: the forward is recorded once (after an eager
    # warm-up inside capture()) and replayed with one launch; the step reads
    # its input from x_dev.  With an asynchronous logits gather (N > 1,
    # --gather logits) two graphs with separate output buffers alternate, so
    # step k+1's forward runs while step k's logits cross NVLink.
    pipelined = comm is not None and args.gather == "logits" and wl.output_ids
    graphs = []
    if not args.eager and not idle:
        graphs = [wxx.graph.capture(forward, x_dev) for _ in range(2 if pipelined else 1)]
    pending = [None, None]
    counter = [0]

    def run_forward():
        if idle:
            return None
        if graphs:
            return graphs[counter[0] % len(graphs)].replay()
        return forward(x_dev)

    def step():
        """forward + gather; returns the step's (gathered) output or a
        PendingGather (pipelined logits)."""
        k = counter[0]
        if pipelined:
            g = k % 2
            if pending[g] is not None:
                pending[g].wait()       # graph g's output buffer is free again
                pending[g] = None
            out = run_forward()
            pending[g] = comm.allgather_rows(out, rows_global, row_shape, out_dtype, slot=g)
            counter[0] += 1
            return pending[g]
        out = run_forward()
        counter[0] += 1
        if comm is not None:
            out = comm.allgather_rows(out, rows_global, row_shape, out_dtype)
        return out

    def drain():
        for g in (0, 1):
            if pending[g] is not None:
                pending[g].wait()
                pending[g] = None

    def barrier():
        drain()
        dev.synchronize()
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    barrier()
    gpu_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[0]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")[0].isdigit() else local
    from wxx_b200.Tensor import Tensor

    flush_buf = L2Flush(F) if wl.flush_l2 else None
    sampler = ClockSampler(gpu_index)
    sampler.start()
    n0 = dev.launch_count()

    def timed_steps(fn, n):
        """(device ms per step, host enqueue ms per step, launches per step).
        With flush_l2 the L2 flush runs before every step, outside its events.
        Pipelined gathers still in flight are waited for inside the last
        step's events."""
        nl0 = dev.launch_count()
        host = 0.0
        if flush_buf is None:
            a, b = dev.Event(), dev.Event()
            a.record()
            h = time.perf_counter()
            for _ in range(n):
                fn()
            drain()
            host = time.perf_counter() - h
            b.record()
            barrier()
            total = a.elapsed_ms(b)
        else:
            evs = []
            for _ in range(n):
                flush_buf()
                a, b = dev.Event(), dev.Event()
                a.record()
                h = time.perf_counter()
                fn()
                drain()
                host += time.perf_counter() - h
                b.record()
                evs.append((a, b))
            barrier()
            total = sum(a.elapsed_ms(b) for a, b in evs)
        nl = dev.launch_count() - nl0 - (n * L2Flush.LAUNCHES if flush_buf is not None else 0)
        return total / n, host * 1000.0 / n, nl / n

    def max_over_ranks(v):
        if dist is None:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # the forward alone (no collective), then the full step (forward + gather)
    fwd_ms = max_over_ranks(timed_steps(run_forward, args.steps)[0]) if comm is not None \
        else None
    ms, host_ms, launches = timed_steps(step, args.steps)
    log_path = os.environ.get("WXX_LAUNCH_LOG")
    if log_path and rank == 0:
        with open(log_path, "w") as f:
            json.dump({"before_timed": n0, "per_step": launches}, f)
    clocks = sampler.stop()
    ms = max_over_ranks(ms)
    units_total = rows_global * wl.units_per_row()
    value = units_total / (ms / 1000.0)

    # e2e: pinned host inputs -> device -> step (forward, output ids/logits,
    # all-gather) -> host.  The gathered ids (or ResNet logits) are read back
    # whole; with --gather logits each rank reads back its own rows of the
    # gathered logits.
    pin_in = dev.PinnedHostBuffer(max(4, x_host.nbytes))
    if x_host.nbytes:
        pin_in.as_numpy(x_host.dtype, x_host.shape)[...] = x_host
    out_elems = rows_global * int(np.prod(row_shape))
    own_elems = (hi - lo) * int(np.prod(row_shape))
    d2h_elems = out_elems if (out_ids or not wl.output_ids) else own_elems
    pin_out = dev.PinnedHostBuffer(max(4, d2h_elems * 4))

    def e2e_step():
        if not idle:
            # the graphs read their input from x_dev
            wxx.backend.lib.F.wxx_memcpy_h2d(x_dev.buffer.ptr, pin_in.ptr, x_host.nbytes)
        out = step()
        if hasattr(out, "wait"):
            out = out.wait()
        if d2h_elems == 0:
            return 0
        src = out.ptr + (lo * int(np.prod(row_shape)) * 4 if d2h_elems != out_elems else 0)
        wxx.backend.lib.F.wxx_memcpy_d2h_async(pin_out.ptr, src, d2h_elems * 4)
        return d2h_elems * 4

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    d2h = e2e_step()
    barrier()
    e2e_ms = max_over_ranks(timed_steps(e2e_step, args.steps)[0])
    e2e_value = units_total / (e2e_ms / 1000.0)

    # roofline of the dominant kernel (the tcgen05 GEMM): every GEMM launch of
    # one forward bracketed by CUDA events on the library stream.  With graphs
    # the bracketed forward is itself captured (the events become graph event
    # nodes) and replayed, so host launch gaps stay out of the kernel times.
    if idle:
        ks = {"flops": 0.0, "ms": 0.0, "launches": 0}
    elif graphs:
        with KernelTimer() as kt:
            timed_graph = wxx.graph.CapturedGraph(
                forward, (x_dev,), {}, arena_bytes=graphs[0].stats()["arena_bytes"],
                warmup=False)
        runs = []
        for _ in range(3):
            if flush_buf is not None:
                flush_buf()
            timed_graph.replay()
            dev.synchronize()
            runs.append(kt.summary())
        timed_graph.close()
        ks = dict(runs[-1], ms=sum(r["ms"] for r in runs) / len(runs))
    else:
        with KernelTimer() as kt:
            forward(x_dev)
        dev.synchronize()
        ks = kt.summary()
    peaks, peak_kind = load_peaks()
    # The GEMMs run inside a step of many milliseconds at the power cap: the
    # sustained figure is the denominator (the burst one for kernels timed
    # alone, the sweeps).
    sustained = "bf16_tflops_sustained" in peaks
    tf32_peak = peaks.get("bf16_tflops_sustained",
                          peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])) / 2.0
    achieved = ks["flops"] / (ks["ms"] / 1000.0) / 1e12 if ks["ms"] > 0 else 0.0
    roofline = {
        "kernel": "tcgen05 kind::tf32 GEMM / implicit-GEMM conv (TMA-fed, TMEM accumulators)",
        "bound": "tensor", "achieved": achieved, "peak": tf32_peak, "unit": "TFLOP/s",
        "frac": achieved / tf32_peak, **_traffic_keys(wl.name),
        "peak_basis": f"{peak_kind} {'sustained ' if sustained else ''}bf16 dense TFLOP/s / 2 "
                      "(B200 TF32 rate is half of BF16; kernel timed inside a long step)",
        "gemm_share_of_step": ks["ms"] / ms if ms > 0 else None,
        "gemm_launches_per_step": ks["launches"],
    }

    # The same step with every product in 3xTF32 (the fp32-faithful mode the
    # parity tests hold to 1e-5 of the oracle), N = 1: what exactness costs.
    faithful = None
    if world == 1 and not idle and not args.no_faithful:
        wxx.set_matmul_mode("3xtf32")
        g3 = None
        try:
            if graphs:
                g3 = wxx.graph.capture(forward, x_dev)
                fn3 = g3.replay
            else:
                def fn3():
                    return forward(x_dev)
            for _ in range(2):
                fn3()
            barrier()
            n3 = max(3, min(args.steps, 10))
            ms3 = timed_steps(fn3, n3)[0]
            faithful = {"matmul_mode": "3xtf32", "value": units_total / (ms3 / 1000.0),
                        "unit": wl.unit, "ms_per_step": ms3, "steps": n3,
                        "l2": L2_FLUSHED if flush_buf is not None else "inputs > L2"}
        finally:
            if g3 is not None:
                g3.close()
            wxx.set_matmul_mode("tf32")

    line = {
        "metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak" if wl.rows(2) == 2 * wl.rows(1) else "strong", "vs_baseline": None,
        "dtype": "f32 (tf32 tensor-core products)", "data": "synthetic",
        "config": line_config(wl, world, args),
        "roofline": roofline, "clocks": clocks,
        "gpu_launches": int(round(launches * args.steps)),
        "host_enqueue_ms_per_step": host_ms,
        "e2e": {"value": e2e_value, "unit": wl.unit,
                "h2d_bytes_per_step": int(x_host.nbytes), "d2h_bytes_per_step": int(d2h),
                "includes": "pinned H2D of inputs, forward, output (argmax ids or logits), "
                            "all-gather, D2H of the gathered outputs (own rows for logits)"},
    }
    if faithful is not None:
        line["faithful_3xtf32"] = faithful
    if comm is not None:
        # the forward alone and the step with its gather
        line["forward_ms_per_step"] = fwd_ms
        line["forward_value"] = units_total / (fwd_ms / 1000.0)
        line["gather_ms_per_step"] = ms - fwd_ms
        line["idle_ranks"] = sum(1 for r in range(world)
                                 if wd.shard_bounds(rows_global, world, r)[0]
                                 == wd.shard_bounds(rows_global, world, r)[1])
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


# ------------------------------------------------------------------ training and generation

EXTRA = {
    # GPT2 config 0 trained: forward in training mode, CCELoss over the next
    # token, backward, AdamW step.  FLOPs ~ 3x the forward's products.
    "gpt2_small_train": {"metric": "GPT2 train tokens/s", "unit": "tokens/s"},
    # GPT2-scaled generation: 8 prompts of 128 tokens, 128 new tokens each,
    # greedy, K/V cache, one CUDA-graph replay per decode step.
    "gpt2_scaled_generate": {"metric": "GPT2 generate tokens/s", "unit": "tokens/s"},
}


def run_extra(args, rank, world, local):
    """Training step / generation throughput on one GPU (N > 1: replicas)."""
    os.environ.setdefault("WXX_DEVICE", str(local))
    import wxx_b200 as wxx
    from wxx_b200.backend import device as dev
    from wxx_b200 import distributed as wd

    dist = wd.init_host_group() if world > 1 else None
    F = wxx.functional
    wxx.manual_seed(1234)
    wxx.set_matmul_mode("tf32")
    rng = np.random.default_rng(rank)
    peaks, kind = load_peaks()
    if args.workload == "gpt2_small_train":
        V, D, H, L, S, B = 1024, 256, 8, 6, 256, 4
        model = wxx.nn.GPT2(V, D, H, L, max_len=S, dropout=0.0)
        opt = wxx.nn.AdamW(model.parameters(), lr=1e-4)
        ids_h = rng.integers(0, V, size=(B, S), dtype=np.uint32)
        tgt_h = np.roll(ids_h, -1, axis=1).reshape(-1)
        loss_fn = wxx.nn.CCELoss()
        ids_dev = F.from_numpy(ids_h, dtype=np.uint32)
        tgt_dev = F.from_numpy(tgt_h, dtype=np.uint32)

        def train_step():
            opt.zero_grad()
            logits = model(ids_dev)
            loss = loss_fn(logits.reshape((B * S, V)), tgt_dev)
            loss.backward()
            opt.step()
            return loss

        # the whole step (forward, loss, backward, AdamW with its device step
        # count) recorded once and replayed: one launch per step
        graph = wxx.graph.capture(train_step)
        lib = wxx.backend.lib.F

        def step():
            # host batch in, loss value out: the call a training loop makes
            lib.wxx_memcpy_h2d(ids_dev.ptr, ids_h.ctypes.data, ids_h.nbytes)
            lib.wxx_memcpy_h2d(tgt_dev.ptr, tgt_h.ctypes.data, tgt_h.nbytes)
            return float(graph.replay().numpy().reshape(-1)[0])

        units, flops = B * S, 3 * 11.81e9
        flush = L2Flush(F)
    else:
        V, D, H, L, S = 50304, 1024, 16, 24, 1024
        B, P, N = 8, 128, 128
        model = wxx.nn.GPT2(V, D, H, L, max_len=S)
        prompt = rng.integers(0, V, size=(B, P), dtype=np.uint32)

        def step():
            return model.generate(prompt, max_new_tokens=N, temperature=0.0)

        units, flops = B * N, None
        flush = None

    for _ in range(args.warmup):
        step()
    dev.synchronize()
    if dist is not None:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    n0 = dev.launch_count()
    total = 0.0
    for _ in range(args.steps):
        if flush is not None:
            flush()
        a, b = dev.Event(), dev.Event()
        a.record()
        out = step()
        b.record()
        dev.synchronize()
        total += a.elapsed_ms(b)
        del out
    launches = dev.launch_count() - n0 - (args.steps * L2Flush.LAUNCHES if flush else 0)
    clocks = sampler.stop()
    ms = total / args.steps
    if dist is not None:
        import torch

        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * units / (ms / 1000.0)
    info = EXTRA[args.workload]
    if flops is not None:
        peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]) / 2.0
        ach = flops / (ms / 1000.0) / 1e12
        roof = {"kernel": "whole step (forward + backward products, AdamW)", "bound": "tensor",
                "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                "traffic": None, "peak_basis": f"{kind} bf16 dense TFLOP/s / 2"}
        e2e_h2d = ids_h.nbytes + tgt_h.nbytes
        cfg = {"workload": "GPT2(1024,256,8,6) train step: fwd + CCELoss + bwd + AdamW, "
                           "batch 4, seq 256, replayed from one CUDA graph",
               "parallelism": "replicas", "l2": L2_FLUSHED}
    else:
        # A decode step reads every weight once (q/k/v, out, fc1, fc2 per
        # layer and the tied head) and each layer's K / V cache up to the
        # current length (on average P + N / 2 positions).  Its time: the call
        # minus a prefill-only call (one new token), over the N - 1 steps.
        weight_bytes = 4 * (L * 12 * D * D + V * D)
        cache_bytes = 4 * L * 2 * B * (P + N // 2) * D
        pre = []
        for _ in range(3):
            a, b = dev.Event(), dev.Event()
            a.record()
            model.generate(prompt, max_new_tokens=1, temperature=0.0)
            b.record()
            dev.synchronize()
            pre.append(a.elapsed_ms(b))
        prefill_ms = sorted(pre)[1]
        step_ms = max(ms - prefill_ms, 1e-6) / (N - 1)
        ach = (weight_bytes + cache_bytes) / (step_ms / 1000.0) / 1e9
        peak = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
        roof = {"kernel": "decode step (weights and K/V cache streamed once per token step)",
                "bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                "traffic": None, "peak_basis": f"{kind} HBM copy GB/s",
                "bytes_per_decode_step": weight_bytes + cache_bytes,
                "decode_ms_per_token_step": step_ms, "prefill_ms": prefill_ms}
        e2e_h2d = prompt.nbytes
        cfg = {"workload": "GPT2(50304,1024,16,24) generate: 8 prompts x 128 tokens, 128 new "
                           "tokens each, greedy, K/V cache", "parallelism": "replicas"}
    line = {
        "metric": info["metric"], "value": value, "unit": info["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (tf32 tensor-core products)",
        "data": "synthetic", "config": cfg, "roofline": roof, "clocks": clocks,
        "gpu_launches": int(launches),
        "e2e": {"value": value, "unit": info["unit"], "h2d_bytes_per_step": int(e2e_h2d),
                "d2h_bytes_per_step": 4 if flops is not None else B * (P + N) * 4,
                "includes": "the public API call per step (host inputs, result read back)"},
    }
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
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(SWEEPS) + sorted(EXTRA),
                    default="gpt2_scaled")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-faithful", action="store_true",
                    help="skip the extra 3xTF32 timing of the model workloads")
    ap.add_argument("--gather", choices=["ids", "logits", "logits-serial"], default="ids",
                    help="language models, N > 1: all-gather the argmax token ids (default) "
                         "or the fp32 logits (BASELINE config 5's collective; 'logits' overlaps "
                         "step k's gather with step k+1's forward, 'logits-serial' runs it "
                         "after the forward on the same stream)")
    ap.add_argument("--eager", action="store_true",
                    help="model workloads: launch every kernel from Python each step "
                         "instead of replaying the step's CUDA graph")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.workload in SWEEPS:
        return run_sweep(args, rank, world, local)
    if args.workload in EXTRA:
        return run_extra(args, rank, world, local)
    return run_ours(args, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
