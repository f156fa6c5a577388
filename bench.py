"""Benchmark of the B200 block-quantized matmul hot path.

Metric: 2MNK int-ops/s and weight GB/s against the HBM /
int8 tensor-core roofline.

Default workload (the decode configuration):
one step = the activation row x (fp32, K=4096, seeded N(0,1)) quantized to
q8_0 on the device and multiplied by two q4_0 weight matrices,
N=4096 x K=4096 and N=11008 x K=4096 (seeded N(0,1), quantized on the device
with the bit-exact q4_0 quantizer), through pfng_b200_compute_grouped -- the
quantization is fused into the HBM-streaming GEMV and both matrices, which
share the activation row, stream in one launch.
The steps rotate over enough weight copies that the weights of a step are
never in the 126 MB L2 (inputs larger than L2).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's own CPU implementation of the same
step (oracle/_ref: bench/llama_reference compiled from the reference's
sources; all host threads) on the same config and metric.

With --gpus N > 1 (launched by torchrun, one process per GPU) every rank runs
an independent replica of the workload (the decode GEMV is too small to
shard: the NCCL latency of gathering its output exceeds its runtime), timed
as the max over ranks; `value` is the whole-job aggregate.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "qgemm-perf-framework-ng_b200"))

METRIC = "2MNK int-ops/s and weight GB/s vs int8-TC/HBM roofline, 1/2/4/8 B200"
UNIT = "Gop/s"
K_DIM = 4096
N_DIMS = (4096, 11008)
Q4_0_ROW_BYTES = K_DIM // 32 * 18
L2_BYTES = 126 * 1024 * 1024


def step_ops() -> float:
    return float(sum(2 * 1 * n * K_DIM for n in N_DIMS))


def step_weight_bytes() -> int:
    return sum(n * Q4_0_ROW_BYTES for n in N_DIMS)


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(kernel_tag: str):
    """DRAM bytes per launch from a committed ncu summary, if one exists."""
    path = ROOT / "profiles" / f"{kernel_tag}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.file.flush()
        rows = []
        for line in pathlib.Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[1].isdigit():
                rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [int(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": int(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


# ------------------------------------------------------------------ CPU arms
def cpu_library():
    """(library, kind): the reference's own code if it was compiled, else the oracle port."""
    sys.path.insert(0, str(ROOT / "tests"))
    from oracle_lib import Oracle, reference_or_none
    ref = reference_or_none()
    if ref is not None:
        return ref, "reference"
    return Oracle(), "port"


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_step_inputs(seed: int = 1):
    import numpy as np
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((1, K_DIM)).astype(np.float32)
    ws = [rng.standard_normal((n, K_DIM)).astype(np.float32) for n in N_DIMS]
    return x, ws


def run_cpu_steps(lib, kind: str, weights, x, steps: int, threads: int) -> float:
    """Seconds for `steps` decode steps of the reference CPU path."""
    t0 = time.perf_counter()
    for _ in range(steps):
        a = lib.quantize("q8_0", x)
        for w, n in zip(weights, N_DIMS):
            if kind == "reference":
                lib.mm_threads("q4_0", w, a, 1, n, K_DIM, threads)
            else:
                lib.mm("q4_0", w, a, 1, n, K_DIM)
    return time.perf_counter() - t0


def cpu_baseline(budget_s: float = 10.0):
    lib, kind = cpu_library()
    threads = cpu_threads() if kind == "reference" else int(os.environ.get("OMP_NUM_THREADS", cpu_threads()))
    x, wf = cpu_step_inputs()
    weights = [lib.quantize("q4_0", w) for w in wf]
    run_cpu_steps(lib, kind, weights, x, 1, threads)
    one = run_cpu_steps(lib, kind, weights, x, 1, threads)
    steps = max(1, int(budget_s / max(one, 1e-6)))
    secs = run_cpu_steps(lib, kind, weights, x, steps, threads)
    value = steps * step_ops() / secs / 1e9
    return {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{steps} decode steps (q8_0 quantize + q4_0 1x4096x4096 + 1x11008x4096) in {secs:.2f} s"}


def reference_arm(args) -> int:
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    lib, kind = cpu_library()
    threads = cpu_threads()
    x, wf = cpu_step_inputs()
    weights = [lib.quantize("q4_0", w) for w in wf]
    run_cpu_steps(lib, kind, weights, x, args.warmup, threads)
    secs = run_cpu_steps(lib, kind, weights, x, args.steps, threads)
    value = args.steps * step_ops() / secs / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/int32 dot, fp32 fold",
        "data": "synthetic: seeded N(0,1) fp32 weights and activations, quantized by the reference quantizers",
        "config": dict(workload_config(), workload=workload_config()["workload"].replace(
            "activation quantized on device (fused)", "activation quantized on the host by the reference")),
        "weight_GBps": args.steps * step_weight_bytes() / secs / 1e9,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"{args.steps} timed steps of the full workload"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config():
    return {
        "workload": "configs[1]: q4_0 x q8_0 decode GEMV, M=1, (N,K) = (4096,4096) + (11008,4096), "
                    "activation quantized on device (fused)",
        "m": 1, "n": list(N_DIMS), "k": K_DIM, "weight_type": "q4_0", "activation_type": "q8_0",
        "l2": "inputs larger than L2: weights rotate over copies totalling > 4x the 126 MB L2",
    }


# ------------------------------------------------------------------ GPU arm
def ours(args) -> int:
    import torch
    import pfng_b200 as pb

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))

    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)  # graph capture needs a non-default stream
    copies = max(2, -(-4 * L2_BYTES // step_weight_bytes()))
    gen = torch.Generator(device="cuda").manual_seed(1 + rank)
    weights = []
    for _ in range(copies):
        per = []
        for n in N_DIMS:
            wf = torch.randn((n, K_DIM), generator=gen, device="cuda", dtype=torch.float32)
            per.append(pb.quantize_q4_0(wf))
            del wf
        weights.append(per)
    x = torch.randn((1, K_DIM), generator=torch.Generator(device="cuda").manual_seed(2), device="cuda")
    outs = [torch.empty((1, n), device="cuda") for n in N_DIMS]
    ws = torch.empty(max(1, pb.compute_workspace_size(pb.Q4_0, 1, max(N_DIMS), K_DIM)), dtype=torch.uint8,
                     device="cuda")
    torch.cuda.synchronize()

    # The weights are constant, so consecutive steps may overlap: each launch
    # starts streaming its weights while the previous one drains
    # (PFNG_B200_OVERLAP_WEIGHTS); activations and outputs stay ordered.
    calls = [pb.GroupedCall(pb.Q4_0, weights[r], N_DIMS, outs, x, overlap_weights=True) for r in range(copies)]

    def step(i: int, xin=None):
        calls[i % copies](x=xin, stream=stream)

    def barrier():
        if dist is not None:
            dist.barrier()

    # warm-up (also loads the kernels)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    # ---- device-resident timing: capture the K steps in one CUDA graph
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(args.steps):
            step(i)
    graph.replay()  # warm the graph once
    torch.cuda.synchronize()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        torch.cuda.synchronize()
        barrier()
        start.record(stream)
        graph.replay()
        end.record(stream)
        torch.cuda.synchronize()
        barrier()
    elapsed = start.elapsed_time(end) / 1e3
    clock_info = clocks.summary()
    elapsed_max = elapsed
    if dist is not None:
        t = torch.tensor([elapsed], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_max = float(t.item())
    pb.check_kernel_error()

    # ---- per-launch duration of the GEMV kernel: the timed region above is
    # exactly K back-to-back launches of it on one stream (CUDA events on
    # that stream), so its average launch duration is elapsed / K.
    avg_launch = elapsed / args.steps
    bytes_launch = step_weight_bytes() + K_DIM * 4 + sum(N_DIMS) * 4

    # ---- end to end through the public API with host buffers
    x_host = x.cpu().pin_memory()
    x_dev = torch.empty_like(x)
    outs_host = [torch.empty((1, n), pin_memory=True) for n in N_DIMS]
    for i in range(args.warmup):
        x_dev.copy_(x_host, non_blocking=True)
        step(i, x_dev)
        for o, oh in zip(outs, outs_host):
            oh.copy_(o, non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for i in range(args.steps):
        x_dev.copy_(x_host, non_blocking=True)
        step(i, x_dev)
        for o, oh in zip(outs, outs_host):
            oh.copy_(o, non_blocking=True)
    e_end.record(stream)
    torch.cuda.synchronize()
    e2e_elapsed = e_start.elapsed_time(e_end) / 1e3
    if dist is not None:
        t = torch.tensor([e2e_elapsed], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_elapsed = float(t.item())
    pb.check_kernel_error()

    del graph
    peak, peak_kind = measured_peaks()
    if rank == 0:
        value = world * args.steps * step_ops() / elapsed_max / 1e9
        achieved = bytes_launch / avg_launch / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed_max / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8/int32 dot, fp32 fold (q4_0 x q8_0)",
            "data": "synthetic: seeded N(0,1) fp32 weights (quantized to q4_0 on device) and activations",
            "config": dict(workload_config(), parallelism=f"replicas x{world}" if world > 1 else "single GPU",
                           weight_copies=copies, weight_bytes_resident=copies * step_weight_bytes()),
            "weight_GBps": world * args.steps * step_weight_bytes() / elapsed_max / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": profile_traffic("gemv_q4_0_decode"),
                         "kernel": "gemv_kernel<q4_0, m=1, fp32 activations>, both matrices in one launch",
                         "bytes_per_launch": bytes_launch, "avg_launch_us": avg_launch * 1e6,
                         "timing": "CUDA events around K back-to-back launches on the launching stream, / K",
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s"},
            "clocks": clock_info,
            "e2e": {"value": world * args.steps * step_ops() / e2e_elapsed / 1e9, "unit": UNIT,
                    "h2d_bytes_per_step": K_DIM * 4, "d2h_bytes_per_step": sum(N_DIMS) * 4,
                    "api": "pfng_b200_compute_grouped (overlapped launches) with pinned host activations in, "
                   "host C out"},
            "gpu_launches": args.steps,
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the timed CPU baseline leg")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        return reference_arm(args)
    return ours(args)


if __name__ == "__main__":
    sys.exit(main())
