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


def step_weight_bytes(wtype: str = "q4_0") -> int:
    return sum(weight_bytes(wtype, n, K_DIM) for n in N_DIMS)


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


def profile_traffic(kernel_tag: str, variant: str | None = None):
    """DRAM bytes per launch from a committed ncu summary, if one exists (the
    line `traffic_bytes_per_launch:` or `traffic_bytes_per_launch (variant):`)."""
    path = ROOT / "profiles" / f"{kernel_tag}.md"
    if not path.exists():
        return None
    key = "traffic_bytes_per_launch" + (f" ({variant})" if variant else "") + ":"
    for line in path.read_text().splitlines():
        if line.startswith(key):
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


def workload_config(layout: str = "ggml", wtype: str = "q4_0"):
    if wtype == "q4_0":
        workload = ("configs[1]: q4_0 x q8_0 decode GEMV, M=1, (N,K) = (4096,4096) + (11008,4096), "
                    "activation quantized on device (fused)")
    else:
        workload = (f"decode GEMV with {wtype} x q8_K weights on the shapes of configs[1] (M=1, (N,K) = (4096,4096) "
                    "+ (11008,4096), activation quantized on device, fused); not a BASELINE configuration")
    return {
        "workload": workload,
        "m": 1, "n": list(N_DIMS), "k": K_DIM, "weight_type": wtype,
        "activation_type": "q8_0" if wtype == "q4_0" else "q8_K",
        "weight_layout": "ggml block_q4_0 rows" if layout == "ggml" else
                         "q4_0 planar rows (same bytes, repacked once on the device before timing)",
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
    wtype = args.wtype
    copies = max(2, -(-4 * L2_BYTES // step_weight_bytes(wtype)))
    gen = torch.Generator(device="cuda").manual_seed(1 + rank)
    planar = args.layout == "planar"
    if planar and wtype != "q4_0":
        raise SystemExit("--layout planar applies to q4_0 weights")
    wt = pb.Q4_0_PLANAR if planar else pb.WTYPES[wtype]
    weights = []
    for _ in range(copies):
        per = []
        for n in N_DIMS:
            q = make_weights_device(pb, torch, wtype, n, K_DIM, gen)
            # planar: the one-time repack a reference adapter does in prepare
            per.append(pb.pack_q4_0_planar(q, n, K_DIM) if planar else q)
            del q
        weights.append(per)
    x = torch.randn((1, K_DIM), generator=torch.Generator(device="cuda").manual_seed(2), device="cuda")
    outs = [torch.empty((1, n), device="cuda") for n in N_DIMS]
    ws = torch.empty(max(1, pb.compute_workspace_size(pb.Q4_0, 1, max(N_DIMS), K_DIM)), dtype=torch.uint8,
                     device="cuda")
    torch.cuda.synchronize()

    # The weights are constant, so consecutive steps may overlap: each launch
    # starts streaming its weights while the previous one drains
    # (PFNG_B200_OVERLAP_WEIGHTS); activations and outputs stay ordered.
    calls = [pb.GroupedCall(wt, weights[r], N_DIMS, outs, x, overlap_weights=True) for r in range(copies)]

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
    bytes_launch = step_weight_bytes(wtype) + K_DIM * 4 + sum(N_DIMS) * 4

    # ---- end to end through the public API with host buffers.  Every step
    # copies its activation row from pinned host memory, runs the grouped
    # launch and reads its outputs (one contiguous [1][sum N] buffer) back to
    # pinned host memory, all on the launching stream; the K steps are
    # captured in one CUDA graph like the device-resident timing above (as a
    # decode loop would be), so the copies cost their transfer and latency,
    # not a host launch each.
    x_host = x.cpu().pin_memory()
    x_dev = torch.empty_like(x)
    out_dev = torch.empty((1, sum(N_DIMS)), device="cuda")
    out_host = torch.empty((1, sum(N_DIMS)), pin_memory=True)
    cols, o = [], 0
    for n in N_DIMS:
        cols.append(out_dev[:, o:o + n])
        o += n
    e2e_calls = [pb.GroupedCall(wt, weights[r], N_DIMS, cols, x_dev, overlap_weights=True) for r in range(copies)]

    def e2e_step(i):
        x_dev.copy_(x_host, non_blocking=True)
        e2e_calls[i % copies](stream=stream)
        out_host.copy_(out_dev, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph, stream=stream):
        for i in range(args.steps):
            e2e_step(i)
    e2e_graph.replay()
    torch.cuda.synchronize()
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    e2e_graph.replay()
    e_end.record(stream)
    torch.cuda.synchronize()
    del e2e_graph
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
            "scaling": "weak", "vs_baseline": None,
            "dtype": f"int8/int32 dot, fp32 fold ({wtype} x {'q8_0' if wtype == 'q4_0' else 'q8_K'})",
            "data": "synthetic: seeded N(0,1) fp32 weights (quantized on device) and activations"
                    if wtype != "iq2_xxs" else "synthetic: seeded iq2_xxs blocks (uniform indices, signs, scales) "
                    "and N(0,1) activations",
            "config": dict(workload_config(args.layout, wtype),
                           parallelism=f"replicas x{world}" if world > 1 else "single GPU",
                           weight_copies=copies, weight_bytes_resident=copies * step_weight_bytes(wtype)),
            "weight_GBps": world * args.steps * step_weight_bytes(wtype) / elapsed_max / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": profile_traffic("gemv_q4_0_planar_decode") if planar
                         else profile_traffic("gemv_q4_0_decode") if wtype == "q4_0"
                         else profile_traffic("gemv_k_types_decode", wtype),
                         "kernel": f"gemv_kernel<{'q4_0 planar' if planar else wtype}, m=1, fp32 activations>, "
                                   "both matrices in one launch",
                         "bytes_per_launch": bytes_launch, "avg_launch_us": avg_launch * 1e6,
                         "timing": "CUDA events around K back-to-back launches on the launching stream, / K",
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s"},
            "clocks": clock_info,
            "e2e": {"value": world * args.steps * step_ops() / e2e_elapsed / 1e9, "unit": UNIT,
                    "h2d_bytes_per_step": K_DIM * 4, "d2h_bytes_per_step": sum(N_DIMS) * 4,
                    "api": "pfng_b200_compute_grouped (overlapped launches) with pinned host activations in and "
                   "host C out every step, the K steps captured in one CUDA graph"},
            "gpu_launches": args.steps,
        }
        if not args.no_cpu_baseline and wtype == "q4_0":
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0



# ------------------------------------------------------- other BASELINE configs
def make_weights_device(pb, torch, wtype: str, n: int, k: int, gen, std: float = 1.0):
    """Seeded synthetic weights on the device in the ggml layout of `wtype`."""
    if wtype == "q4_0":
        return pb.quantize_q4_0(torch.randn((n, k), generator=gen, device="cuda") * std)
    if wtype == "q4_K":
        return pb.quantize_q4_K(torch.randn((n, k), generator=gen, device="cuda") * std)
    nb = n * (k // 256)  # iq2_xxs: random grid indices / signs / scales, d ~ U[1e-3, 1e-2]
    blocks = torch.randint(0, 256, (nb, 66), generator=gen, device="cuda", dtype=torch.int32).to(torch.uint8)
    d = torch.empty(nb, device="cuda").uniform_(1e-3, 1e-2, generator=gen).half()
    blocks[:, :2] = d.view(torch.uint8).view(nb, 2)
    return blocks.reshape(-1).contiguous()


def weight_bytes(wtype: str, n: int, k: int) -> int:
    return n * (k // 32 * 18 if wtype == "q4_0" else k // 256 * (144 if wtype == "q4_K" else 66))


def int8_peak_tops():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return 2.0 * float(json.loads(path.read_text())["bf16_tflops"]), "2x measured bf16 GEMM (MEASURED_PEAKS.json)"
    return 2.0 * 1590.0, "2x fallback bf16 1.59 PFLOP/s"


def time_graph(torch, stream, fn, steps: int, warmup: int) -> float:
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            fn(i)
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    graph.replay()
    b.record(stream)
    torch.cuda.synchronize()
    del graph
    return a.elapsed_time(b) / 1e3


def prefill(args) -> int:
    """configs[0] / [2] / [3]: one C = quantize(x) . W^T, M=480 N=1536 K=1536, on one GPU."""
    import torch
    import pfng_b200 as pb
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    m, n, k = args.m, args.n, args.k
    gen = torch.Generator(device="cuda").manual_seed(1)
    per = weight_bytes(args.wtype, n, k) + m * k * 4
    copies = max(2, -(-4 * L2_BYTES // per))
    ws_ = [make_weights_device(pb, torch, args.wtype, n, k, gen) for _ in range(copies)]
    xs = [torch.randn((m, k), generator=gen, device="cuda") for _ in range(copies)]
    if args.out == "f32":
        out = torch.empty((m, n), device="cuda")
        wsp = torch.empty(max(1, pb.compute_workspace_size(args.wtype, m, n, k)), dtype=torch.uint8, device="cuda")
        step = lambda i: pb.compute(args.wtype, ws_[i % copies], xs[i % copies], n, out=out, workspace=wsp,
                                    stream=stream)
    else:
        # the result in another format, converted in the GEMM's epilogue
        out = pb._out_tensor(pb.OUT_FORMATS[args.out], m, n, "cuda")
        wsp = torch.empty(max(1, pb.lib().pfng_b200_compute_out_workspace_size(
            pb._wt(args.wtype), pb.OUT_FORMATS[args.out], m, n, k, 0)), dtype=torch.uint8, device="cuda")
        step = lambda i: pb.compute_out(args.wtype, ws_[i % copies], xs[i % copies], n, args.out, out=out,
                                        workspace=wsp, stream=stream)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        elapsed = time_graph(torch, stream, step, args.steps, args.warmup)
    pb.check_kernel_error()
    ops = 2.0 * m * n * k
    peak, peak_src = int8_peak_tops()
    achieved = ops / (elapsed / args.steps) / 1e12
    print(json.dumps({
        "metric": METRIC, "workload": f"{args.wtype} GEMM M={m} N={n} K={k} (quantize x + matmul, one step)"
                                      + ("" if args.out == "f32" else f", output {args.out} (fused epilogue)"),
        "value": args.steps * ops / elapsed / 1e9, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "us_per_step": elapsed / args.steps * 1e6,
        "weight_GBps": args.steps * weight_bytes(args.wtype, n, k) / elapsed / 1e9,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s",
                     "frac": achieved / peak, "peak_source": peak_src},
        "clocks": clocks.summary(), "l2": f"{copies} rotating (W, x) copies > 4x L2",
    }), flush=True)
    return 0


LLAMA_SHAPES = [(nn, kk) for nn, kk in ((4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096))]


def llama(args) -> int:
    """Llama-2-7B q4_0 prefill shapes, weight rows sharded over the ranks, x quantized on
    rank 0 and broadcast as q8_0, each rank's output columns stored into every rank's C by its matmul
    (pfng_b200_mm_gather); the NCCL all-gather variant is timed beside it.  One JSON line per shape."""
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
    torch.cuda.set_stream(stream)
    granule = 128
    ms = [args.m] if args.m_given else [32, 512, 2048]
    for m in ms:
        for n, k in LLAMA_SHAPES:
            b, e = pb.shard_rows(n, world, rank, granule)
            width = max(pb.shard_rows(n, world, r, granule)[1] - pb.shard_rows(n, world, r, granule)[0]
                        for r in range(world))
            gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
            per = weight_bytes("q4_0", max(e - b, 1), k) + m * k * 4
            copies = max(2, -(-4 * L2_BYTES // per))
            wsh = [make_weights_device(pb, torch, "q4_0", max(e - b, 1), k, gen, 0.02) for _ in range(copies)]
            x = torch.randn((m, k), generator=torch.Generator(device="cuda").manual_seed(7), device="cuda")
            slice_ = torch.zeros((m, width), device="cuda")
            gathered = torch.empty((world, m, width), device="cuda")
            full = torch.empty((m, n), device="cuda")
            wsp = torch.empty(max(1, pb.compute_workspace_size("q4_0", m, width, k)), dtype=torch.uint8,
                              device="cuda")

            def local_gemm(i):
                if e > b:
                    pb.compute("q4_0", wsh[i % copies], x, e - b, out=slice_[:, : e - b], workspace=wsp,
                               stream=stream)

            def full_step(i):
                if dist is not None:
                    dist.broadcast(x, src=0)
                local_gemm(i)
                if dist is not None:
                    dist.all_gather_into_tensor(gathered, slice_)
                    pb.unshard_columns(gathered, m, n, world, granule, out=full, stream=stream)
                else:
                    full.copy_(slice_[:, :n])

            # the all-gather fused into the GEMM: every rank's epilogue stores
            # its columns into every rank's full C over NVLink (CUDA IPC);
            # a one-element all-reduce after it orders the ranks
            # rank 0 quantizes x and broadcasts the q8_0 bytes (1.06 bytes per
            # value instead of 4); a one-element all-reduce after the matmul
            # orders the ranks
            gc = pb.GatheredC(m, n) if dist is not None else None
            dsts = gc.destinations(b) if gc is not None else [full]
            flag = torch.zeros(1, device="cuda")
            aq = torch.empty(m * (k // 32) * pb.Q8_0_BYTES, dtype=torch.uint8, device="cuda")
            wsm = torch.empty(max(1, pb.mm_workspace_size("q4_0", m, width, k)), dtype=torch.uint8, device="cuda")

            def fused_step(i):
                if rank == 0:
                    pb.quantize_q8_0(x, out=aq, stream=stream)
                if dist is not None:
                    dist.broadcast(aq, src=0)
                if e > b:
                    pb.mm_gather("q4_0", wsh[i % copies], aq, m, e - b, k, dsts, n, workspace=wsm, stream=stream)
                if dist is not None:
                    dist.all_reduce(flag)

            def timed(fn):
                for i in range(args.warmup):
                    fn(i)
                torch.cuda.synchronize()
                if dist is not None:
                    dist.barrier()
                a, bb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for i in range(args.steps):
                    fn(i)
                bb.record(stream)
                torch.cuda.synchronize()
                t = a.elapsed_time(bb) / 1e3
                if dist is not None:
                    tt = torch.tensor([t], device="cuda", dtype=torch.float64)
                    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                    t = float(tt.item())
                return t

            t_compute = timed(local_gemm)
            t_nccl = timed(full_step)
            t_e2e = timed(fused_step)
            pb.check_kernel_error()
            if gc is not None:
                torch.cuda.synchronize()
                gc.close()
            if rank == 0:
                ops = 2.0 * m * n * k
                peak, peak_src = int8_peak_tops()
                print(json.dumps({
                    "metric": METRIC, "workload": f"configs[4] Llama-2-7B q4_0 M={m} N={n} K={k}",
                    "n_gpus": world, "scaling": "strong", "value": args.steps * ops / t_e2e / 1e9, "unit": UNIT,
                    "compute_only": args.steps * ops / t_compute / 1e9, "us_per_step_e2e": t_e2e / args.steps * 1e6,
                    "us_per_step_compute": t_compute / args.steps * 1e6,
                    "us_per_step_e2e_nccl_all_gather": t_nccl / args.steps * 1e6,
                    "compute_frac_of_int8_peak": ops / (t_compute / args.steps) / 1e12 / peak,
                    "peak_source": peak_src, "rows_per_rank": e - b,
                    "exchange": "x quantized to q8_0 on rank 0 and NCCL-broadcast; each rank's matmul stores its C "
                    "columns into every rank's C (CUDA IPC over NVLink, pfng_b200_mm_gather); one-element NCCL "
                    "all-reduce as the completion barrier; us_per_step_e2e_nccl_all_gather: fp32 x broadcast, "
                    "NCCL all-gather of C slices and a device unshard instead" if world > 1 else "none",
                }), flush=True)
            del wsh, gathered, full, slice_
            torch.cuda.empty_cache()
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
    ap.add_argument("--workload", choices=["decode", "prefill", "llama"], default="decode",
                    help="decode: configs[1] (the bench line); prefill: configs[0]/[2]/[3]; llama: configs[4]")
    ap.add_argument("--wtype", choices=["q4_0", "q4_K", "iq2_xxs"], default="q4_0")
    ap.add_argument("--out", choices=["f32", "f16", "bf16", "q8_0"], default="f32",
                    help="prefill: format of C, converted in the GEMM's epilogue")
    ap.add_argument("--layout", choices=["ggml", "planar"], default="ggml",
                    help="decode: q4_0 weights as ggml blocks or repacked once into the planar row layout")
    ap.add_argument("--m", type=int, default=None)
    ap.add_argument("--n", type=int, default=1536)
    ap.add_argument("--k", type=int, default=1536)
    args = ap.parse_args()
    args.m_given = args.m is not None
    if args.m is None:
        args.m = 480
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        return reference_arm(args)
    if args.workload == "prefill":
        return prefill(args)
    if args.workload == "llama":
        return llama(args)
    return ours(args)


if __name__ == "__main__":
    sys.exit(main())
