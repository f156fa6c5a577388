"""Benchmark of the B200 block-quantized matmul hot path.

Metric: 2MNK int-ops/s and weight GB/s against the int8
tensor-core / HBM roofline, on 1/2/4/8 B200s.

Headline workload (the bench line; BASELINE.json configs[4], its largest
shape, the only configuration quoted for 1/2/4/8 GPUs): one step is
C[2048][32000] = quantize_q8_0(x) . W^T with q4_0 weights W [32000][4096]
(seeded N(0, 0.02), quantized on the device by the bit-exact q4_0 quantizer)
and fp32 activations x [2048][4096] (seeded N(0, 1)).
  * 1 GPU: pfng_b200_compute_q4_0 (activation quantizer + tensor-core GEMM).
  * N GPUs (torchrun, one process per GPU): the weight rows are sharded
    (pfng_b200_shard_rows, 128-row granules); rank 0 quantizes x to q8_0 and
    NCCL-broadcasts the bytes; every rank's pfng_b200_mm_gather computes its
    columns of C and stores them into every rank's full C over NVLink (CUDA
    IPC peer pointers); a one-element NCCL all-reduce orders the ranks.  The
    total work is fixed ("scaling": "strong").
Inputs are larger than L2: the steps rotate over copies of (W, x) totalling
more than 4x the 126 MB L2, and every step writes the 262 MB C.

Keys of the JSON line beyond the driver contract:
  * roofline   -- the GEMM kernel alone (pfng_b200_mm_prepared on prepared
                  activations; K back-to-back launches between CUDA events on
                  the launching stream), 2 m n_rank k per launch against 2x
                  the measured bf16 tensor peak (the dense int8 rate); traffic
                  from profiles/ncu_traffic.json (ncu DRAM bytes of one launch).
  * e2e        -- the same step through the public entry points with pinned
                  HOST x in and HOST C out every step; the copies of step i+1
                  (x in) and i-1 (C out) run on two more streams beside step
                  i's compute (double-buffered device x and C).
  * sweep      -- every other BASELINE configuration, measured in the same
                  run: configs[0]/[2]/[3] (480x1536x1536 for q4_0, q4_K,
                  iq2_xxs), configs[1] (the m=1 decode GEMV) and all twelve
                  configs[4] shapes (sharded under N GPUs).
  * cpu_baseline -- the reference's own scalar llama_reference code
                  (oracle/_ref; the C restatement if it was not built) on a
                  row sample of the headline workload, at 1 thread and at all
                  host threads, min and median over samples.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--repeats R]
                  [--impl ours|reference] [--no-sweep] [--no-cpu-baseline]

--impl reference times the reference's own CPU implementation of the same
step (quantize + dots of bench/llama_reference, element-parallel over all
host threads) on a row sample of the headline workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
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
HEADLINE = ("q4_0", 2048, 32000, 4096)  # configs[4], largest shape
LLAMA_MS = (32, 512, 2048)
LLAMA_NK = ((4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096))
SMALL_CONFIGS = (("configs[0]", "q4_0"), ("configs[2]", "q4_K"), ("configs[3]", "iq2_xxs"))  # 480x1536x1536
DECODE_NS, DECODE_K = (4096, 11008), 4096  # configs[1]
GRANULE = 128
L2_BYTES = 126 * 1024 * 1024


def weight_bytes(wtype: str, n: int, k: int) -> int:
    return n * (k // 32 * 18 if wtype == "q4_0" else k // 256 * (144 if wtype == "q4_K" else 66))


def dist_env():
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), \
        int(os.environ.get("LOCAL_RANK", "0"))


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "int8_tops": 2.0 * float(d["bf16_tflops"]),
                "source": "measured (MEASURED_PEAKS.json: hbm_gbs; int8 = 2 x bf16_tflops burst)"}
    return {"hbm_gbs": 6650.0, "int8_tops": 2.0 * 1590.0,
            "source": "fallback (6.65 TB/s; int8 = 2 x 1.59 PFLOP/s bf16)"}


def ncu_traffic(key: str):
    """DRAM bytes (read + write) per launch from the committed ncu counters, or None."""
    path = ROOT / "profiles" / "ncu_traffic.json"
    if not path.exists():
        return None
    entry = json.loads(path.read_text()).get(key)
    if not entry:
        return None
    return float(entry["dram_bytes_read"]) + float(entry["dram_bytes_write"])


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


# ====================================================================== CPU
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


def cpu_model() -> str:
    try:
        for line in pathlib.Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def host_headline_weights(lib, seed: int = 11):
    """q4_0 blocks of seeded N(0, 0.02) weights [N][K], quantized by the CPU library."""
    import numpy as np
    _, _, n, k = HEADLINE
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
    return lib.quantize("q4_0", w)


def cpu_rows_step(lib, kind: str, w, x, threads: int) -> float:
    """Seconds for one sample: quantize x's rows to q8_0 and multiply by all of W."""
    _, _, n, k = HEADLINE
    t0 = time.perf_counter()
    a = lib.quantize("q8_0", x)
    if kind == "reference":
        lib.mm_threads("q4_0", w, a, x.shape[0], n, k, threads)
    else:
        lib.mm("q4_0", w, a, x.shape[0], n, k)
    return time.perf_counter() - t0


def cpu_sample_rows(lib, kind, w, threads: int, target_s: float, seed: int) -> int:
    import numpy as np
    _, m, _, k = HEADLINE
    x = np.random.default_rng(seed).standard_normal((1, k), dtype=np.float32)
    one = cpu_rows_step(lib, kind, w, x, threads)
    return max(1, min(m, int(target_s / max(one, 1e-6))))


def cpu_measure(lib, kind, w, threads: int, rows: int, samples: int, seed: int) -> dict:
    import numpy as np
    _, _, n, k = HEADLINE
    x = np.random.default_rng(seed).standard_normal((rows, k), dtype=np.float32)
    cpu_rows_step(lib, kind, w, x, threads)  # warm (thread pool, pages)
    times = [cpu_rows_step(lib, kind, w, x, threads) for _ in range(samples)]
    ops = 2.0 * rows * n * k
    return {"threads": threads, "rows": rows, "samples": samples,
            "min_s": min(times), "median_s": statistics.median(times),
            "value_median": ops / statistics.median(times) / 1e9, "value_best": ops / min(times) / 1e9}


def cpu_baseline() -> dict:
    lib, kind = cpu_library()
    threads = cpu_threads() if kind == "reference" else 1
    w = host_headline_weights(lib)
    one = cpu_measure(lib, kind, w, 1, cpu_sample_rows(lib, kind, w, 1, 0.3, 3), 5, 4)
    allt = cpu_measure(lib, kind, w, threads, cpu_sample_rows(lib, kind, w, threads, 0.3, 5), 5, 6) \
        if threads > 1 else one
    _, m, n, k = HEADLINE
    return {
        "value": allt["value_median"], "unit": UNIT, "cores": threads, "kind": kind,
        "sample": (f"headline workload q4_0 M={m} N={n} K={k}: {allt['rows']} of the {m} activation rows per sample "
                   f"(q8_0 quantization of those rows + their dot products with all {n} weight rows), "
                   f"median of {allt['samples']} samples at {threads} threads; scaled by the ops of the sample"),
        "one_thread": one, "all_threads": allt, "cpu_model": cpu_model(), "nproc": os.cpu_count(),
        "code": "bench/llama_reference quantize_row_q8_0 + dot_q4_0_q8_0 (oracle/_ref), element-parallel "
                "OpenMP over C" if kind == "reference" else "C restatement of bench/llama_reference (oracle)",
    }


def reference_arm(args) -> int:
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    import numpy as np
    lib, kind = cpu_library()
    threads = cpu_threads() if kind == "reference" else 1
    w = host_headline_weights(lib)
    rows = cpu_sample_rows(lib, kind, w, threads, 0.25, 5)
    _, m, n, k = HEADLINE
    x = np.random.default_rng(6).standard_normal((rows, k), dtype=np.float32)
    for _ in range(args.warmup):
        cpu_rows_step(lib, kind, w, x, threads)
    times = [cpu_rows_step(lib, kind, w, x, threads) for _ in range(args.steps)]
    ops = 2.0 * rows * n * k
    total = sum(times)
    value = args.steps * ops / total / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8/int32 dot, fp32 fold (q4_0 x q8_0)",
        "data": "synthetic: seeded N(0,0.02) weights and N(0,1) activations, quantized by the reference quantizers",
        "config": headline_config(world),
        "weight_GBps": args.steps * weight_bytes("q4_0", n, k) / total / 1e9,
        "step_min_ms": min(times) * 1e3, "step_median_ms": statistics.median(times) * 1e3,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"each step: {rows} of the {m} activation rows (q8_0 quantization + dot products "
                                   f"with all {n} weight rows), scaled by the ops of the sample",
                         "cpu_model": cpu_model(), "nproc": os.cpu_count()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ====================================================================== GPU
def headline_config(world: int) -> dict:
    wtype, m, n, k = HEADLINE
    return {
        "workload": f"configs[4] largest shape: {wtype} x q8_0 prefill GEMM M={m} N={n} K={k} (Llama-2-7B output "
                    "projection), fp32 activations quantized on the device each step",
        "m": m, "n": n, "k": k, "weight_type": wtype, "activation_type": "q8_0",
        "parallelism": "single GPU" if world == 1 else
        f"weight rows sharded over {world} GPUs (x broadcast as q8_0 by NCCL, C all-gathered by the matmul over "
        "NVLink peer stores)",
        "l2": "inputs larger than L2: (W, x) copies totalling > 4x the 126 MB L2 rotate; every step writes C (262 MB)",
    }


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


class Ctx:
    """Per-process state: torch, the binding, the process group and the stream."""

    def __init__(self):
        import torch
        import pfng_b200 as pb
        self.torch, self.pb = torch, pb
        self.world, self.rank, self.local = dist_env()
        torch.cuda.set_device(self.local)
        self.dist = None
        if self.world > 1:
            import torch.distributed as dist
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.dist = dist
        self.stream = torch.cuda.Stream()
        torch.cuda.set_stream(self.stream)

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()

    def max_over_ranks(self, t: float) -> float:
        if self.dist is None:
            return t
        v = self.torch.tensor([t], device="cuda", dtype=self.torch.float64)
        self.dist.all_reduce(v, op=self.dist.ReduceOp.MAX)
        return float(v.item())

    def timed(self, fn, steps: int, warmup: int, repeats: int) -> list[float]:
        """Seconds of `repeats` timed regions of `steps` calls of fn(i), each
        bracketed by barrier + synchronize, CUDA events on the stream, max over ranks."""
        torch = self.torch
        for i in range(warmup):
            fn(i)
        torch.cuda.synchronize()
        out = []
        for _ in range(repeats):
            self.barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(self.stream)
            for i in range(steps):
                fn(i)
            b.record(self.stream)
            torch.cuda.synchronize()
            self.barrier()
            out.append(self.max_over_ranks(a.elapsed_time(b) / 1e3))
        return out

    def timed_graph(self, fn, steps: int, warmup: int, repeats: int) -> list[float]:
        """timed() with the `steps` calls captured in one CUDA graph (single-GPU small shapes)."""
        torch = self.torch
        for i in range(warmup):
            fn(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.stream):
            for i in range(steps):
                fn(i)
        graph.replay()
        torch.cuda.synchronize()
        out = []
        for _ in range(repeats):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(self.stream)
            graph.replay()
            b.record(self.stream)
            torch.cuda.synchronize()
            out.append(a.elapsed_time(b) / 1e3)
        del graph
        return out


class ShardedStep:
    """One step of the sharded product on this rank: x (rank 0) -> q8_0 ->
    broadcast -> this rank's columns of C into every rank's full C -> barrier."""

    def __init__(self, ctx: Ctx, m: int, n: int, k: int, nbuf: int = 1):
        pb, torch = ctx.pb, ctx.torch
        self.ctx, self.m, self.n, self.k = ctx, m, n, k
        self.b, self.e = pb.shard_rows(n, ctx.world, ctx.rank, GRANULE)
        self.gcs = [pb.GatheredC(m, n) for _ in range(nbuf)]
        self.aq = torch.empty(m * (k // 32) * pb.Q8_0_BYTES, dtype=torch.uint8, device="cuda")
        self.ws = torch.empty(max(1, pb.mm_workspace_size("q4_0", m, max(self.e - self.b, 1), k)),
                              dtype=torch.uint8, device="cuda")
        self.flag = torch.zeros(1, device="cuda")
        self.dsts = [gc.destinations(self.b) for gc in self.gcs]

    def __call__(self, w, x, buf: int = 0):
        ctx, pb = self.ctx, self.ctx.pb
        if ctx.rank == 0:
            pb.quantize_q8_0(x, out=self.aq, stream=ctx.stream)
        ctx.dist.broadcast(self.aq, src=0)
        if self.e > self.b:
            pb.mm_gather("q4_0", w, self.aq, self.m, self.e - self.b, self.k, self.dsts[buf], self.n,
                         workspace=self.ws, stream=ctx.stream)
        ctx.dist.all_reduce(self.flag)

    def c(self, buf: int = 0):
        return self.gcs[buf].tensor()

    def close(self):
        self.ctx.torch.cuda.synchronize()
        for gc in self.gcs:
            gc.close()


def launches_per_step(world: int, rank: int) -> int:
    """Kernels of this library one headline step launches on this rank."""
    if world == 1:
        return 2  # activation quantizer (split operand), GEMM
    # q8_0 quantizer on rank 0; q8_0 -> operand; the GEMM as two row bands
    # (their copies to the peers run on copy engines), or one GEMM and the
    # peer-store copy kernel for products under four 128-row tiles
    return (1 if rank == 0 else 0) + 3


def headline(ctx: Ctx, args) -> dict:
    torch, pb = ctx.torch, ctx.pb
    wtype, m, n, k = HEADLINE
    b, e = pb.shard_rows(n, ctx.world, ctx.rank, GRANULE)
    ns = max(e - b, 1)
    per_copy = weight_bytes(wtype, ns, k) + m * k * 4
    copies = max(2, -(-4 * L2_BYTES // per_copy))
    gen = torch.Generator(device="cuda").manual_seed(1000 + ctx.rank)
    gx = torch.Generator(device="cuda").manual_seed(7)
    W = [make_weights_device(pb, torch, wtype, ns, k, gen, 0.02) for _ in range(copies)]
    X = [torch.randn((m, k), generator=gx, device="cuda") for _ in range(copies)]
    torch.cuda.synchronize()

    # ---- device-resident step (value)
    sharded = None
    if ctx.world == 1:
        C = torch.empty((m, n), device="cuda")
        ws = torch.empty(max(1, pb.compute_workspace_size(wtype, m, n, k)), dtype=torch.uint8, device="cuda")

        def step(i):
            pb.compute(wtype, W[i % copies], X[i % copies], n, out=C, workspace=ws, stream=ctx.stream)
    else:
        sharded = ShardedStep(ctx, m, n, k, nbuf=2)

        def step(i):
            sharded(W[i % copies], X[i % copies], 0)

    with ClockSampler(torch.cuda.current_device()) as clocks:
        reps = ctx.timed(step, args.steps, args.warmup, args.repeats)
    ctx.pb.check_kernel_error()
    clock_info = clocks.summary()

    # ---- the GEMM kernel alone (roofline): K launches on prepared activations
    prep = [pb.prepare_activations(wtype, X[i]) for i in range(copies)]
    Cl = torch.empty((m, ns), device="cuda")
    kws = torch.empty(max(1, pb.mm_prepared_workspace_size(wtype, m, ns, k)), dtype=torch.uint8, device="cuda")

    def kstep(i):
        pb.mm_prepared(wtype, W[i % copies], prep[i % copies], m, ns, k, out=Cl, workspace=kws, stream=ctx.stream)

    kreps = ctx.timed(kstep, args.steps, args.warmup, args.repeats)
    pb.check_kernel_error()
    del prep, Cl

    # ---- end to end: host x in, host C out, copies overlapped with compute
    e2e_reps, h2d, d2h = e2e_headline(ctx, args, W, X[0], sharded)
    if sharded is not None:
        sharded.close()
    del W, X
    torch.cuda.empty_cache()

    ops = 2.0 * m * n * k
    t_step = statistics.median(reps)
    t_kernel = statistics.median(kreps)
    pk = peaks()
    achieved = 2.0 * m * ns * k / (t_kernel / args.steps) / 1e12
    traffic = ncu_traffic("gemm_q4_0_m2048_n32000_k4096") if ctx.world == 1 else None
    return {
        "value": args.steps * ops / t_step / 1e9, "ms_per_step": t_step / args.steps * 1e3,
        "ms_per_step_min": min(reps) / args.steps * 1e3, "ms_per_step_median": t_step / args.steps * 1e3,
        "repeats": args.repeats, "weight_GBps": args.steps * weight_bytes(wtype, n, k) / t_step / 1e9,
        "clocks": clock_info, "copies": copies,
        "roofline": {
            "bound": "tensor", "achieved": achieved, "peak": pk["int8_tops"], "unit": "TFLOP/s",
            "frac": achieved / pk["int8_tops"], "traffic": traffic,
            "kernel": "gemm_kernel (q4_0 x q8_0, int8 mma.sync m16n8k32, 128x128 tiles, direct B fragments, "
                      "stages filled by tensor-map bulk copies)"
                      if not os.environ.get("PFNG_B200_GEMM") else f"GEMM ({os.environ['PFNG_B200_GEMM']})",
            "flops_per_launch": 2.0 * m * ns * k, "avg_launch_us": t_kernel / args.steps * 1e6,
            "timing": "CUDA events around K back-to-back pfng_b200_mm_prepared launches on the launching "
                      "stream (median of repeats), / K; max over ranks",
            "peak_source": pk["source"] + "; TFLOP/s here counts int8 ops (2 per MAC)",
            "traffic_source": "profiles/ncu_traffic.json (dram__bytes_read.sum + dram__bytes_write.sum, one launch)"
            if traffic is not None else None,
        },
        "e2e": {"value": args.steps * ops / statistics.median(e2e_reps) / 1e9, "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": statistics.median(e2e_reps) / args.steps * 1e3,
                "api": "pfng_b200_compute_q4_0" if ctx.world == 1 else
                "pfng_b200_quantize_q8_0 (rank 0) + NCCL broadcast + pfng_b200_mm_gather + NCCL all-reduce",
                "copies": "pinned host x -> device every step and device C -> pinned host every step (each rank "
                          "its row band of the gathered C), on two more streams overlapping the previous / next "
                          "step's compute; double-buffered device x and C"},
        "gpu_launches": launches_per_step(ctx.world, ctx.rank) * args.steps,
    }


def e2e_headline(ctx: Ctx, args, W, x0, sharded):
    """Timed repeats of K pipelined steps with host x in and host C out; returns (seconds list, h2d, d2h)."""
    torch, pb = ctx.torch, ctx.pb
    wtype, m, n, k = HEADLINE
    copies = len(W)
    r0, r1 = (0, m) if ctx.world == 1 else (ctx.rank * m // ctx.world, (ctx.rank + 1) * m // ctx.world)
    x_host = x0.cpu().pin_memory()
    xd = [torch.empty_like(x0) for _ in range(2)]
    if ctx.world == 1:
        cd = [torch.empty((m, n), device="cuda") for _ in range(2)]
        ws = torch.empty(max(1, pb.compute_workspace_size(wtype, m, n, k)), dtype=torch.uint8, device="cuda")
    c_host = torch.empty((r1 - r0, n), pin_memory=True)
    s_h2d, s_d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev = {name: [torch.cuda.Event() for _ in range(2)] for name in ("x_ready", "x_free", "c_ready", "c_free")}
    loads_x = ctx.world == 1 or ctx.rank == 0

    def band(bi):
        return cd[bi][r0:r1] if ctx.world == 1 else sharded.c(bi)[r0:r1]

    def step(i):
        bi = i % 2
        with torch.cuda.stream(s_h2d):
            if i >= 2:
                s_h2d.wait_event(ev["x_free"][bi])
            if loads_x:
                xd[bi].copy_(x_host, non_blocking=True)
            ev["x_ready"][bi].record(s_h2d)
        ctx.stream.wait_event(ev["x_ready"][bi])
        if i >= 2:
            ctx.stream.wait_event(ev["c_free"][bi])
        if ctx.world == 1:
            pb.compute(wtype, W[i % copies], xd[bi], n, out=cd[bi], workspace=ws, stream=ctx.stream)
        else:
            sharded(W[i % copies], xd[bi], bi)
        ev["x_free"][bi].record(ctx.stream)
        ev["c_ready"][bi].record(ctx.stream)
        with torch.cuda.stream(s_d2h):
            s_d2h.wait_event(ev["c_ready"][bi])
            c_host.copy_(band(bi), non_blocking=True)
            ev["c_free"][bi].record(s_d2h)

    def run(steps):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(ctx.stream)
        s_h2d.wait_event(t0)
        s_d2h.wait_event(t0)
        for i in range(steps):
            step(i)
        for bi in range(min(2, steps)):
            ctx.stream.wait_event(ev["c_free"][bi])
        t1.record(ctx.stream)
        return t0, t1

    run(args.warmup)
    torch.cuda.synchronize()
    reps = []
    for _ in range(max(1, min(args.repeats, 3))):
        ctx.barrier()
        torch.cuda.synchronize()
        t0, t1 = run(args.steps)
        torch.cuda.synchronize()
        ctx.barrier()
        reps.append(ctx.max_over_ranks(t0.elapsed_time(t1) / 1e3))
    pb.check_kernel_error()
    del xd, c_host
    return reps, m * k * 4, m * n * 4


# ---------------------------------------------------------------- the sweep
def sweep_small(ctx: Ctx, args, wtype: str, m: int, n: int, k: int, std: float = 1.0) -> dict:
    """One single-GPU configuration through pfng_b200_compute_*, K steps in a CUDA graph."""
    torch, pb = ctx.torch, ctx.pb
    gen = torch.Generator(device="cuda").manual_seed(1)
    per = weight_bytes(wtype, n, k) + m * k * 4
    copies = max(2, -(-4 * L2_BYTES // per))
    Ws = [make_weights_device(pb, torch, wtype, n, k, gen, std) for _ in range(copies)]
    Xs = [torch.randn((m, k), generator=gen, device="cuda") for _ in range(copies)]
    out = torch.empty((m, n), device="cuda")
    wsp = torch.empty(max(1, pb.compute_workspace_size(wtype, m, n, k)), dtype=torch.uint8, device="cuda")
    reps = ctx.timed_graph(lambda i: pb.compute(wtype, Ws[i % copies], Xs[i % copies], n, out=out, workspace=wsp,
                                                stream=ctx.stream), args.steps, args.warmup, args.repeats)
    pb.check_kernel_error()
    t = statistics.median(reps) / args.steps
    ops = 2.0 * m * n * k
    return {"us_per_step": t * 1e6, "us_per_step_min": min(reps) / args.steps * 1e6, "value": ops / t / 1e9,
            "frac_int8_peak": ops / t / 1e12 / peaks()["int8_tops"],
            "weight_GBps": weight_bytes(wtype, n, k) / t / 1e9}


def sweep_decode(ctx: Ctx, args) -> dict:
    """x [1][4096] quantized in the GEMV launch, both q4_0 matrices in one launch."""
    torch, pb = ctx.torch, ctx.pb
    step_w = sum(weight_bytes("q4_0", n, DECODE_K) for n in DECODE_NS)
    copies = max(2, -(-4 * L2_BYTES // step_w))
    gen = torch.Generator(device="cuda").manual_seed(1)
    weights = [[make_weights_device(pb, torch, "q4_0", n, DECODE_K, gen) for n in DECODE_NS] for _ in range(copies)]
    x = torch.randn((1, DECODE_K), generator=torch.Generator(device="cuda").manual_seed(2), device="cuda")
    outs = [torch.empty((1, n), device="cuda") for n in DECODE_NS]
    calls = [pb.GroupedCall("q4_0", weights[r], DECODE_NS, outs, x, overlap_weights=True) for r in range(copies)]
    reps = ctx.timed_graph(lambda i: calls[i % copies](stream=ctx.stream), args.steps, args.warmup, args.repeats)
    pb.check_kernel_error()
    t = statistics.median(reps) / args.steps
    launch_bytes = step_w + DECODE_K * 4 + sum(DECODE_NS) * 4
    ops = sum(2.0 * n * DECODE_K for n in DECODE_NS)
    pk = peaks()
    return {"workload": "configs[1]: q4_0 decode GEMV M=1, (N,K) = (4096,4096) + (11008,4096), x quantized in the "
                        "same launch (pfng_b200_compute_grouped, overlapped launches, K steps in a CUDA graph)",
            "us_per_step": t * 1e6, "us_per_step_min": min(reps) / args.steps * 1e6, "value": ops / t / 1e9,
            "weight_GBps": step_w / t / 1e9, "hbm_GBps": launch_bytes / t / 1e9,
            "frac_hbm": launch_bytes / t / 1e9 / pk["hbm_gbs"], "bytes_per_launch": launch_bytes,
            "traffic": ncu_traffic("gemv_q4_0_decode"), "copies": copies}


def sweep_sharded(ctx: Ctx, args, m: int, n: int, k: int) -> dict:
    """A configs[4] shape under N GPUs: the sharded step (broadcast + matmul with fused gather)."""
    torch, pb = ctx.torch, ctx.pb
    step = ShardedStep(ctx, m, n, k)
    ns = max(step.e - step.b, 1)
    gen = torch.Generator(device="cuda").manual_seed(1000 + ctx.rank)
    per = weight_bytes("q4_0", ns, k) + m * k * 4
    copies = max(2, -(-4 * L2_BYTES // per))
    Ws = [make_weights_device(pb, torch, "q4_0", ns, k, gen, 0.02) for _ in range(copies)]
    x = torch.randn((m, k), generator=torch.Generator(device="cuda").manual_seed(7), device="cuda")
    reps = ctx.timed(lambda i: step(Ws[i % copies], x), args.steps, args.warmup, args.repeats)
    # the local GEMM alone
    C = torch.empty((m, ns), device="cuda")
    wsp = torch.empty(max(1, pb.compute_workspace_size("q4_0", m, ns, k)), dtype=torch.uint8, device="cuda")
    creps = ctx.timed(lambda i: pb.compute("q4_0", Ws[i % copies], x, ns, out=C, workspace=wsp, stream=ctx.stream),
                      args.steps, args.warmup, args.repeats)
    pb.check_kernel_error()
    step.close()
    t, tc = statistics.median(reps) / args.steps, statistics.median(creps) / args.steps
    ops = 2.0 * m * n * k
    return {"us_per_step": t * 1e6, "value": ops / t / 1e9, "us_per_step_compute_only": tc * 1e6,
            "frac_int8_peak_compute": 2.0 * m * ns * k / tc / 1e12 / peaks()["int8_tops"], "rows_per_rank": ns}


def sweep(ctx: Ctx, args) -> dict:
    out = {}
    if ctx.world == 1:
        for name, wtype in SMALL_CONFIGS:
            out[f"{name} {wtype} 480x1536x1536"] = sweep_small(ctx, args, wtype, 480, 1536, 1536)
        out["configs[1] decode"] = sweep_decode(ctx, args)
    for m in LLAMA_MS:
        for n, k in LLAMA_NK:
            key = f"configs[4] q4_0 {m}x{n}x{k}"
            out[key] = sweep_small(ctx, args, "q4_0", m, n, k, 0.02) if ctx.world == 1 else \
                sweep_sharded(ctx, args, m, n, k)
            ctx.torch.cuda.empty_cache()
    return out


def ours(args) -> int:
    ctx = Ctx()
    h = headline(ctx, args)
    sw = sweep(ctx, args) if not args.no_sweep else None
    if ctx.rank == 0:
        wtype, m, n, k = HEADLINE
        line = {
            "metric": METRIC, "value": h["value"], "unit": UNIT, "n_gpus": ctx.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": h["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8/int32 dot, fp32 fold (q4_0 x q8_0)",
            "data": "synthetic: seeded N(0,0.02) fp32 weights (quantized to q4_0 on the device) and N(0,1) fp32 "
                    "activations, the distributions BASELINE.json names for configs[4]",
            "config": dict(headline_config(ctx.world), weight_copies=h["copies"]),
            "weight_GBps": h["weight_GBps"], "ms_per_step_min": h["ms_per_step_min"],
            "ms_per_step_median": h["ms_per_step_median"], "repeats": h["repeats"],
            "roofline": h["roofline"], "clocks": h["clocks"], "e2e": h["e2e"], "gpu_launches": h["gpu_launches"],
        }
        if sw is not None:
            line["sweep"] = sw
        if ctx.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if ctx.dist is not None:
        ctx.dist.barrier()
        ctx.dist.destroy_process_group()
    return 0


# ------------------------------------------------ single-config dev runs
def one_config(args) -> int:
    """--workload prefill/decode: one configuration, printed as its own line (development runs)."""
    ctx = Ctx()
    if args.workload == "decode":
        r = sweep_decode(ctx, args)
    else:
        r = sweep_small(ctx, args, args.wtype, args.m, args.n, args.k, 0.02 if args.wtype == "q4_0" else 1.0)
    line = dict(workload=args.workload, wtype=args.wtype, m=args.m, n=args.n, k=args.k)
    line.update(r)
    print(json.dumps(line), flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--repeats", type=int, default=5, help="timed regions of K steps (min and median reported)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the timed CPU baseline leg")
    ap.add_argument("--no-sweep", action="store_true", help="only the headline configuration")
    ap.add_argument("--workload", choices=["headline", "prefill", "decode"], default="headline",
                    help="headline: the bench line; prefill / decode: one configuration (development)")
    ap.add_argument("--wtype", choices=["q4_0", "q4_K", "iq2_xxs"], default="q4_0")
    ap.add_argument("--m", type=int, default=480)
    ap.add_argument("--n", type=int, default=1536)
    ap.add_argument("--k", type=int, default=1536)
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        return reference_arm(args)
    if args.workload != "headline":
        return one_config(args)
    return ours(args)


if __name__ == "__main__":
    sys.exit(main())
