"""The reference's own pfng-bench CLI driving the B200 kernel IDs.

integration/build_pfng_bench.py builds pfng-bench from the reference's
sources (bench/main.cpp, the kernel registry, run_benchmark, llama_reference)
with the platform overlay -- PlatformId::NvidiaB200, its CUDA detector, the
three kernel IDs declared as cmake/Kernel.cmake declares kernels -- and the
adapters of qgemm-perf-framework-ng_b200/host/b200_kernels.cpp.  The CLI
flags (--kernel/--m/--n/--k/--warmup/--samples/--iterations) and the built-in
verification (every element against llama_reference::compute, failing when
both its absolute and relative error exceed 1e-3; bench/framework/
benchmark.cpp:131-168) are the reference's, unchanged.

The binary is built where the reference checkout is present and travels
with the tree; these tests skip when it is absent.  Hosts without a PMU (as
this pool's containers) refuse the hardware "cycles" perf event, so the
verification runs time with the software "task-clock" event and an explicit
--iterations (run_benchmark calibrates with "cycles" otherwise); the run with
the CLI's default event is checked to verify before the perf-event refusal.
"""
import pathlib
import subprocess

import pytest

BIN = pathlib.Path(__file__).resolve().parent.parent / "integration" / "_build" / "pfng-bench"
IDS = ["q4_0-q8_0-B200", "q4_K-q8_K-B200", "iq2_xxs-q8_K-B200"]

needs_bin = pytest.mark.skipif(not BIN.exists(), reason="pfng-bench not built (needs the reference checkout)")


def run(*args, timeout=600):
    return subprocess.run([str(BIN), *map(str, args)], capture_output=True, text=True, timeout=timeout)


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except ImportError:
        return False


@needs_bin
def test_build_info_names_the_b200_platform():
    r = run("--build-info")
    assert r.returncode == 0, r.stderr
    assert "platform: nvidia-b200" in r.stdout


@needs_bin
def test_platform_check_fails_closed_without_a_b200():
    if gpu_available():
        pytest.skip("a GPU is present")
    r = run("--check-platform")
    assert r.returncode == 3 and "platform check failed" in r.stderr


@needs_bin
@pytest.mark.gpu
def test_platform_check_and_list():
    r = run("--check-platform")
    assert r.returncode == 0 and "platform check: PASS" in r.stdout, r.stdout + r.stderr
    r = run("--list")
    assert r.returncode == 0, r.stderr
    listed = [line.split()[0] for line in r.stdout.splitlines() if line.strip()]
    assert listed == IDS
    assert all("[platform=nvidia-b200]" in line for line in r.stdout.splitlines() if line.strip())


@needs_bin
@pytest.mark.gpu
@pytest.mark.parametrize("kid,m,n,k", [
    (IDS[0], 1, 4096, 4096), (IDS[0], 480, 1536, 1536), (IDS[0], 3, 300, 1024), (IDS[0], 33, 200, 96),
    (IDS[1], 480, 1536, 1536), (IDS[1], 1, 1536, 1536),
    (IDS[2], 480, 1536, 1536), (IDS[2], 1, 1536, 1536),
])
def test_cli_verifies_every_kernel(kid, m, n, k):
    r = run("--kernel", kid, "--m", m, "--n", n, "--k", k, "--warmup", 2, "--samples", 3, "--iterations", 5,
            "--perf-events", "task-clock")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "verify: PASS" in r.stdout and f"error elements: 0/{m * n}" in r.stdout
    assert "perf: event=task-clock" in r.stdout and "checksum:" in r.stdout


@needs_bin
@pytest.mark.gpu
def test_cli_default_invocation():
    # SURVEY's minimum slice, with the CLI's default perf event ("cycles"):
    # verification must pass; a host without a PMU then refuses the event
    r = run("--kernel", IDS[0], "--m", 1, "--n", 4096, "--k", 4096)
    assert "error elements: 0/4096" in r.stdout, r.stdout + r.stderr
    if r.returncode == 0:
        assert "verify: PASS" in r.stdout
    else:
        assert "perf_event_open(cycles)" in r.stdout, r.stdout + r.stderr


@needs_bin
@pytest.mark.gpu
def test_cli_rejects_unknown_kernel():
    r = run("--kernel", "no-such-kernel", "--m", 1, "--n", 64, "--k", 256)
    assert r.returncode == 2 and "unknown kernel" in r.stderr
