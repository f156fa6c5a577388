"""The C++ adapters of the reference's plugin interface (KernelCallbacks,
bench/framework/kernel_registry.h:92-101), driven by tests/host_harness:
the reference's own input generator (create_input, seed 1) and its
verification rule (benchmark.cpp:130-168: an element fails when both its
absolute and relative error exceed 1e-3 against llama_reference::compute).

The harness binary is built by `make -C tests/host_harness` where the
reference checkout is present (it compiles against the reference's headers)
and travels with the tree; the tests skip when it is not built.
"""
import pathlib
import subprocess

import pytest

HARNESS = pathlib.Path(__file__).resolve().parent / "host_harness" / "_build" / "pfng-bench-b200"
IDS = ["q4_0-q8_0-B200", "q4_K-q8_K-B200", "iq2_xxs-q8_K-B200"]

needs_harness = pytest.mark.skipif(not HARNESS.exists(), reason="host harness not built (needs the reference checkout)")


def run(*args, timeout=300):
    return subprocess.run([str(HARNESS), *map(str, args)], capture_output=True, text=True, timeout=timeout)


@needs_harness
def test_lists_the_three_kernel_ids():
    r = run("--list")
    assert r.returncode == 0, r.stderr
    assert [line.split()[0] for line in r.stdout.splitlines()] == IDS


@needs_harness
def test_rejects_bad_requests():
    assert run("--kernel", "no-such-kernel", "--m", 1, "--n", 1, "--k", 32).returncode == 2
    assert run("--kernel", IDS[0], "--m", 1, "--n", 64).returncode == 2


@needs_harness
def test_validate_reports_skip_reasons():
    # k not a multiple of the super-block: SKIP with a reason, on any host
    r = run("--kernel", IDS[1], "--m", 1, "--n", 64, "--k", 96)
    assert r.returncode == 4 and "multiple of 256" in r.stdout


@needs_harness
@pytest.mark.gpu
@pytest.mark.parametrize("kid,m,n,k", [
    (IDS[0], 480, 1536, 1536), (IDS[0], 1, 4096, 4096), (IDS[0], 3, 300, 1024), (IDS[0], 33, 200, 96),
    (IDS[1], 480, 1536, 1536), (IDS[1], 1, 1536, 1536),
    (IDS[2], 480, 1536, 1536), (IDS[2], 1, 1536, 1536),
])
def test_reference_verification_passes(kid, m, n, k):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    r = run("--kernel", kid, "--m", m, "--n", n, "--k", k, "--iterations", 5)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "verify: PASS" in r.stdout and "error elements: 0/" in r.stdout
