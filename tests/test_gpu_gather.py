"""pfng_b200_compute_gather on the GPU: C stored to several destinations.

* One process: every destination must hold exactly what pfng_b200_compute_*
  writes for the same arguments (bit for bit, on every path, with split-K
  and ragged shapes; copies written by the push kernel, by copy engines
  per row band (from four 128-row tiles the product runs as two bands, or
  as many as PFNG_B200_GATHER_BANDS forces, and each band's copies overlap
  the next band's GEMM), or by the
  GEMM epilogue), and nothing outside the [m][n] window of its rows; the
  pre-quantized entry (mm_gather) likewise equals mm().
* Two processes through CUDA IPC (GatheredC): each rank computes the columns
  of its weight rows into every rank's full C; after a host barrier every
  rank's C holds each rank's slice exactly as compute() gives it.  On a box
  with one GPU both ranks share it; no kernel waits on another rank.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import pfng_b200 as pb  # noqa: E402
from test_gpu_parity import act_kind, dev, dev_bytes, host, make_weights  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    yield
    pb.check_kernel_error()


CASES = [
    # (wtype, path, m, n, k)
    ("q4_0", "mma", 480, 1536, 1536), ("q4_0", "mma", 130, 300, 1536), ("q4_0", "mma", 32, 1024, 4096),
    ("q4_0", "mma", 2048, 256, 512), ("q4_0", "gemv", 1, 300, 1024), ("q4_0", "gemv", 5, 96, 512),
    ("q4_0", "simple", 3, 40, 256), ("q4_K", "mma", 70, 256, 1536), ("iq2_xxs", "mma", 40, 192, 512),
    ("q4_0_planar", "mma", 200, 384, 2048),
    # two row bands (the split follows the destination count and k; a ragged last band in the first two)
    ("q4_0", "mma", 1100, 640, 1024), ("q4_K", "mma", 600, 256, 1536), ("iq2_xxs", "mma", 1024, 192, 512),
]


@pytest.mark.parametrize("mode", ["push", "epilogue"])
@pytest.mark.parametrize("ndst", [1, 3, 8])
@pytest.mark.parametrize("wtype,path,m,n,k", CASES)
def test_every_destination_equals_compute(oracle, monkeypatch, wtype, path, m, n, k, ndst, mode):
    # mode: copies written by the push kernel after the GEMM (default) or by
    # the GEMM's epilogue
    if mode == "epilogue":
        monkeypatch.setenv("PFNG_B200_COPIES", "epilogue")
    rng = np.random.default_rng(m * 7 + n + k + ndst)
    base = "q4_0" if wtype == "q4_0_planar" else wtype
    wd = dev_bytes(make_weights(oracle, base, n, k, rng))
    if wtype == "q4_0_planar":
        wd = pb.pack_q4_0_planar(wd, n, k)
    xd = dev(rng.standard_normal((m, k)).astype(np.float32))
    ref = host(pb.compute(wtype, wd, xd, n, path=path))
    for ldd in (n, n + 5):  # n + 5: an odd row stride takes the scalar stores
        big = torch.full((ndst, m, ldd), -7.0, device="cuda")
        pb.compute_gather(wtype, wd, xd, n, [big[d] for d in range(ndst)], ldd, path=path)
        got = host(big)
        for d in range(ndst):
            assert got[d, :, :n].tobytes() == ref.tobytes(), f"{wtype}/{path}/{m}x{n}x{k} destination {d}"
            assert np.all(got[d, :, n:] == -7.0)


@pytest.mark.parametrize("bands", ["3", "8"])
@pytest.mark.parametrize("wtype,m,n,k", [("q4_0", 1100, 640, 1024), ("q4_K", 600, 256, 1536)])
def test_forced_band_counts(oracle, monkeypatch, bands, wtype, m, n, k):
    # PFNG_B200_GATHER_BANDS=3 / 8: equal row bands (ragged last band), each
    # band's copies overlapping the next band's GEMM; same bytes as compute()
    monkeypatch.setenv("PFNG_B200_GATHER_BANDS", bands)
    rng = np.random.default_rng(m + n + int(bands))
    wd = dev_bytes(make_weights(oracle, wtype, n, k, rng))
    xd = dev(rng.standard_normal((m, k)).astype(np.float32))
    ref = host(pb.compute(wtype, wd, xd, n, path="mma"))
    big = torch.full((3, m, n + 5), -7.0, device="cuda")
    pb.compute_gather(wtype, wd, xd, n, [big[d] for d in range(3)], n + 5, path="mma")
    got = host(big)
    for d in range(3):
        assert got[d, :, :n].tobytes() == ref.tobytes(), f"{wtype} {m}x{n}x{k} bands={bands} destination {d}"
        assert np.all(got[d, :, n:] == -7.0)


@pytest.mark.parametrize("wtype,path,m,n,k", [c for c in CASES if c[1] != "simple"])
def test_mm_gather_equals_mm(oracle, wtype, path, m, n, k):
    rng = np.random.default_rng(m + 3 * n + k)
    base = "q4_0" if wtype == "q4_0_planar" else wtype
    wd = dev_bytes(make_weights(oracle, base, n, k, rng))
    if wtype == "q4_0_planar":
        wd = pb.pack_q4_0_planar(wd, n, k)
    a = dev_bytes(oracle.quantize(act_kind(base), rng.standard_normal((m, k)).astype(np.float32)))
    ref = host(pb.mm(wtype, wd, a, m, n, k, path=path))
    outs = [torch.full((m, n), -7.0, device="cuda") for _ in range(3)]
    pb.mm_gather(wtype, wd, a, m, n, k, outs, n, path=path)
    for o in outs:
        assert host(o).tobytes() == ref.tobytes(), f"{wtype}/{path}/{m}x{n}x{k}"


def test_zero_k_and_empty_shapes():
    w = torch.zeros(18, dtype=torch.uint8, device="cuda")
    outs = [torch.full((3, 8), 5.0, device="cuda") for _ in range(2)]
    pb.compute_gather("q4_0", w, torch.zeros((3, 0), device="cuda"), 8, outs, 8)
    assert all(float(o.abs().sum()) == 0.0 for o in outs)
    pb.compute_gather("q4_0", w, torch.zeros((0, 32), device="cuda"), 8, outs, 8)  # m = 0: nothing


def test_gather_rejections():
    w = torch.zeros(18 * 8 * 64, dtype=torch.uint8, device="cuda")
    x = torch.zeros((2, 256), device="cuda")
    c = torch.zeros((2, 64), device="cuda")
    for bad, status in (([], -1), ([c] * 9, -1), ([c, 0], -1)):
        with pytest.raises(pb.PfngError) as e:
            pb.compute_gather("q4_0", w, x, 64, bad, 64)
        assert e.value.status == status
    with pytest.raises(pb.PfngError) as e:
        pb.compute_gather("q4_0", w, x, 64, [c, c.data_ptr() + 2], 64)  # misaligned destination
    assert e.value.status == -3
    with pytest.raises(pb.PfngError) as e:
        pb.compute_gather("q4_0", w, x, 64, [c, c], 32)  # ldd < n
    assert e.value.status == -2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("m,n,k,path", [(512, 1000, 1024, "mma"), (32, 4096, 4096, "mma"), (4, 640, 512, "gemv")])
def test_gather_across_processes(m, n, k, path):
    import torch.multiprocessing as mp
    import sharding_worker
    tests_dir = os.path.dirname(os.path.abspath(__file__))
    pkg_dir = os.path.join(os.path.dirname(tests_dir), "qgemm-perf-framework-ng_b200")
    old = os.environ.get("PYTHONPATH", "")
    os.environ["PYTHONPATH"] = os.pathsep.join([tests_dir, pkg_dir] + ([old] if old else []))
    try:
        mp.start_processes(sharding_worker.gather_gpu_rank_main, args=(2, _free_port(), m, n, k, 128, path),
                           nprocs=2, join=True, start_method="spawn")
    finally:
        os.environ["PYTHONPATH"] = old
