"""Parity on every BASELINE configuration, against the reference's own path (GPU).

The device results come from the library's default path (PFNG_B200_PATH_AUTO:
the decode GEMV for m <= 8, the tensor-core GEMM above) through the C ABI,
with the activations quantized on the device from fp32.  The expected values
come from the reference's scalar llama_reference code compiled in place
(oracle/_ref: quantize_row_q*_ref and dot_*, element-parallel over host
threads, bit-identical to llama_reference::compute), on the same inputs
quantized by the reference's own quantizers.  The bar
every element within
1e-5 * sum_k |d_w q_w d_a q_a| of the reference.

  configs[0] q4_0 x q8_0 480x1536x1536, W and x ~ N(0, 1)     whole C
  configs[1] q4_0 decode 1x4096x4096 + 1x11008x4096            whole C (single and grouped launch)
  configs[2] q4_K x q8_K 480x1536x1536                          whole C
  configs[3] iq2_xxs x q8_K 480x1536x1536, uniform indices      whole C (against the C restatement:
             the reference's decoder has grid entries 0..31 only)
  configs[4] q4_0 M in {32, 512, 2048} x the four Llama-2-7B (N, K), W ~ N(0, 0.02):
             whole C for M <= 512; for M = 2048 the first and last 128-row
             tiles and every 16th row in between.

Integer per-32 partial products of the kernels that run by default (the
direct-operand kernel for q4_0 / q4_K, the overlapped kernel for iq2_xxs,
on 32-, 64- and 128-row tiles, split and unsplit) are compared bit for bit
with the oracle's.
"""
import functools
import os

import numpy as np
import pytest

from oracle_lib import TYPES

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import pfng_b200 as pb  # noqa: E402

TOL = 1e-5
THREADS = os.cpu_count() or 1


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    yield
    pb.check_kernel_error()


def dev(a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def dev_bytes(blocks: np.ndarray):
    return dev(blocks.view(np.uint8).reshape(-1))


def host(t) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def act_kind(wtype):
    return "q8_0" if wtype == "q4_0" else "q8_K"


def iq2_weights(n, k, rng):
    w = np.zeros((n, k // 256), TYPES["iq2_xxs"][0])
    w["d"] = rng.uniform(1e-3, 1e-2, size=w.shape).astype(np.float16).view(np.uint16)
    qs = w["qs"].view(np.uint8).reshape(n, k // 256, 8, 8)
    qs[...] = rng.integers(0, 256, size=qs.shape)  # grid indices, sign fields and scales all uniform
    return w


def check_close(c, ref, bound, what):
    err = np.abs(c.astype(np.float64) - ref.astype(np.float64))
    limit = TOL * bound + 1e-30
    bad = ~(err <= limit)  # NaN fails too
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} elements out of tolerance, " \
                          f"worst {np.nanmax(err / limit):.3g}x the bound"


def q4_0_bound(w: np.ndarray, a: np.ndarray, chunk: int = 8192) -> np.ndarray:
    """sum_k |w_k| |a_k| for q4_0 x q8_0 as a float32 matrix product of the
    dequantized magnitudes (exact per term; the oracle's bound, computed on
    the host's BLAS so that the large configurations stay fast)."""
    aa = (np.abs(a["qs"].astype(np.float32)) *
          np.abs(a["d"].view(np.float16).astype(np.float32))[..., None]).reshape(a.shape[0], -1)
    out = np.empty((a.shape[0], w.shape[0]), np.float64)
    for j0 in range(0, w.shape[0], chunk):
        wb = w[j0:j0 + chunk]
        d = np.abs(wb["d"].view(np.float16).astype(np.float32))
        lo = np.abs((wb["qs"] & 15).astype(np.float32) - 8)
        hi = np.abs((wb["qs"] >> 4).astype(np.float32) - 8)
        ww = (np.concatenate([lo, hi], axis=-1) * d[..., None]).reshape(wb.shape[0], -1)
        out[:, j0:j0 + chunk] = aa @ ww.T
    return out


# ------------------------------------------------- configs[0], [2], [3]
@pytest.mark.parametrize("wtype", ["q4_0", "q4_K", "iq2_xxs"])
def test_480x1536x1536_whole_matrix(oracle, reference, wtype):
    m, n, k = 480, 1536, 1536
    rng = np.random.default_rng({"q4_0": 100, "q4_K": 102, "iq2_xxs": 103}[wtype])
    w = iq2_weights(n, k, rng) if wtype == "iq2_xxs" else \
        reference.quantize(wtype, rng.standard_normal((n, k)).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    a = reference.quantize(act_kind(wtype), x)
    c = host(pb.compute(wtype, dev_bytes(w), dev(x), n))
    # the reference's own iq2_xxs decoder holds only grid entries 0..31
    # (kernels/common/iq2_xxs.h:12-23); full-range indices go through the C
    # restatement, whose 256-entry grid is pinned to the upstream table
    ref = oracle.mm(wtype, w, a, m, n, k) if wtype == "iq2_xxs" else reference.mm_threads(wtype, w, a, m, n, k, THREADS)
    check_close(c, ref, oracle.bound(wtype, w, a, m, n, k), f"{wtype} {m}x{n}x{k}")


# ------------------------------------------------------------ configs[1]
def test_decode_configs_whole_output(oracle, reference):
    rng = np.random.default_rng(101)
    k = 4096
    ws = [reference.quantize("q4_0", rng.standard_normal((n, k)).astype(np.float32)) for n in (4096, 11008)]
    x = rng.standard_normal((1, k)).astype(np.float32)
    a = reference.quantize("q8_0", x)
    wds = [dev_bytes(w) for w in ws]
    grouped = pb.compute_grouped("q4_0", wds, dev(x), [4096, 11008])
    for w, wd, g, n in zip(ws, wds, grouped, (4096, 11008)):
        ref = reference.mm_threads("q4_0", w, a, 1, n, k, THREADS)
        bound = oracle.bound("q4_0", w, a, 1, n, k)
        single = host(pb.compute("q4_0", wd, dev(x), n))
        check_close(single, ref, bound, f"decode 1x{n}x{k}")
        np.testing.assert_array_equal(host(g).view(np.uint32), single.view(np.uint32))


# ------------------------------------------------------------ configs[4]
@functools.lru_cache(maxsize=1)
def llama_weights(n: int, k: int):
    from oracle_lib import reference_or_none
    ref = reference_or_none()
    rng = np.random.default_rng(n * 7 + k)
    wf = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
    return ref.quantize("q4_0", wf)


LLAMA = [(m, n, k) for n, k in ((4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)) for m in (32, 512, 2048)]


@pytest.mark.parametrize("m,n,k", LLAMA)
def test_llama_shapes(reference, m, n, k):
    w = llama_weights(n, k)
    rng = np.random.default_rng(m + n + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    wd = dev_bytes(w)
    c = host(pb.compute("q4_0", wd, dev(x), n))
    if m <= 512:
        rows = np.arange(m)
    else:
        rows = np.unique(np.concatenate([np.arange(128), np.arange(m - 128, m), np.arange(0, m, 16)]))
    a = reference.quantize("q8_0", x[rows])
    ref = reference.mm_threads("q4_0", w, a, len(rows), n, k, THREADS)
    check_close(c[rows], ref, q4_0_bound(w, a), f"q4_0 {m}x{n}x{k} ({len(rows)} rows)")
    # the device's quantized activations are the reference's: the rows not
    # compared above still went through the same kernels; spot-check that the
    # prepared-activation entry points give the same bits as compute
    prep = pb.prepare_activations("q4_0", dev(x))
    c2 = host(pb.mm_prepared("q4_0", wd, prep, m, n, k))
    np.testing.assert_array_equal(c2.view(np.uint32), c.view(np.uint32))


# ------------------------------------- integer partials of the default kernels
@pytest.mark.parametrize("wtype", ["q4_0", "q4_K", "iq2_xxs"])
@pytest.mark.parametrize("m,n,k", [(32, 512, 1024),     # 32-row tiles, split k
                                   (256, 1024, 1024),   # 64-row tiles, split k
                                   (512, 2048, 512),    # 64-row tiles, unsplit (overlapped kernel for iq2_xxs)
                                   (1024, 2048, 256)])  # 128-row tiles
def test_partials_of_default_kernels(oracle, wtype, m, n, k):
    rng = np.random.default_rng(m + 3 * n + k)
    w = iq2_weights(n, k, rng) if wtype == "iq2_xxs" else \
        oracle.quantize(wtype, rng.standard_normal((n, k)).astype(np.float32))
    a = oracle.quantize(act_kind(wtype), rng.standard_normal((m, k)).astype(np.float32))
    got = host(pb.partials(wtype, dev_bytes(w), dev_bytes(a), m, n, k, path="auto"))
    np.testing.assert_array_equal(got, oracle.partials(wtype, w, a, m, n, k))
