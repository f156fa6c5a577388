"""q4_0 weights in the planar row layout, on the GPU, through the C ABI.

The planar layout is this library's repacked W (pfng_b200_pack_q4_0_planar):
the device repack must be the oracle's byte permutation, unpacking must give
the ggml bytes back, and every kernel path must compute on planar W what the
oracle computes on the ggml-layout W:
  * integer per-32 partials bit-exact;
  * fp32 within 1e-5 * sum_k |w_k a_k| per element;
  * the SIMPLE path bit-identical to the reference's operation order.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import pfng_b200 as pb  # noqa: E402
from test_gpu_parity import check_close, dev, dev_bytes, host  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    yield
    pb.check_kernel_error()


def planar_weights(oracle, n, k, seed):
    rng = np.random.default_rng(seed)
    w = oracle.quantize("q4_0", rng.standard_normal((n, k)).astype(np.float32))
    wd = dev_bytes(w)
    wp = pb.pack_q4_0_planar(wd, n, k)
    return w, wd, wp, rng


@pytest.mark.parametrize("n,k", [(1, 256), (37, 1536), (300, 4096), (64, 11008)])
def test_pack_is_the_oracle_permutation(oracle, n, k):
    w, wd, wp, _ = planar_weights(oracle, n, k, n + k)
    got = host(wp).reshape(n, -1)
    np.testing.assert_array_equal(got, oracle.pack_q4_0_planar(w, n, k))
    back = host(pb.unpack_q4_0_planar(wp, n, k))
    assert back.tobytes() == w.tobytes()
    assert oracle.unpack_q4_0_planar(got, n, k).tobytes() == w.tobytes()


CASES = [
    # (path, m, n, k)
    ("gemv", 1, 300, 256), ("gemv", 1, 257, 1536), ("gemv", 1, 130, 4096), ("gemv", 1, 64, 11008),
    ("gemv", 2, 100, 1024), ("gemv", 5, 77, 4096), ("gemv", 8, 64, 2048),
    ("mma", 9, 129, 256), ("mma", 130, 300, 1536), ("mma", 256, 256, 4096),
    ("simple", 5, 17, 256), ("simple", 33, 40, 512),
]


@pytest.mark.parametrize("path,m,n,k", CASES)
def test_planar_partials_bitexact(oracle, path, m, n, k):
    w, _, wp, rng = planar_weights(oracle, n, k, m * 7 + n + k)
    a = oracle.quantize("q8_0", rng.standard_normal((m, k)).astype(np.float32))
    got = host(pb.partials("q4_0_planar", wp, dev_bytes(a), m, n, k, path=path))
    np.testing.assert_array_equal(got, oracle.partials("q4_0", w, a, m, n, k))


@pytest.mark.parametrize("path,m,n,k", CASES)
def test_planar_mm_parity(oracle, path, m, n, k):
    w, wd, wp, rng = planar_weights(oracle, n, k, m * 1000 + n + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    a = oracle.quantize("q8_0", x)
    ref = oracle.mm("q4_0", w, a, m, n, k)
    c = host(pb.mm("q4_0_planar", wp, dev_bytes(a), m, n, k, path=path))
    if path == "simple":
        np.testing.assert_array_equal(c.view(np.uint32), ref.view(np.uint32))
    else:
        check_close(c, ref, oracle.bound("q4_0", w, a, m, n, k), f"planar/{path}/{m}x{n}x{k}")
    # fused fp32 entry: same bits as mm on the quantized rows
    c2 = host(pb.compute("q4_0_planar", wp, dev(x), n, path=path))
    np.testing.assert_array_equal(c2.view(np.uint32), c.view(np.uint32))
    if path == "mma":
        # the GEMM folds the same sub-block sums in the same order for both layouts
        c_raw = host(pb.compute("q4_0", wd, dev(x), n, path=path))
        np.testing.assert_array_equal(c2.view(np.uint32), c_raw.view(np.uint32))


@pytest.mark.parametrize("m", [1, 4])
def test_planar_grouped_matches_single(oracle, m):
    k, ns = 4096, [4096, 1000, 256]
    rng = np.random.default_rng(5 + m)
    ws = [oracle.quantize("q4_0", rng.standard_normal((n, k)).astype(np.float32)) for n in ns]
    wps = [pb.pack_q4_0_planar(dev_bytes(w), n, k) for w, n in zip(ws, ns)]
    x = rng.standard_normal((m, k)).astype(np.float32)
    xd = dev(x)
    a = oracle.quantize("q8_0", x)
    for overlap in (False, True):
        outs = pb.compute_grouped("q4_0_planar", wps, xd, ns, overlap_weights=overlap)
        for w, wp, n, o in zip(ws, wps, ns, outs):
            single = host(pb.compute("q4_0_planar", wp, xd, n, path="gemv"))
            got = host(o)
            np.testing.assert_array_equal(got.view(np.uint32), single.view(np.uint32))
            check_close(got, oracle.mm("q4_0", w, a, m, n, k), oracle.bound("q4_0", w, a, m, n, k), "grouped")


@pytest.mark.parametrize("n", [4096, 11008])
def test_planar_decode_full_size(oracle, n):
    # the decode configurations (m = 1, k = 4096): GEMV on planar W against
    # the bit-exact simple path on the ggml W, plus exact oracle partials
    k = 4096
    w, wd, wp, rng = planar_weights(oracle, n, k, n)
    x = rng.standard_normal((1, k)).astype(np.float32)
    a = oracle.quantize("q8_0", x)
    c = host(pb.compute("q4_0_planar", wp, dev(x), n))
    c_simple = host(pb.compute("q4_0", wd, dev(x), n, path="simple"))
    ref = oracle.mm("q4_0", w, a, 1, n, k)
    np.testing.assert_array_equal(c_simple.view(np.uint32), ref.view(np.uint32))
    check_close(c, ref, oracle.bound("q4_0", w, a, 1, n, k), f"planar decode n={n}")
    got = host(pb.partials("q4_0_planar", wp, dev_bytes(a), 1, n, k))
    np.testing.assert_array_equal(got, oracle.partials("q4_0", w, a, 1, n, k))


def test_planar_rejections():
    wp = torch.zeros(18 * 8 * 64, dtype=torch.uint8, device="cuda")
    x = torch.zeros((1, 256), device="cuda")
    with pytest.raises(pb.PfngError) as e:
        pb.compute("q4_0_planar", wp, torch.zeros((1, 96), device="cuda"), 8)  # k % 256 != 0
    assert e.value.status == -2
    with pytest.raises(pb.PfngError) as e:
        pb.compute("q4_0_planar", wp[2:], x, 8)  # planar W must be 16-byte aligned
    assert e.value.status == -3
    with pytest.raises(pb.PfngError) as e:
        pb.pack_q4_0_planar(wp, 8, 256, out=wp)  # overlapping buffers
    assert e.value.status == -1
