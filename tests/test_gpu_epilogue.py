"""Output formats of the matmul (fused epilogue), on the GPU, through the C ABI.

pfng_b200_compute_out / pfng_b200_mm_out write the result as fp16, bf16 or
q8_0 blocks along n.  Each must be exactly the conversion of the fp32 C the
same path computes (pfng_b200_compute_* / pfng_b200_mm_*, itself checked
against the oracle in test_gpu_parity.py):
  * q8_0: byte-identical to the oracle's quantize_row_q8_0 restatement of the
    reference (llama_reference.cpp:38-52) applied to that fp32 C;
  * fp16: numpy's IEEE round-to-nearest-even conversion of that C;
  * bf16: round-to-nearest-even of the fp32 bit pattern (restated below).
"""
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


def bf16_rne(c: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even (finite inputs)."""
    u = c.astype(np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def expected(oracle, fmt: str, c: np.ndarray) -> bytes:
    if fmt == "f16":
        return c.astype(np.float16).tobytes()
    if fmt == "bf16":
        return bf16_rne(c).tobytes()
    return oracle.quantize("q8_0", c).tobytes()


def got_bytes(t) -> bytes:
    torch.cuda.synchronize()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().tobytes()
    return t.cpu().numpy().tobytes()


CASES = [
    # (wtype, path, m, n, k)
    ("q4_0", "gemv", 1, 256, 1024), ("q4_0", "gemv", 3, 96, 512), ("q4_0", "mma", 130, 320, 1536),
    ("q4_0", "mma", 480, 1536, 1536), ("q4_0", "mma", 9, 64, 256), ("q4_0", "simple", 5, 64, 96),
    ("q4_K", "gemv", 1, 128, 1536), ("q4_K", "mma", 140, 256, 1536), ("iq2_xxs", "mma", 70, 192, 512),
    ("iq2_xxs", "simple", 3, 32, 256), ("q4_0_planar", "mma", 200, 384, 2048), ("q4_0_planar", "gemv", 2, 160, 4096),
]


@pytest.mark.parametrize("fmt", ["f16", "bf16", "q8_0"])
@pytest.mark.parametrize("wtype,path,m,n,k", CASES)
def test_output_format_is_conversion_of_fp32(oracle, wtype, path, m, n, k, fmt):
    rng = np.random.default_rng(m * 131 + n + k)
    base = "q4_0" if wtype == "q4_0_planar" else wtype
    w = make_weights(oracle, base, n, k, rng)
    wd = dev_bytes(w)
    if wtype == "q4_0_planar":
        wd = pb.pack_q4_0_planar(wd, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    xd = dev(x)
    c32 = host(pb.compute(wtype, wd, xd, n, path=path))
    out = pb.compute_out(wtype, wd, xd, n, fmt, path=path)
    assert got_bytes(out) == expected(oracle, fmt, c32), f"{wtype}/{path}/{m}x{n}x{k}/{fmt}"
    # quantized activations in (mm_out): same bytes
    a = oracle.quantize(act_kind(base), x)
    out2 = pb.mm_out(wtype, wd, dev_bytes(a), m, n, k, fmt, path=path)
    assert got_bytes(out2) == got_bytes(out)


@pytest.mark.parametrize("path", ["gemv", "mma"])
def test_output_strides_leave_padding(oracle, path):
    m, n, k = (4, 64, 512) if path == "gemv" else (100, 128, 512)
    rng = np.random.default_rng(9)
    w = make_weights(oracle, "q4_0", n, k, rng)
    wd, xd = dev_bytes(w), dev(rng.standard_normal((m, k)).astype(np.float32))
    c32 = host(pb.compute("q4_0", wd, xd, n, path=path))
    big = torch.full((m, n + 8), -3.0, dtype=torch.float16, device="cuda")
    pb.compute_out("q4_0", wd, xd, n, "f16", out=big[:, :n], path=path)
    hb = host(big)
    assert np.all(hb[:, n:] == -3.0)
    assert hb[:, :n].tobytes() == c32.astype(np.float16).tobytes()
    # q8_0 rows ldo blocks apart: rows of n / 32 blocks, then untouched padding
    ldo = n // 32 + 3
    qb = torch.full((m * ldo * 34,), 0x5A, dtype=torch.uint8, device="cuda")
    st = pb.lib().pfng_b200_compute_out(0, wd.data_ptr(), xd.data_ptr(), k, qb.data_ptr(), pb.OUT_Q8_0, ldo, m, n, k,
                                        None, 0, pb.PATHS[path], pb._stream(None))
    if st == -4:  # this path needs its fp32 scratch
        wsz = pb.lib().pfng_b200_compute_out_workspace_size(0, pb.OUT_Q8_0, m, n, k, pb.PATHS[path])
        ws = torch.empty(wsz, dtype=torch.uint8, device="cuda")
        st = pb.lib().pfng_b200_compute_out(0, wd.data_ptr(), xd.data_ptr(), k, qb.data_ptr(), pb.OUT_Q8_0, ldo, m,
                                            n, k, ws.data_ptr(), wsz, pb.PATHS[path], pb._stream(None))
    assert st == 0
    rows = host(qb).reshape(m, ldo * 34)
    assert rows[:, : n // 32 * 34].tobytes() == oracle.quantize("q8_0", c32).tobytes()
    assert np.all(rows[:, n // 32 * 34:] == 0x5A)


def test_output_format_rejections():
    w = torch.zeros(18 * 8 * 48, dtype=torch.uint8, device="cuda")
    x = torch.zeros((2, 256), device="cuda")
    with pytest.raises(pb.PfngError) as e:
        pb.compute_out("q4_0", w, x, 48, "q8_0")  # n % 32 != 0
    assert e.value.status == -2
    with pytest.raises(pb.PfngError) as e:
        pb.compute_out("q4_0", w, x, 48, 7, out=torch.empty((2, 48), device="cuda"))  # unknown format
    assert e.value.status == -1
